"""GraphedDecodeStep: a decode step captured once in a CUDA graph with its
host transfers (queries in from pinned memory, output out) and the Philox
step counter read from a device word.  Every replay must equal the plain
DecodeStep call of the same step bit for bit, and different steps must draw
different samples."""
import pytest
import torch

from santapp_b200.attention import santapp as S
from santapp_b200.synthetic import QWEN7B_32K, make_decode_workload, scaled_shape

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

SHAPE = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx4096-b2", batch=2, context=4096,
                     true_clusters=64, n_clusters=64, topk_clusters=8, samples=128, steps=4)


def test_graphed_step_replays_match_the_api_call():
    sh = SHAPE
    w = make_decode_workload(sh)
    kc, vc = w.keys.cuda(), w.values.cuda()
    labels = w.labels[:, :, :sh.sample_end].to(torch.int32).cuda()
    summ = S.build_summary(kc, vc, labels, sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    kw = dict(num_query_heads=sh.num_query_heads, mode="hybrid", n_total=sh.context,
              topk_clusters=sh.topk_clusters, samples=sh.samples, seed=11)
    plain = S.DecodeStep(kc, vc, summ, **kw)
    want = [plain(w.queries[i].cuda().contiguous(), step=100 + i).clone() for i in range(4)]
    torch.cuda.synchronize()
    q_host = torch.empty(tuple(w.queries[0].shape), dtype=torch.float32).pin_memory()
    out_host = torch.empty_like(q_host).pin_memory()
    g = S.DecodeStep(kc, vc, summ, **kw).graphed(q_host, out_host)
    for i in (2, 0, 3, 1):
        q_host.copy_(w.queries[i])
        g.run(100 + i)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(out_host, want[i].cpu()), i
    # the counter moves the draws: steps 100 and 101 on the same queries differ
    q_host.copy_(w.queries[0])
    g.run(101)
    torch.cuda.current_stream().synchronize()
    assert not torch.equal(out_host, want[0].cpu())
