"""Paged KV cache: every kernel that reads the cache through the block table
gives results bit-identical to the contiguous cache holding the same tokens.

The contiguous path is checked against the oracle in test_decode_gpu.py; here
the same workloads are moved into page pools whose pages are handed out in a
seeded random order, with the pool's unused pages filled with NaN (a read
through a wrong page would turn outputs into NaN or change them), and the
summary fields, selections, sample rows and decode outputs of every mode must
be equal bit for bit.  One case per path: fp32 head_dim 64 (the SIMT gather
path) and bf16 head_dim 128 (the warp-tiled gather kernel), at page sizes
that split the recent window across pages.
"""
import math

import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention import santapp as S
from santapp_b200.attention.paged import PagedKVCache
from santapp_b200.synthetic import QWEN05B_4K, QWEN7B_32K, make_decode_workload, scaled_shape

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

QWEN7B_SMALL = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx2048-b3", batch=3,
                            context=2048, true_clusters=32, n_clusters=32,
                            topk_clusters=4, samples=64, steps=1)
SHAPES = {"fp32_d64": QWEN05B_4K, "bf16_d128": QWEN7B_SMALL}
SUMMARY_FIELDS = ("members", "positions", "starts", "lengths_long", "log_n", "key_centroids",
                  "n_groups", "sorted_key", "sorted_value")


def _paged(kc, vc, n_total, page_size, seed=1):
    """Pages for tokens [0, n_total) in a random page order, with spare pages
    full of NaN."""
    B, Hkv, cap, D = kc.shape
    need = B * -(-cap // page_size)
    cache = PagedKVCache.from_contiguous(kc, vc, length=n_total, page_size=page_size,
                                         num_pages=need + 7, page_order_seed=seed)
    used = torch.zeros(cache.num_pages, dtype=torch.bool, device=kc.device)
    t = cache.block_table.long()
    used[t[t >= 0]] = True
    cache.key_pool[~used] = float("nan")
    cache.value_pool[~used] = float("nan")
    return cache


def _setup(name, page_size):
    sh = SHAPES[name]
    w = make_decode_workload(sh)
    kc, vc = w.keys.cuda().contiguous(), w.values.cuda().contiguous()
    n_total = sh.context - 5          # the recent window ends inside a page
    se = sh.sample_end
    labels = w.labels[:, :, :se].to(torch.int32).cuda()
    contig = S.build_summary(kc, vc, labels, sh.n_clusters, sample_end=se, n_total=n_total)
    cache = _paged(kc, vc, n_total, page_size)
    paged = S.build_summary(cache, None, labels, sh.n_clusters, sample_end=se, n_total=n_total)
    torch.cuda.synchronize()
    return sh, w, kc, vc, n_total, contig, cache, paged


def _mode_kwargs(sh, mode):
    if mode == "topk":
        return dict(token_budget=4 * sh.samples)
    if mode == "hybrid":
        return dict(topk_clusters=sh.topk_clusters, samples=sh.samples)
    return dict(samples=sh.samples)


@pytest.mark.parametrize("name,page_size", [("fp32_d64", 16), ("fp32_d64", 256),
                                            ("bf16_d128", 32), ("bf16_d128", 128)])
def test_paged_summary_and_every_mode_bit_identical(name, page_size):
    sh, w, kc, vc, n_total, contig, cache, paged = _setup(name, page_size)
    for f in SUMMARY_FIELDS:
        a, b = getattr(contig, f), getattr(paged, f)
        assert torch.equal(a, b), f"summary field {f} differs (page_size {page_size})"
    q = w.queries[0].cuda().contiguous()
    for mode in ("topk", "guided", "uniform", "santa", "hybrid"):
        kw = dict(mode=mode, n_total=n_total, seed=77, step=3, with_stats=True,
                  **_mode_kwargs(sh, mode))
        a = S.santa_decode(q, kc, vc, contig, **kw)
        b = S.santa_decode(q, cache, None, paged, **kw)
        torch.cuda.synchronize()
        assert torch.isfinite(b.out).all(), mode
        assert torch.equal(a.out, b.out), mode
        assert torch.equal(a.lse, b.lse), mode
        assert torch.equal(a.n_exact, b.n_exact), mode
        assert torch.equal(a.ess, b.ess), mode
        kw.pop("with_stats")
        sa = S.santa_decode_select(q, kc, vc, contig, **kw)
        sb = S.santa_decode_select(q, cache, None, paged, **kw)
        for x, y in zip(sa, sb):
            assert torch.equal(x, y), mode


def test_paged_decode_step_matches_and_against_oracle():
    """DecodeStep (plan + execute) over pages equals the contiguous call, and
    the hybrid output stays within the stated bf16 tolerance of the oracle."""
    sh, w, kc, vc, n_total, contig, cache, paged = _setup("bf16_d128", 64)
    q = w.queries[0].cuda().contiguous()
    kw = dict(num_query_heads=sh.num_query_heads, mode="hybrid", n_total=n_total,
              topk_clusters=sh.topk_clusters, samples=sh.samples, seed=5)
    step_c = S.DecodeStep(kc, vc, contig, **kw)
    step_p = S.DecodeStep(cache, None, paged, **kw)
    a = step_c(q, step=2).clone()
    b = step_p(q, step=2).clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    se, scale = sh.sample_end, 1.0 / math.sqrt(sh.head_dim)
    errs = []
    for bb in range(sh.batch):
        for kv in range(sh.num_kv_heads):
            K = w.keys[bb, kv, :n_total].float().numpy()
            V = w.values[bb, kv, :n_total].float().numpy()
            o = O.build_summary(K[:se], w.labels[bb, kv, :se].numpy().astype(np.int64),
                                sh.n_clusters)
            for h in range(kv * sh.group, (kv + 1) * sh.group):
                qh = w.queries[0, bb, h].numpy()
                chosen = O.select_topk(O.centroid_guess(o, qh, scale), sh.topk_clusters)
                n_rest = se - int(o.lengths[chosen].sum())
                ranks = O.philox_ranks(5, 2, bb, h, sh.samples, n_rest)
                ref = O.decode_hybrid(qh, K, V, o, se, sh.topk_clusters, ranks, scale)
                errs.append(np.abs(b[bb, h].cpu().numpy() - ref.out))
    e = np.stack(errs)
    assert e.max() < 2e-2 and e.mean() < 2e-3, (e.max(), e.mean())


def test_paged_rope_append_matches_contiguous():
    """santa_rope_append_paged writes the same rotated keys and values as the
    contiguous append, across page boundaries and into pages mapped on demand;
    pages of other sequences and spare pages stay untouched."""
    from santapp_b200 import _lib
    torch.manual_seed(0)
    B, Hq, Hkv, D, cap, page = 3, 28, 4, 128, 1000, 64
    dev = torch.device("cuda")
    kc = torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    cache = PagedKVCache.allocate(B, Hkv, D, max_tokens=cap, page_size=page,
                                  num_pages=B * 16 + 3, page_order_seed=4)
    cache.key_pool.fill_(float("nan"))
    cache.value_pool.fill_(float("nan"))
    lib = _lib.load()
    pos = 0
    for T in (300, 1, 37, 1, 90):      # a prompt, then decode steps and a chunk
        q = torch.randn(B, T, Hq, D, device=dev).to(torch.bfloat16)
        k = torch.randn(B, T, Hkv, D, device=dev).to(torch.bfloat16)
        v = torch.randn(B, T, Hkv, D, device=dev).to(torch.bfloat16)
        ang = torch.arange(pos, pos + T, device=dev)[:, None] * torch.linspace(
            0.01, 1.0, D, device=dev)[None]
        cos = ang.cos().to(torch.bfloat16)[None].expand(B, T, D).contiguous()
        sin = ang.sin().to(torch.bfloat16)[None].expand(B, T, D).contiguous()
        qa = torch.empty(B, Hq, T, D, dtype=torch.float32, device=dev)
        qb = torch.empty_like(qa)
        _lib.check("santa_rope_append", lib.santa_rope_append(
            B, T, Hq, Hkv, D, q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(),
            sin.data_ptr(), kc.data_ptr(), vc.data_ptr(), cap, pos, None, qa.data_ptr(), None))
        cache.append(q, k, v, cos, sin, pos, q_rot_f32=qb)
        pos += T
        torch.cuda.synchronize()
        assert torch.equal(qa, qb)
        kp, vp = cache.to_contiguous(pos)
        assert torch.equal(kp, kc[:, :, :pos]) and torch.equal(vp, vc[:, :, :pos])
    # every page not mapped by the table is still all NaN
    t = cache.block_table.long()
    used = torch.zeros(cache.num_pages, dtype=torch.bool, device=dev)
    used[t[t >= 0]] = True
    assert int(used.sum()) == B * -(-pos // page)
    assert torch.isnan(cache.key_pool[~used].float()).all()
    assert torch.isnan(cache.value_pool[~used].float()).all()
    # the mapped slots past the last token were not written either
    last = cache.key_pool[t[:, (pos - 1) // page]][:, :, (pos % page):]
    assert torch.isnan(last.float()).all()


def test_paged_prefill_bit_identical():
    """santa_prefill over page pools (random page order, NaN spare pages)
    equals the contiguous-cache prefill bit for bit, output and LSE."""
    from santapp_b200.attention.prefill import santa_prefill
    torch.manual_seed(3)
    B, Hq, Hkv, D, T = 2, 8, 2, 128, 1000
    dev = torch.device("cuda")
    q = torch.randn(B, Hq, T, D, device=dev).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, T + 24, D, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    cache = _paged(kc, vc, T, 64, seed=9)
    a, la = santa_prefill(q, kc, vc, causal=True, return_lse=True)
    b, lb = santa_prefill(q, cache, None, causal=True, return_lse=True)
    torch.cuda.synchronize()
    assert int(a._santa_error_flag.item()) == 0 and int(b._santa_error_flag.item()) == 0
    assert torch.isfinite(b.float()).all()
    assert torch.equal(a, b) and torch.equal(la, lb)
