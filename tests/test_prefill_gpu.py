"""tcgen05 causal prefill against an fp32 PyTorch reference of the same op
(and the float64 oracle on a small case).  Tolerance: max-abs 2e-2,
mean-abs 2e-3 (bf16 inputs and output, P rounded to bf16)."""
import math

import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention.prefill import santa_prefill

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _inputs(B, Hq, Hkv, T, D=128, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, generator=g).to(torch.bfloat16)
    return q.cuda(), k.cuda(), v.cuda()


def _reference(q, k, v, causal):
    g = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(q.float(), kf, vf, is_causal=causal)


def _check(out, ref, tol=(2e-2, 2e-3)):
    e = (out.float() - ref).abs()
    assert torch.isfinite(out.float()).all()
    assert e.max().item() < tol[0] and e.mean().item() < tol[1], (e.max().item(), e.mean().item())


def test_single_tile_single_head():
    q, k, v = _inputs(1, 1, 1, 128)
    out = santa_prefill(q, k, v)
    torch.cuda.synchronize()
    assert int(out._santa_error_flag.item()) == 0
    _check(out, _reference(q, k, v, True))


@pytest.mark.parametrize("B,Hq,Hkv,T,causal", [
    (1, 7, 1, 640, True),     # GQA 7, several tiles
    (2, 4, 2, 1000, True),    # ragged last tile (T % 128 != 0)
    (1, 7, 1, 701, True),     # T % 8 != 0: padded V^T rows
    (1, 2, 1, 384, False),    # non-causal
])
def test_prefill_matches_fp32_reference(B, Hq, Hkv, T, causal):
    q, k, v = _inputs(B, Hq, Hkv, T, seed=T)
    out, lse = santa_prefill(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert int(out._santa_error_flag.item()) == 0
    _check(out, _reference(q, k, v, causal))
    # lse against the fp32 reference's log-sum-exp
    g = Hq // Hkv
    s = torch.einsum("bhtd,bhsd->bhts", q.float(), k.float().repeat_interleave(g, dim=1))
    s = s / math.sqrt(128)
    if causal:
        s = s.masked_fill(torch.ones(T, T, device="cuda", dtype=torch.bool).triu(1), -math.inf)
    assert (lse - torch.logsumexp(s, dim=-1)).abs().max().item() < 2e-2


def test_prefill_matches_oracle_small():
    q, k, v = _inputs(1, 2, 1, 256, seed=3)
    out = santa_prefill(q, k, v).float().cpu().numpy()
    ref = O.prefill_causal(q[0].float().cpu().numpy(), k[0].float().cpu().numpy(),
                           v[0].float().cpu().numpy(), 1.0 / math.sqrt(128))
    e = np.abs(out[0] - ref)
    assert e.max() < 2e-2 and e.mean() < 2e-3


def test_prefill_full_qwen7b_layer_32k_strided_rows():
    """The Qwen2.5-7B prefill layer at full size ([1, 28, 32768, 128] bf16, 4
    KV heads, causal; keys from the decode workloads' Gaussian mixture): a
    strided subset of query rows (every tile position class and the last
    row) against the fp32 reference of the same op, max-abs 2e-2 and
    mean-abs 2e-3."""
    from santapp_b200.synthetic import QWEN7B_32K, make_decode_workload, scaled_shape
    T, Hq, Hkv, D = 32768, 28, 4, 128
    w = make_decode_workload(scaled_shape(QWEN7B_32K, batch=1, steps=1, context=T), seed=2,
                             device="cuda")
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(1, Hq, T, D, device="cuda", generator=g).to(torch.bfloat16)
    k, v = w.keys, w.values
    out = santa_prefill(q, k, v)
    torch.cuda.synchronize()
    assert int(out._santa_error_flag.item()) == 0
    rows = torch.cat([torch.arange(0, T, 257, device="cuda"),
                      torch.tensor([127, 128, 255, T - 129, T - 2, T - 1], device="cuda")])
    rows = torch.unique(rows)
    gsz = Hq // Hkv
    errs = []
    for kv in range(Hkv):
        kf = k[0, kv].float()
        vf = v[0, kv].float()
        qh = q[0, kv * gsz:(kv + 1) * gsz][:, rows].float()       # [g, R, D]
        s = torch.einsum("hrd,td->hrt", qh, kf) / math.sqrt(D)
        s = s.masked_fill(torch.arange(T, device="cuda")[None, None, :] > rows[None, :, None],
                          -math.inf)
        ref = torch.einsum("hrt,td->hrd", torch.softmax(s, dim=-1), vf)
        errs.append((out[0, kv * gsz:(kv + 1) * gsz][:, rows].float() - ref).abs())
        del s
    e = torch.cat(errs)
    assert torch.isfinite(e).all()
    assert e.max().item() < 2e-2 and e.mean().item() < 2e-3, (e.max().item(), e.mean().item())


def test_prefill_rows_with_diverging_maxima():
    """Rows of one warp whose running maxima grow at different key tiles: a
    key planted 300 positions before every third query row (6x that row's
    query) lifts only that row's maximum by far more than the lazy-rescale
    threshold, at a later key tile than its neighbours' maxima settle.  The
    rescale of O is warp-collective in the kernel; the result must match the
    fp32 reference and the kernel's bounded waits must not give up."""
    B, Hq, Hkv, T = 1, 7, 1, 1024
    g = torch.Generator(device="cpu").manual_seed(21)
    q = torch.randn(B, Hq, T, 128, generator=g)
    k = 0.1 * torch.randn(B, Hkv, T, 128, generator=g)
    v = torch.randn(B, Hkv, T, 128, generator=g)
    for r in range(400, T, 3):
        k[0, 0, r - 300] = 6.0 * q[0, 0, r] / q[0, 0, r].norm() * 4.0
    q, k, v = (t.to(torch.bfloat16).cuda() for t in (q, k, v))
    out = santa_prefill(q, k, v)
    torch.cuda.synchronize()
    assert int(out._santa_error_flag.item()) == 0
    _check(out, _reference(q, k, v, True))
