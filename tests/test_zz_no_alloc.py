"""santa_decode_static_scratch: the decode entry point for callers that cannot
allocate device memory (a serving stack whose memory manager owns all of the
GPU's memory, a plugin host that forbids device allocations after start-up, a
decode loop that cannot take cudaMalloc's implicit synchronisation).

It is called here through the C ABI with plain pointers and must give the same
results as santa_decode with a caller-allocated workspace, on two calls in a
row (the second call reuses the shared scratch the first one left behind).
This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from santapp_b200 import _lib
from santapp_b200.attention import santapp as S
from santapp_b200.synthetic import QWEN7B_32K, make_decode_workload, scaled_shape

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

SHAPE = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx2048-b2", batch=2, context=2048,
                     true_clusters=32, n_clusters=32, topk_clusters=4, samples=64, steps=2)
MAX_ABS, MEAN_ABS = 2e-2, 2e-3  # bf16 K/V tolerance used by the decode parity tests


@pytest.fixture(scope="module")
def case():
    w = make_decode_workload(SHAPE, seed=5)
    kc, vc = w.keys.cuda().contiguous(), w.values.cuda().contiguous()
    summ = S.build_summary(kc, vc, w.labels[:, :, :SHAPE.sample_end].cuda(), SHAPE.n_clusters,
                           sample_end=SHAPE.sample_end, n_total=SHAPE.context)
    return w, kc, vc, summ


def _static_call(q, kc, vc, summ, step):
    """One decode step through the C ABI entry point, no workspace passed."""
    lib = _lib.load()
    B, Hq, D = q.shape
    geo = _lib.SantaGeometry(B, SHAPE.num_kv_heads, Hq // SHAPE.num_kv_heads, D, kc.shape[2],
                             SHAPE.context, SHAPE.sample_end, _lib.DTYPE_BF16)
    p = S.decode_params("hybrid", topk_clusters=SHAPE.topk_clusters, samples=SHAPE.samples,
                        scale=SHAPE.scale, seed=9, step=step)
    out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
    n_exact = torch.empty(B, Hq, dtype=torch.int32, device=q.device)
    ess = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
    c = summ.as_c()
    st = lib.santa_decode_static_scratch(
        ctypes.byref(geo), ctypes.byref(p), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
        ctypes.byref(c), None, None, out.data_ptr(), lse.data_ptr(), n_exact.data_ptr(),
        ess.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.SANTA_OK, lib.santa_status_string(st)
    return out, lse, n_exact, ess


def test_static_scratch_matches_santa_decode_on_two_calls(case):
    w, kc, vc, summ = case
    for step in range(2):  # the second call runs on the scratch the first one left
        q = w.queries[step].cuda().contiguous()
        out, lse, n_exact, ess = _static_call(q, kc, vc, summ, step)
        ref = S.santa_decode(q, kc, vc, summ, mode="hybrid", n_total=SHAPE.context,
                             topk_clusters=SHAPE.topk_clusters, samples=SHAPE.samples,
                             seed=9, step=step, with_stats=True)
        torch.cuda.synchronize()
        err = (out - ref.out).abs()
        assert err.max().item() < MAX_ABS and err.mean().item() < MEAN_ABS
        assert (lse - ref.lse).abs().max().item() < 1e-3
        assert torch.equal(n_exact, ref.n_exact)
        assert (ess - ref.ess).abs().max().item() < 1e-3
        assert torch.isfinite(out).all()


def test_static_scratch_refuses_geometries_beyond_its_size(case):
    _, kc, vc, summ = case
    lib = _lib.load()
    # a 128K-token context for 16 x 8 KV heads needs far more than the fixed array
    geo = _lib.SantaGeometry(16, 8, 4, 128, 131072, 131072, 131008, _lib.DTYPE_BF16)
    p = S.decode_params("hybrid", topk_clusters=32, samples=512, scale=0.088)
    need = ctypes.c_size_t()
    assert lib.santa_decode_workspace_bytes(ctypes.byref(geo), ctypes.byref(p), 1024,
                                            ctypes.byref(need)) == 0
    assert need.value > 16 << 20
    big = _lib.SantaSummary(*([summ.members.data_ptr()] * 9), 1024)
    st = lib.santa_decode_static_scratch(ctypes.byref(geo), ctypes.byref(p), kc.data_ptr(),
                                         kc.data_ptr(), vc.data_ptr(), ctypes.byref(big), None,
                                         None, kc.data_ptr(), None, None, None,
                                         torch.cuda.current_stream().cuda_stream)
    assert st == _lib.SANTA_ERR_WORKSPACE
