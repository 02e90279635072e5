"""Fingerprints: probe positions on CPU; the CUDA features bit-exact against
the oracle and within 1e-4 of the reference's formula in fp32 torch."""
import math

import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention.fingerprints import build_fingerprints, cluster_count, probe_positions


def test_probe_strategies():
    p = probe_positions("end_quarter", 4096, 64, probe_seed=3)
    assert p.size == 64 and np.all(np.diff(p) > 0) and p[0] >= 3072 and p[-1] < 4095
    assert np.array_equal(p, probe_positions("end_quarter", 4096, 64, probe_seed=3))
    assert not np.array_equal(p, probe_positions("end_quarter", 4096, 64, probe_seed=4))
    assert np.array_equal(probe_positions("start", 100, 8), np.arange(8))
    assert np.array_equal(probe_positions("end", 100, 8), np.arange(91, 99))
    assert np.array_equal(probe_positions("middle", 101, 8), np.arange(46, 54))
    r = probe_positions("random", 500, 16, probe_seed=1)
    assert r.size == 16 and np.all(np.diff(r) > 0) and r[-1] < 499
    with pytest.raises(ValueError):
        probe_positions("end_quarter", 100, 64)
    with pytest.raises(ValueError):
        probe_positions("sideways", 100, 4)


def test_cluster_count():
    assert cluster_count(4000, 16) == 250 and cluster_count(10, 16) == 2 and cluster_count(1, 16) == 1


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
@pytest.mark.parametrize("dtype,N,D,g,P", [(torch.bfloat16, 3000, 128, 7, 64),
                                           (torch.float32, 777, 64, 4, 10)])
def test_fingerprints_bit_exact_and_close_to_reference(dtype, N, D, g, P):
    rs = np.random.RandomState(N)
    T = N + 100
    keys = torch.from_numpy(rs.randn(N, D).astype(np.float32)).to(dtype)
    q = torch.from_numpy(rs.randn(2 * g, T, D).astype(np.float32))
    probes = np.sort(rs.choice(T, P, replace=False))
    f = build_fingerprints(keys.cuda(), q.cuda(), 1, g, probes)
    torch.cuda.synchronize()
    ref = O.fingerprints(keys.float().numpy(), q[g:2 * g].numpy(), probes)
    assert np.array_equal(f.cpu().numpy(), ref)
    # the reference's own formula (santapp.py:672-691) in fp32 torch
    kf = keys.float()
    raw = torch.cat([kf @ q[h, probes].T / math.sqrt(D) for h in range(g, 2 * g)], dim=1)
    z = (raw - raw.mean(dim=0, keepdim=True)) / (raw.std(dim=0, keepdim=True, unbiased=False)
                                                 + 1e-6)
    assert (f.cpu() - z).abs().max().item() < 1e-4
    raw_dev = build_fingerprints(keys.cuda(), q.cuda(), 1, g, probes, normalize=False)
    assert (raw_dev.cpu() - raw).abs().max().item() < 1e-4
