"""MiniBatchKMeans on the GPU against the oracle and the reference's golden fits.

Bit-exact: labels, cluster centres, counts, step counts and the fixed-point
inertia (the oracle's definition); the reference's own reported inertia is
matched to 1e-5 relative (its fp32 reduction order, see test_oracle_golden).
"""
import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention.kmeans import SklearnLikeTorchMiniBatchKMeans, gpu_minibatch_labels
from santapp_b200.synthetic import QWEN05B_4K, QWEN7B_32K, make_decode_workload, scaled_shape
from santapp_b200 import _lib

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)


def _parse(case):
    src, kv, k, bs, it, s = case.split("_")
    return src, int(kv[2:]), int(k[1:]), int(bs[2:]), int(it[2:]), int(s[1:])


@pytest.fixture(scope="module")
def workloads():
    return {"qwen05b": make_decode_workload(QWEN05B_4K),
            "qwen7b": make_decode_workload(scaled_shape(QWEN7B_32K, batch=1, steps=1))}


def test_golden_fits_bit_exact(golden_kmeans, workloads):
    for case in golden_kmeans["cases"]:
        case = str(case)
        src, kv, k, bs, it, seed = _parse(case)
        w = workloads[src]
        se = w.keys.shape[2] - 64
        x = w.keys[0, kv, :se].float()
        est = SklearnLikeTorchMiniBatchKMeans(k, batch_size=bs, max_iter=it, random_state=seed)
        lab = est.fit_predict(x.cuda())
        assert lab.dtype == torch.int64
        assert np.array_equal(lab.cpu().numpy(), golden_kmeans[case + "_labels"]), case
        assert np.array_equal(est.cluster_centers_.cpu().numpy(),
                              golden_kmeans[case + "_centers"]), case
        assert np.array_equal(est.counts_.cpu().numpy(), golden_kmeans[case + "_counts"]), case
        assert est.n_steps_ == int(golden_kmeans[case + "_n_steps"]), case
        ref = float(golden_kmeans[case + "_inertia"])
        assert abs(est.inertia_ - ref) <= 1e-5 * ref, case
        if src == "qwen05b":  # the oracle's fixed-point inertia, exactly
            o = O.MiniBatchKMeansOracle(k, batch_size=bs, max_iter=it, random_state=seed)
            o.fit_predict(x.numpy())
            assert est.inertia_ == o.inertia_, case
            assert np.array_equal(est.init_ids_.cpu().numpy(), o.init_ids_), case


def test_reference_unit_case(golden_kmeans):
    # santapp-ruler-bench/tests/test_kmeans_optional.py:12-25 (2 features)
    x = torch.tensor([[0.0, 0.0], [0.1, 0.0], [10.0, 10.0], [10.1, 10.0]], device="cuda")
    lab = SklearnLikeTorchMiniBatchKMeans(2, batch_size=4, max_iter=5,
                                          random_state=0).fit_predict(x)
    assert lab.shape == (4,) and lab.dtype == torch.int64 and len(torch.unique(lab)) == 2
    assert np.array_equal(lab.cpu().numpy(), golden_kmeans["tiny_labels"])


def test_rejects_too_few_samples():
    with pytest.raises(ValueError):
        SklearnLikeTorchMiniBatchKMeans(8).fit_predict(torch.zeros(4, 3, device="cuda"))


@pytest.mark.parametrize("n,d,k,bs,it,seed,n_init", [
    (3000, 36, 40, 512, 6, 3, 1),     # d % 4 != 0, ragged last batch row tile
    (2048, 128, 200, 700, 4, 5, 2),   # n_init > 1 (validation inertia decides)
    (600, 8, 600, 600, 2, 1, 1),      # n == k
    (1000, 16, 1, 256, 3, 0, 1),      # one cluster
])
def test_fits_match_oracle(n, d, k, bs, it, seed, n_init):
    rs = np.random.RandomState(n + d)
    cent = rs.randn(max(k // 2, 1), d).astype(np.float32) * 3
    x = (cent[rs.randint(0, len(cent), n)] + rs.randn(n, d).astype(np.float32)).astype(np.float32)
    x[7] = x[3]  # duplicate rows: equal distances, lowest index wins
    o = O.MiniBatchKMeansOracle(k, batch_size=bs, max_iter=it, random_state=seed, n_init=n_init)
    ol = o.fit_predict(x)
    g = SklearnLikeTorchMiniBatchKMeans(k, batch_size=bs, max_iter=it, random_state=seed,
                                        n_init=n_init)
    gl = g.fit_predict(torch.from_numpy(x).cuda())
    assert np.array_equal(gl.cpu().numpy(), ol)
    assert np.array_equal(g.cluster_centers_.cpu().numpy(), o.cluster_centers_)
    assert np.array_equal(g.counts_.cpu().numpy(), o.counts_)
    assert g.n_steps_ == o.n_steps_ and g.inertia_ == o.inertia_
    assert g.reassign_steps_ == o.reassign_steps_


def test_assign_ties_resolve_to_lowest_centre():
    lib = _lib.load()
    rs = np.random.RandomState(0)
    d, k = 64, 130
    c = rs.randn(k, d).astype(np.float32)
    c[100] = c[3]
    c[129] = c[3]  # equal centres: rows nearest to them must pick 3
    x = np.concatenate([c[[3, 100, 129, 5]] + 1e-3, rs.randn(61, d).astype(np.float32)])
    xx = np.empty(len(x), np.float32)
    O.lib().or_sqnorm(x, len(x), d, xx)
    cc = np.empty(k, np.float32)
    O.lib().or_sqnorm(c, k, d, cc)
    lab_o = np.empty(len(x), np.int32)
    md_o = np.empty(len(x), np.float32)
    inertia = O.lib().or_assign(x, xx, len(x), c, cc, k, d, lab_o, md_o)
    X, XX, C, CC = (torch.from_numpy(a).cuda() for a in (x, xx, c, cc))
    lab = torch.empty(len(x), dtype=torch.int32, device="cuda")
    md = torch.empty(len(x), dtype=torch.float32, device="cuda")
    fx = torch.zeros(2, dtype=torch.int64, device="cuda")
    _lib.check("assign", lib.santa_kmeans_assign(X.data_ptr(), None, XX.data_ptr(), len(x), d,
                                                 C.data_ptr(), CC.data_ptr(), k, lab.data_ptr(),
                                                 md.data_ptr(), fx.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(lab.cpu().numpy(), lab_o) and lab_o[0] == 3
    assert np.array_equal(md.cpu().numpy(), md_o)
    w = fx.cpu().numpy().view(np.uint64)
    assert np.float32(float(int(w[1])) + float(int(w[0])) * 2.0 ** -64) == np.float32(inertia)


def test_gpu_minibatch_labels_entry_point(workloads):
    x = workloads["qwen05b"].keys[0, 0, :4032].float()
    a = gpu_minibatch_labels(x.cuda(), 16, 4).cpu().numpy()
    o = O.MiniBatchKMeansOracle(16, batch_size=4096, max_iter=100, random_state=4)
    assert np.array_equal(a, o.fit_predict(x.numpy()))
