"""The oracle is pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py) and against published known-answer vectors."""
import math

import numpy as np
import pytest

from oracle import santa_oracle as O
from santapp_b200.synthetic import (QWEN05B_4K, QWEN7B_32K, make_decode_workload,
                                    scaled_shape, tensor_digest)

QWEN7B_SMALL = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx2048-b2", batch=2,
                            context=2048, true_clusters=32, n_clusters=32,
                            topk_clusters=4, samples=64, steps=1)


def _parse(case):
    src, kv, k, bs, it, s = case.split("_")
    return src, int(kv[2:]), int(k[1:]), int(bs[2:]), int(it[2:]), int(s[1:])


@pytest.fixture(scope="module")
def workloads(golden_kmeans):
    w1 = make_decode_workload(QWEN05B_4K)
    assert tensor_digest(w1.keys, w1.values, w1.queries) == str(golden_kmeans["qwen05b_digest"])
    w2 = make_decode_workload(scaled_shape(QWEN7B_32K, batch=1, steps=1))
    assert tensor_digest(w2.keys, w2.values, w2.queries) == str(golden_kmeans["qwen7b_digest"])
    return {"qwen05b": w1, "qwen7b": w2}


def test_kmeans_matches_reference_bit_exact(golden_kmeans, workloads):
    for case in golden_kmeans["cases"]:
        case = str(case)
        src, kv, k, bs, it, seed = _parse(case)
        w = workloads[src]
        se = w.keys.shape[2] - 64
        x = w.keys[0, kv, :se].float().numpy()
        est = O.MiniBatchKMeansOracle(k, batch_size=bs, max_iter=it, random_state=seed)
        lab = est.fit_predict(x)
        assert np.array_equal(lab, golden_kmeans[case + "_labels"]), case
        assert np.array_equal(est.cluster_centers_, golden_kmeans[case + "_centers"]), case
        assert np.array_equal(est.counts_, golden_kmeans[case + "_counts"]), case
        assert est.n_steps_ == int(golden_kmeans[case + "_n_steps"]), case
        # The final inertia is a reported fp32 total, not a control-flow input.
        # The reference sums MKL distances in torch's fp32 reduction order
        # (about 15 ulp off the exact total at 32K rows); the oracle's
        # fixed-point sum is the correctly rounded total of its own distances.
        ref_inertia = float(golden_kmeans[case + "_inertia"])
        assert abs(est.inertia_ - ref_inertia) <= 1e-5 * ref_inertia, case


def test_kmeans_reference_unit_case(golden_kmeans):
    # santapp-ruler-bench/tests/test_kmeans_optional.py:12-25
    x = np.array([[0.0, 0.0], [0.1, 0.0], [10.0, 10.0], [10.1, 10.0]], np.float32)
    lab = O.MiniBatchKMeansOracle(2, batch_size=4, max_iter=5, random_state=0).fit_predict(x)
    assert lab.shape == (4,) and lab.dtype == np.int64 and len(np.unique(lab)) == 2
    assert np.array_equal(lab, golden_kmeans["tiny_labels"])


def test_kmeans_rejects_too_few_samples():
    with pytest.raises(ValueError):
        O.MiniBatchKMeansOracle(8).fit_predict(np.zeros((4, 3), np.float32))


def _decode_case(golden, prefix, shape):
    w = make_decode_workload(shape)
    assert tensor_digest(w.keys, w.values, w.queries) == str(golden[prefix + "digest"])
    return w


@pytest.mark.parametrize("prefix,shape", [("qwen05b_", QWEN05B_4K), ("qwen7b_", QWEN7B_SMALL)])
def test_summary_matches_reference(golden_decode, golden_kmeans, prefix, shape):
    w = _decode_case(golden_decode, prefix, shape)
    se = shape.sample_end
    for b in range(shape.batch):
        for kv in range(shape.num_kv_heads):
            if prefix == "qwen05b_":
                lab = golden_kmeans[f"qwen05b_kv{kv}_k64_bs1024_it10_s0_labels"]
            else:
                lab = w.labels[b, kv, :se].numpy()
            s = O.build_summary(w.keys[b, kv, :se].float().numpy(), lab, shape.n_clusters)
            key = f"{prefix}summary_{b}_{kv}_"
            assert np.array_equal(s.members, golden_decode[key + "members"])
            assert np.array_equal(s.starts, golden_decode[key + "starts"])
            assert np.array_equal(s.lengths, golden_decode[key + "lengths"])
            assert np.array_equal(s.centroids, golden_decode[key + "centroids"])


@pytest.mark.parametrize("prefix,shape", [("qwen05b_", QWEN05B_4K), ("qwen7b_", QWEN7B_SMALL)])
def test_decode_modes_match_reference(golden_decode, golden_kmeans, prefix, shape):
    w = _decode_case(golden_decode, prefix, shape)
    se, g, scale = shape.sample_end, shape.group, 1.0 / math.sqrt(shape.head_dim)
    summaries = {}
    for b in range(shape.batch):
        for kv in range(shape.num_kv_heads):
            lab = (golden_kmeans[f"qwen05b_kv{kv}_k64_bs1024_it10_s0_labels"]
                   if prefix == "qwen05b_" else w.labels[b, kv, :se].numpy())
            summaries[(b, kv)] = O.build_summary(w.keys[b, kv, :se].float().numpy(), lab,
                                                 shape.n_clusters)
    worst = 0.0
    for mode in ("topk", "guided", "uniform", "santa"):
        ref = golden_decode[f"{prefix}{mode}_out"]
        samples = int(golden_decode[f"{prefix}{mode}_samples"])
        for b in range(shape.batch):
            for h in range(shape.num_query_heads):
                kv = h // g
                K = w.keys[b, kv].float().numpy()
                V = w.values[b, kv].float().numpy()
                q = w.queries[0, b, h].numpy()
                s = summaries[(b, kv)]
                if mode == "topk":
                    r = O.decode_topk(q, K, V, s, se, samples, scale)
                elif mode == "guided":
                    r = O.decode_guided(q, K, V, s, se, golden_decode[f"{prefix}guided_groups"][b, h],
                                        golden_decode[f"{prefix}guided_within"][b, h], scale)
                elif mode == "uniform":
                    r = O.decode_uniform(q, K, V, se, golden_decode[f"{prefix}uniform_idx"][b, h], scale)
                else:
                    r = O.decode_santa(q, K, V, se, golden_decode[f"{prefix}santa_idx"][b, h], scale)
                err = float(np.abs(r.out - ref[b, h]).max())
                worst = max(worst, err)
                assert err < 1e-4, (mode, b, h, err)
    assert worst < 1e-4


def test_hybrid_reduces_to_dense_when_everything_is_selected():
    rs = np.random.RandomState(0)
    T, D, G = 300, 16, 10
    K = rs.randn(T, D).astype(np.float32)
    V = rs.randn(T, D).astype(np.float32)
    q = rs.randn(D).astype(np.float32)
    se = T - 20
    lab = rs.randint(0, G, se)
    s = O.build_summary(K[:se], lab, G)
    r = O.decode_hybrid(q, K, V, s, se, s.num_groups, [], 0.25)
    sc = K.astype(np.float64) @ q * 0.25
    p = np.exp(sc - sc.max())
    dense = p @ V / p.sum()
    assert np.abs(r.out - dense).max() < 1e-12
    assert abs(r.lse - (sc.max() + math.log(p.sum()))) < 1e-12


def test_hybrid_positions_skip_selected_clusters():
    rs = np.random.RandomState(1)
    lab = rs.randint(0, 6, 200)
    s = O.build_summary(rs.randn(200, 4).astype(np.float32), lab, 6)
    sel = np.array([4, 1])
    n_rest = 200 - int(s.lengths[sel].sum())
    pos = O.hybrid_positions(s, sel, np.arange(n_rest))
    excluded = set()
    for gsel in sel:
        excluded |= set(range(s.starts[gsel], s.starts[gsel] + s.lengths[gsel]))
    assert list(pos) == [p for p in range(200) if p not in excluded]


def test_philox_known_answers():
    # Random123 known-answer vectors for Philox4x32-10.
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
        ([0xffffffff] * 4, [0xffffffff] * 2, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
        ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
         [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
    ]
    for ctr, key, want in kat:
        assert list(O.philox4x32(ctr, key)) == want


def test_fixed_point_sum_is_order_independent():
    rs = np.random.RandomState(2)
    v = (rs.rand(10000) * 100).astype(np.float32) ** 3
    a = O.fx_sum(v)
    b = O.fx_sum(v[rs.permutation(v.size)])
    assert a == b
    assert abs(float(a) - float(v.astype(np.float64).sum())) <= 1e-6 * float(a)
    c = O.fx_cumsum(v)
    assert c[-1] == a


def test_log_count_is_correctly_rounded_double_log():
    n = np.arange(1, 1 << 17)
    assert np.array_equal(O.log_count(n), np.array([math.log(i) for i in n], np.float64).astype(np.float32))


@pytest.mark.parametrize("prefix,shape", [("qwen05b_", QWEN05B_4K), ("qwen7b_", QWEN7B_SMALL)])
@pytest.mark.parametrize("mode", ["topk", "guided", "uniform", "santa"])
def test_traffic_tracker_matches_reference(golden_decode, prefix, shape, mode):
    """DecodeTrafficTracker.record_step (one batched call per (sequence, KV
    head) segment) accumulates the counters the reference's per-head
    record() calls produced (santapp.py:419-426, 498-505) over the same head
    calls: same exact-token counts (topk), sample counts, recent window,
    cluster metadata reads and ESS ratios."""
    import json
    from santapp_b200.attention.santapp import DecodeTrafficTracker
    want = json.loads(str(golden_decode[f"{prefix}{mode}_traffic"]))
    draws = golden_decode[f"{prefix}{mode}_draws_per_call"]
    ess = golden_decode[f"{prefix}{mode}_ess"]
    samples = int(golden_decode[f"{prefix}{mode}_samples"])
    g = shape.group
    t = DecodeTrafficTracker()
    for b in range(shape.batch):
        for kv in range(shape.num_kv_heads):
            n_groups = golden_decode[f"{prefix}summary_{b}_{kv}_lengths"].size
            heads = slice(kv * g, (kv + 1) * g)
            t.record_step(mode=mode, n_total=shape.context, sample_end=shape.sample_end,
                          n_exact=draws[b, heads] if mode == "topk" else np.zeros(g, np.int64),
                          samples=samples, n_groups=np.array([n_groups]),
                          ess=None if mode == "topk" else ess[b, heads])
    got = t.as_dict()
    assert set(got) == set(want)
    for k, v in want.items():
        if v is None or isinstance(v, int):
            assert got[k] == v, k
        else:
            assert got[k] == pytest.approx(v, rel=1e-9, abs=1e-12), k
