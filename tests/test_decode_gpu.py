"""Parity of the CUDA summary build and sparse decode against the oracle.

Bit-exact: members, positions, starts, lengths, log counts, centroids,
selected cluster sets, sample rows.  Floating point (attention output):
max-abs 2e-2 and mean-abs 2e-3 against the fp64 oracle for bf16 K/V (the
stated tolerance), 1e-4 / 1e-5 for fp32 K/V.
"""
import math

import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention import santapp as S
from santapp_b200.synthetic import (QWEN05B_4K, QWEN7B_32K, QWEN3_8B_128K, make_decode_workload,
                                    scaled_shape, tensor_digest)

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

QWEN7B_SMALL = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx2048-b2", batch=2,
                            context=2048, true_clusters=32, n_clusters=32,
                            topk_clusters=4, samples=64, steps=1)

TOL = {torch.float32: (1e-4, 1e-5), torch.bfloat16: (2e-2, 2e-3)}


def _labels(prefix, w, golden_kmeans):
    sh = w.shape
    if prefix == "qwen05b_":
        return np.stack([golden_kmeans[f"qwen05b_kv{kv}_k64_bs1024_it10_s0_labels"]
                         for kv in range(sh.num_kv_heads)])[None]
    return w.labels[:, :, :sh.sample_end].numpy()


class Case:
    """A workload on the device plus its oracle summaries."""

    def __init__(self, shape, labels_np, workload=None):
        self.shape = shape
        self.w = workload or make_decode_workload(shape)
        self.labels = labels_np.astype(np.int64)
        self.kc = self.w.keys.cuda().contiguous()
        self.vc = self.w.values.cuda().contiguous()
        se = shape.sample_end
        self.summary = S.build_summary(self.kc, self.vc, torch.from_numpy(self.labels).cuda(),
                                       shape.n_clusters, sample_end=se, n_total=shape.context)
        torch.cuda.synchronize()
        self.osum = {}
        for b in range(shape.batch):
            for kv in range(shape.num_kv_heads):
                self.osum[(b, kv)] = O.build_summary(self.w.keys[b, kv, :se].float().numpy(),
                                                     self.labels[b, kv], shape.n_clusters)

    def q(self, step=0):
        return self.w.queries[step].cuda().contiguous()

    def kv_np(self, b, kv):
        return self.w.keys[b, kv].float().numpy(), self.w.values[b, kv].float().numpy()


@pytest.fixture(scope="module")
def cases(golden_decode, golden_kmeans):
    out = {}
    for prefix, shape in (("qwen05b_", QWEN05B_4K), ("qwen7b_", QWEN7B_SMALL)):
        w = make_decode_workload(shape)
        assert tensor_digest(w.keys, w.values, w.queries) == str(golden_decode[prefix + "digest"])
        out[prefix] = Case(shape, _labels(prefix, w, golden_kmeans), w)
    return out


def _check_summary(case):
    s, sh = case.summary, case.shape
    for (b, kv), o in case.osum.items():
        n = int(s.n_groups[b, kv])
        assert n == o.num_groups
        assert np.array_equal(s.members[b, kv].cpu().numpy(), o.members)
        pos = np.empty_like(o.members)
        pos[o.members] = np.arange(o.members.size)
        assert np.array_equal(s.positions[b, kv].cpu().numpy(), pos)
        assert np.array_equal(s.starts[b, kv, :n].cpu().numpy(), o.starts)
        assert np.array_equal(s.lengths_long[b, kv, :n].cpu().numpy(), o.lengths)
        assert np.array_equal(s.log_n[b, kv, :n].cpu().numpy(), o.log_n)
        assert np.array_equal(s.key_centroids[b, kv, :n].cpu().numpy(), o.centroids)
        kk = case.w.keys[b, kv, :sh.sample_end][torch.from_numpy(o.members)]
        assert torch.equal(s.sorted_key[b, kv].cpu(), kk)
        vv = case.w.values[b, kv, :sh.sample_end][torch.from_numpy(o.members)]
        assert torch.equal(s.sorted_value[b, kv].cpu(), vv)


@pytest.mark.parametrize("prefix", ["qwen05b_", "qwen7b_"])
def test_summary_matches_oracle(cases, golden_decode, prefix):
    case = cases[prefix]
    _check_summary(case)
    # and therefore the reference's own _build_summary output
    for (b, kv), o in case.osum.items():
        key = f"{prefix}summary_{b}_{kv}_"
        n = int(case.summary.n_groups[b, kv])
        assert np.array_equal(case.summary.key_centroids[b, kv, :n].cpu().numpy(),
                              golden_decode[key + "centroids"])


@pytest.mark.parametrize("dtype,D,N,G,pattern", [
    (torch.float32, 64, 2500, 64, "even"),       # empty clusters, ragged chunk
    (torch.bfloat16, 128, 3000, 1024, "random"),  # many empty clusters, G at its maximum
    (torch.bfloat16, 64, 1025, 7, "single"),      # one cluster holds everything
    (torch.float32, 128, 700, 5, "random"),
])
def test_summary_edge_cases(dtype, D, N, G, pattern):
    rs = np.random.RandomState(N)
    B, H = 2, 3
    if pattern == "even":
        lab = 2 * rs.randint(0, G // 2, (B, H, N))
    elif pattern == "single":
        lab = np.full((B, H, N), G - 1)
    else:
        lab = rs.randint(0, G, (B, H, N))
    T = N + 17
    k = torch.from_numpy(rs.randn(B, H, T, D).astype(np.float32)).to(dtype)
    v = torch.from_numpy(rs.randn(B, H, T, D).astype(np.float32)).to(dtype)
    sh = scaled_shape(QWEN05B_4K, batch=B, num_kv_heads=H, num_query_heads=H, head_dim=D,
                      context=T, n_clusters=G, recent_window=17, kv_dtype=dtype)

    class W:
        keys, values = k, v
    case = Case.__new__(Case)
    case.shape, case.w, case.labels = sh, W, lab
    case.kc, case.vc = k.cuda(), v.cuda()
    case.summary = S.build_summary(case.kc, case.vc, torch.from_numpy(lab).cuda(), G,
                                   sample_end=N, n_total=T)
    case.osum = {(b, h): O.build_summary(k[b, h, :N].float().numpy(), lab[b, h], G)
                 for b in range(B) for h in range(H)}
    _check_summary(case)


def _oracle_decode(case, mode, b, h, budget=None, draws=None, topk=None):
    sh = case.shape
    kv = h // sh.group
    K, V = case.kv_np(b, kv)
    q = case.w.queries[0, b, h].numpy()
    o = case.osum[(b, kv)]
    se, scale = sh.sample_end, 1.0 / math.sqrt(sh.head_dim)
    if mode == "topk":
        return O.decode_topk(q, K, V, o, se, budget, scale)
    if mode == "guided":
        return O.decode_guided(q, K, V, o, se, draws[0][b, h], draws[1][b, h], scale)
    if mode == "uniform":
        return O.decode_uniform(q, K, V, se, draws[0][b, h], scale)
    if mode == "santa":
        return O.decode_santa(q, K, V, se, draws[0][b, h], scale)
    return O.decode_hybrid(q, K, V, o, se, topk, draws[0][b, h], scale)


def _compare(case, res, oracle_results, golden=None):
    sh = case.shape
    tol_max, tol_mean = TOL[sh.kv_dtype]
    got = res.out.cpu().numpy().astype(np.float64)
    want = np.stack([[oracle_results[(b, h)].out for h in range(sh.num_query_heads)]
                     for b in range(sh.batch)])
    err = np.abs(got - want)
    assert err.max() < tol_max, err.max()
    assert err.mean() < tol_mean, err.mean()
    lse = np.array([[oracle_results[(b, h)].lse for h in range(sh.num_query_heads)]
                    for b in range(sh.batch)])
    assert np.abs(res.lse.cpu().numpy() - lse).max() < 1e-3
    if golden is not None:
        gerr = np.abs(got - golden.astype(np.float64))
        assert gerr.max() < tol_max and gerr.mean() < tol_mean, (gerr.max(), gerr.mean())
    return err.max()


@pytest.mark.parametrize("prefix", ["qwen05b_", "qwen7b_"])
@pytest.mark.parametrize("mode", ["topk", "guided", "uniform", "santa"])
def test_reference_modes_match_oracle_and_reference(cases, golden_decode, prefix, mode):
    case = cases[prefix]
    sh = case.shape
    n = int(golden_decode[f"{prefix}{mode}_samples"])
    kw = dict(mode=mode, n_total=sh.context, with_stats=True)
    draws = None
    if mode == "topk":
        kw["token_budget"] = n
    else:
        kw["samples"] = n
        if mode == "guided":
            draws = (golden_decode[f"{prefix}guided_groups"], golden_decode[f"{prefix}guided_within"])
            kw["sample_a"] = torch.from_numpy(draws[0].astype(np.int32)).cuda()
            kw["sample_b"] = torch.from_numpy(draws[1].astype(np.int32)).cuda()
        else:
            draws = (golden_decode[f"{prefix}{mode}_idx"],)
            kw["sample_a"] = torch.from_numpy(draws[0].astype(np.int32)).cuda()
    res = S.santa_decode(case.q(), case.kc, case.vc, case.summary, **kw)
    torch.cuda.synchronize()
    orc = {(b, h): _oracle_decode(case, mode, b, h, budget=n, draws=draws)
           for b in range(sh.batch) for h in range(sh.num_query_heads)}
    _compare(case, res, orc, golden_decode[f"{prefix}{mode}_out"])
    if mode == "topk":
        n_exact = np.array([[orc[(b, h)].n_exact for h in range(sh.num_query_heads)]
                            for b in range(sh.batch)])
        assert np.array_equal(res.n_exact.cpu().numpy(), n_exact)
        sel, _, _ = S.santa_decode_select(case.q(), case.kc, case.vc, case.summary, **{
            k: v for k, v in kw.items() if k != "with_stats"})
        sel = sel.cpu().numpy()
        for (b, h), r in orc.items():
            want = np.zeros(case.summary.max_groups, np.uint8)
            want[r.selected] = 1
            assert np.array_equal(sel[b, h], want), (b, h)
    else:
        ess = np.array([[orc[(b, h)].ess for h in range(sh.num_query_heads)]
                        for b in range(sh.batch)])
        assert np.abs(res.ess.cpu().numpy() - ess).max() < 1e-3


@pytest.mark.parametrize("prefix", ["qwen05b_", "qwen7b_"])
def test_hybrid_injected_matches_oracle(cases, prefix):
    case = cases[prefix]
    sh = case.shape
    rs = np.random.RandomState(7)
    topk, S_ = sh.topk_clusters, sh.samples
    # ranks must lie in [0, n_rest): draw per head from the oracle's n_rest
    ranks = np.zeros((sh.batch, sh.num_query_heads, S_), np.int64)
    for b in range(sh.batch):
        for h in range(sh.num_query_heads):
            o = case.osum[(b, h // sh.group)]
            g = O.centroid_guess(o, case.w.queries[0, b, h].numpy(), 1.0 / math.sqrt(sh.head_dim))
            sel = O.select_topk(g, topk)
            n_rest = sh.sample_end - int(o.lengths[sel].sum())
            ranks[b, h] = rs.randint(0, n_rest, S_)
    a = torch.from_numpy(ranks.astype(np.int32)).cuda()
    res = S.santa_decode(case.q(), case.kc, case.vc, case.summary, mode="hybrid",
                         n_total=sh.context, topk_clusters=topk, samples=S_, sample_a=a,
                         with_stats=True)
    sel, rows, n_exact = S.santa_decode_select(case.q(), case.kc, case.vc, case.summary,
                                               mode="hybrid", n_total=sh.context,
                                               topk_clusters=topk, samples=S_, sample_a=a)
    torch.cuda.synchronize()
    orc = {(b, h): _oracle_decode(case, "hybrid", b, h, draws=(ranks,), topk=topk)
           for b in range(sh.batch) for h in range(sh.num_query_heads)}
    _compare(case, res, orc)
    sel, rows = sel.cpu().numpy(), rows.cpu().numpy()
    for (b, h), r in orc.items():
        want = np.zeros(case.summary.max_groups, np.uint8)
        want[r.selected] = 1
        assert np.array_equal(sel[b, h], want)
        o = case.osum[(b, h // sh.group)]
        assert np.array_equal(rows[b, h], O.hybrid_positions(o, r.selected, ranks[b, h]))
        assert int(n_exact[b, h]) == r.n_exact


@pytest.mark.parametrize("mode", ["hybrid", "uniform"])
def test_out_of_range_injected_draws_raise(cases, mode):
    """An injected draw outside its range is clamped by the kernel, flagged for
    its segment and reported as ValueError; the next valid call is clean (the
    selection kernel clears the flags)."""
    case = cases["qwen7b_"]
    sh = case.shape
    kw = dict(mode=mode, n_total=sh.context, topk_clusters=sh.topk_clusters, samples=sh.samples)
    a = torch.zeros(sh.batch, sh.num_query_heads, sh.samples, dtype=torch.int32, device="cuda")
    a[-1, -1, 3] = sh.sample_end + 5  # beyond n_rest and beyond sample_end
    with pytest.raises(ValueError, match="out of range"):
        S.santa_decode(case.q(), case.kc, case.vc, case.summary, sample_a=a, **kw)
    with pytest.raises(ValueError, match="out of range"):
        S.santa_decode_select(case.q(), case.kc, case.vc, case.summary, sample_a=a, **kw)
    a[-1, -1, 3] = 0
    S.santa_decode(case.q(), case.kc, case.vc, case.summary, sample_a=a, **kw)


def test_hybrid_device_sampler_matches_philox_oracle(cases):
    case = cases["qwen7b_"]
    sh = case.shape
    seed, step = 0x1234_5678_9ABC, 5
    sel, rows, n_exact = S.santa_decode_select(case.q(), case.kc, case.vc, case.summary,
                                               mode="hybrid", n_total=sh.context,
                                               topk_clusters=sh.topk_clusters,
                                               samples=sh.samples, seed=seed, step=step)
    rows = rows.cpu().numpy()
    n_exact = n_exact.cpu().numpy()
    for b in range(sh.batch):
        for h in range(sh.num_query_heads):
            o = case.osum[(b, h // sh.group)]
            g = O.centroid_guess(o, case.w.queries[0, b, h].numpy(), 1.0 / math.sqrt(sh.head_dim))
            chosen = O.select_topk(g, sh.topk_clusters)
            n_rest = sh.sample_end - int(o.lengths[chosen].sum())
            assert int(n_exact[b, h]) == sh.sample_end - n_rest
            ranks = O.philox_ranks(seed, step, b, h, sh.samples, n_rest)
            assert np.array_equal(rows[b, h], O.hybrid_positions(o, chosen, ranks))


def test_guided_device_sampler_stays_in_clusters(cases):
    case = cases["qwen7b_"]
    sh = case.shape
    _, rows, _ = S.santa_decode_select(case.q(), case.kc, case.vc, case.summary, mode="guided",
                                       n_total=sh.context, samples=sh.samples, seed=3)
    rows = rows.cpu().numpy()
    assert rows.min() >= 0 and rows.max() < sh.sample_end
    res = S.santa_decode(case.q(), case.kc, case.vc, case.summary, mode="guided",
                         n_total=sh.context, samples=sh.samples, seed=3, with_stats=True)
    assert torch.isfinite(res.out).all()
    assert ((res.ess > 0) & (res.ess <= 1.0 + 1e-5)).all()


def _chi2_pvalue(counts, expected):
    """Pearson chi-square goodness of fit, cells with expected < 5 pooled."""
    from scipy import stats
    small = expected < 5
    obs = np.append(counts[~small], counts[small].sum())
    exp = np.append(expected[~small], expected[small].sum())
    if exp[-1] == 0:
        obs, exp = obs[:-1], exp[:-1]
    return stats.chisquare(obs, exp * obs.sum() / exp.sum()).pvalue


def test_guided_device_sampler_distribution_matches_reference_draws(cases):
    """The on-device guided sampler (Philox, inverse CDF over the clusters,
    then a uniform position inside the cluster) draws from the reference's
    proposal (santapp.py:429-449: torch.multinomial over softmax(log n +
    C q scale), then floor(rand * len)).  Over 16 steps x 1024 draws per
    head, for every query head: the cluster counts fit the proposal
    (chi-square), they are indistinguishable from the same number of draws
    by the reference's torch sampler (two-sample chi-square), and the
    position inside the cluster is uniform (randomised PIT, Kolmogorov-
    Smirnov).  Threshold p > 1e-5 per test; the seeds are fixed, so the
    outcome is deterministic."""
    from scipy import stats
    case = cases["qwen7b_"]
    sh = case.shape
    n_draw, steps = 1024, 16
    q = case.q()
    rows = np.concatenate([S.santa_decode_select(q, case.kc, case.vc, case.summary,
                                                 mode="guided", n_total=sh.context,
                                                 samples=n_draw, seed=5, step=st)[1].cpu().numpy()
                           for st in range(steps)], axis=-1)
    qn = q.cpu().numpy()
    gen = torch.Generator().manual_seed(11)
    rs = np.random.RandomState(3)
    N = n_draw * steps
    for b in range(sh.batch):
        for h in range(sh.num_query_heads):
            o = case.osum[(b, h // sh.group)]
            G = o.num_groups
            p = O.group_probability(o, qn[b, h], sh.scale)
            r = rows[b, h]
            assert (r >= 0).all() and (r < sh.sample_end).all()
            grp = np.searchsorted(o.starts, r, side="right") - 1
            within = r - o.starts[grp]
            assert (within < o.lengths[grp]).all()
            counts = np.bincount(grp, minlength=G)
            assert _chi2_pvalue(counts, p * N) > 1e-5, (b, h)
            # the reference's own draws (torch.multinomial + rand) of the same size
            tg = torch.multinomial(torch.from_numpy(p), N, replacement=True, generator=gen)
            tcounts = np.bincount(tg.numpy(), minlength=G)
            assert _chi2_pvalue(tcounts, p * N) > 1e-5  # the test itself accepts the reference
            keep = (counts + tcounts) > 0
            table = np.stack([counts[keep], tcounts[keep]])
            assert stats.chi2_contingency(table).pvalue > 1e-5, (b, h)
            u = (within + rs.random_sample(N)) / o.lengths[grp]
            assert stats.kstest(u, "uniform").pvalue > 1e-5, (b, h)


def test_decode_rejects_bad_budgets(cases):
    case = cases["qwen7b_"]
    sh = case.shape
    with pytest.raises(RuntimeError, match="invalid argument"):
        S.santa_decode(case.q(), case.kc, case.vc, case.summary, mode="hybrid",
                       n_total=sh.context, topk_clusters=sh.n_clusters + 1, samples=4)
    with pytest.raises(RuntimeError, match="Invalid sampled-prefix"):
        S.santa_decode(case.q(), case.kc, case.vc, case.summary, mode="topk",
                       n_total=sh.context, sample_end=sh.context + 1, token_budget=8)


def _dense_reference(q, K, V, scale, n_total):
    """fp32 torch dense attention over [0, n_total) for every (b, q-head)."""
    B, Hq, D = q.shape
    g = Hq // K.shape[1]
    Kf = K[:, :, :n_total].float().repeat_interleave(g, dim=1)
    Vf = V[:, :, :n_total].float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhd,bhtd->bht", q, Kf) * scale
    lse = torch.logsumexp(s, dim=-1)
    return torch.einsum("bht,bhtd->bhd", torch.softmax(s, dim=-1), Vf), lse


def test_full_size_selecting_every_cluster_is_dense_attention():
    """At the Qwen2.5-7B batch-8 32K shape, exact top-k over every cluster has
    no remainder to sample and must equal dense softmax attention."""
    sh = QWEN7B_32K
    w = make_decode_workload(scaled_shape(sh, steps=1), device="cuda")
    labels = w.labels[:, :, :sh.sample_end].contiguous()
    summ = S.build_summary(w.keys, w.values, labels, sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    q = w.queries[0].contiguous()
    res = S.santa_decode(q, w.keys, w.values, summ, mode="hybrid", n_total=sh.context,
                         topk_clusters=sh.n_clusters, samples=sh.samples, with_stats=True)
    ref, ref_lse = _dense_reference(q, w.keys, w.values, sh.scale, sh.context)
    err = (res.out - ref).abs()
    assert err.max().item() < 2e-2 and err.mean().item() < 2e-3
    assert (res.lse - ref_lse).abs().max().item() < 1e-3
    assert (res.n_exact == sh.sample_end).all()


def test_full_size_hybrid_selection_bit_exact_and_output_close():
    """Qwen2.5-7B batch-8 32K: every head's selected cluster set equals the
    oracle's; outputs of a subset of heads match the oracle within tolerance."""
    sh = QWEN7B_32K
    w = make_decode_workload(scaled_shape(sh, steps=1), device="cuda")
    labels = w.labels[:, :, :sh.sample_end].contiguous()
    summ = S.build_summary(w.keys, w.values, labels, sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    q = w.queries[0].contiguous()
    sel, rows, n_exact = S.santa_decode_select(q, w.keys, w.values, summ, mode="hybrid",
                                               n_total=sh.context,
                                               topk_clusters=sh.topk_clusters,
                                               samples=sh.samples, seed=11, step=0)
    res = S.santa_decode(q, w.keys, w.values, summ, mode="hybrid", n_total=sh.context,
                         topk_clusters=sh.topk_clusters, samples=sh.samples, seed=11, step=0)
    sel, rows, out = sel.cpu().numpy(), rows.cpu().numpy(), res.out.cpu().numpy()
    qn = q.cpu().numpy()
    keys_cpu = w.keys.cpu()
    vals_cpu = w.values.cpu()
    lab_cpu = labels.cpu().numpy()
    checked = 0
    errs = []
    for b in range(sh.batch):
        for kv in range(sh.num_kv_heads):
            o = O.build_summary(keys_cpu[b, kv, :sh.sample_end].float().numpy(), lab_cpu[b, kv],
                                sh.n_clusters)
            assert np.array_equal(summ.key_centroids[b, kv, :o.num_groups].cpu().numpy(),
                                  o.centroids)
            for hh in range(sh.group):
                h = kv * sh.group + hh
                g = O.centroid_guess(o, qn[b, h], sh.scale)
                chosen = O.select_topk(g, sh.topk_clusters)
                want = np.zeros(sh.n_clusters, np.uint8)
                want[chosen] = 1
                assert np.array_equal(sel[b, h], want), (b, h)
                n_rest = sh.sample_end - int(o.lengths[chosen].sum())
                ranks = O.philox_ranks(11, 0, b, h, sh.samples, n_rest)
                assert np.array_equal(rows[b, h], O.hybrid_positions(o, chosen, ranks))
                if (b + hh) % 7 == 0:
                    K = keys_cpu[b, kv].float().numpy()
                    V = vals_cpu[b, kv].float().numpy()
                    r = O.decode_hybrid(qn[b, h], K, V, o, sh.sample_end, sh.topk_clusters,
                                        ranks, sh.scale)
                    errs.append(np.abs(out[b, h] - r.out))
                    checked += 1
    assert checked >= 8
    e = np.stack(errs)
    assert e.max() < 2e-2 and e.mean() < 2e-3, (e.max(), e.mean())


@pytest.mark.parametrize("mode", ["hybrid", "topk"])
def test_many_clusters_selection_bit_exact(mode):
    """More than 256 clusters per KV head takes the 32-keys-per-lane top-k path."""
    sh = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx8192-g600", batch=1, context=8192,
                      true_clusters=600, n_clusters=600, topk_clusters=40, samples=96, steps=1)
    w = make_decode_workload(sh, seed=3)
    kc, vc = w.keys.cuda(), w.values.cuda()
    labels = w.labels[:, :, :sh.sample_end]
    summ = S.build_summary(kc, vc, labels.cuda(), sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    q = w.queries[0].cuda()
    budget = 40 * (sh.sample_end // sh.n_clusters)
    kw = dict(mode=mode, n_total=sh.context, seed=4, step=1)
    if mode == "hybrid":
        kw.update(topk_clusters=sh.topk_clusters, samples=sh.samples)
    else:
        kw.update(token_budget=budget)
    sel, rows, n_exact = S.santa_decode_select(q, kc, vc, summ, **kw)
    res = S.santa_decode(q, kc, vc, summ, **kw)
    sel, rows, out = sel.cpu().numpy(), rows.cpu().numpy(), res.out.cpu().numpy()
    for kv in range(sh.num_kv_heads):
        K = w.keys[0, kv].float().numpy()
        V = w.values[0, kv].float().numpy()
        o = O.build_summary(K[:sh.sample_end], labels[0, kv].numpy(), sh.n_clusters)
        for hh in range(sh.group):
            h = kv * sh.group + hh
            qh = w.queries[0, 0, h].numpy()
            if mode == "hybrid":
                chosen = O.select_topk(O.centroid_guess(o, qh, sh.scale), sh.topk_clusters)
                n_rest = sh.sample_end - int(o.lengths[chosen].sum())
                ranks = O.philox_ranks(4, 1, 0, h, sh.samples, n_rest)
                assert np.array_equal(rows[0, h], O.hybrid_positions(o, chosen, ranks))
                r = O.decode_hybrid(qh, K, V, o, sh.sample_end, sh.topk_clusters, ranks, sh.scale)
            else:
                r = O.decode_topk(qh, K, V, o, sh.sample_end, budget, sh.scale)
                chosen = r.selected
            want = np.zeros(sh.n_clusters, np.uint8)
            want[chosen] = 1
            assert np.array_equal(sel[0, h], want), (kv, hh)
            assert int(n_exact[0, h]) == int(o.lengths[chosen].sum())
            assert np.abs(out[0, h] - r.out).max() < 2e-2


@pytest.mark.parametrize("name,changes", [
    # Qwen3-8B group of 4 with 1024 clusters and top-32 (the 128K selection)
    ("g4-1024c-k32", dict(base=QWEN3_8B_128K, batch=2, context=24576, samples=512)),
    # cluster counts that are not a multiple of the 32-key batches
    ("g7-600c-k32", dict(batch=1, context=8192, true_clusters=600, n_clusters=600,
                         topk_clusters=32, samples=96)),
    # empty clusters: fewer non-empty groups than summary rows
    ("g7-empty-k20", dict(batch=2, context=4096, true_clusters=80, n_clusters=96,
                          topk_clusters=20, samples=128)),
    # one query head per KV head (cluster of one CTA) and a full group of 8
    ("g1-d64", dict(num_query_heads=4, num_kv_heads=4, head_dim=64, batch=2, context=4096,
                    true_clusters=64, n_clusters=64, topk_clusters=8, samples=64)),
    ("g8-k1", dict(num_query_heads=16, num_kv_heads=2, batch=2, context=4096, true_clusters=40,
                   n_clusters=40, topk_clusters=1, samples=32)),
    # 32 (sequence, KV head) segments over 148 CTAs: a handful of CTA partials
    # per segment, merged without staging (head_dim 64: two dims per lane)
    ("g2-d64-b8", dict(num_query_heads=8, num_kv_heads=4, head_dim=64, batch=8, context=4096,
                       true_clusters=48, n_clusters=48, topk_clusters=6, samples=64)),
])
def test_hybrid_selection_shapes_bit_exact(name, changes):
    """The hybrid selection (one CTA per query head, a cluster per KV head)
    across group sizes, cluster counts and k: selected sets, n_exact and
    sample rows bit-exact, outputs within the bf16 tolerance."""
    changes = dict(changes)
    base = changes.pop("base", QWEN7B_32K)
    sh = scaled_shape(base, name=name, steps=1, **changes)
    w = make_decode_workload(sh, seed=5)
    kc, vc = w.keys.cuda(), w.values.cuda()
    labels = w.labels[:, :, :sh.sample_end]
    summ = S.build_summary(kc, vc, labels.cuda(), sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    q = w.queries[0].cuda()
    kw = dict(mode="hybrid", n_total=sh.context, topk_clusters=sh.topk_clusters,
              samples=sh.samples, seed=9, step=2)
    sel, rows, n_exact = S.santa_decode_select(q, kc, vc, summ, **kw)
    res = S.santa_decode(q, kc, vc, summ, **kw)
    sel, rows, out = sel.cpu().numpy(), rows.cpu().numpy(), res.out.cpu().numpy()
    n_exact = n_exact.cpu().numpy()
    for b in range(sh.batch):
        for kv in range(sh.num_kv_heads):
            K = w.keys[b, kv].float().numpy()
            V = w.values[b, kv].float().numpy()
            o = O.build_summary(K[:sh.sample_end], labels[b, kv].numpy(), sh.n_clusters)
            for hh in range(sh.group):
                h = kv * sh.group + hh
                qh = w.queries[0, b, h].numpy()
                chosen = O.select_topk(O.centroid_guess(o, qh, sh.scale), sh.topk_clusters)
                want = np.zeros(sh.n_clusters, np.uint8)
                want[chosen] = 1
                assert np.array_equal(sel[b, h], want), (b, kv, hh)
                assert int(n_exact[b, h]) == int(o.lengths[chosen].sum())
                n_rest = sh.sample_end - int(o.lengths[chosen].sum())
                ranks = O.philox_ranks(9, 2, b, h, sh.samples, n_rest)
                assert np.array_equal(rows[b, h], O.hybrid_positions(o, chosen, ranks))
                if (b + kv + hh) % 3 == 0:
                    r = O.decode_hybrid(qh, K, V, o, sh.sample_end, sh.topk_clusters, ranks,
                                        sh.scale)
                    assert np.abs(out[b, h] - r.out).max() < 2e-2


def _rest_positions(o, chosen, ranks):
    """O.hybrid_positions vectorised: the r-th member position outside the
    chosen clusters (checked against the oracle's loop on a few heads)."""
    sel = np.sort(np.asarray(chosen, np.int64))
    st, ln = o.starts[sel], o.lengths[sel]
    gap = st - (np.cumsum(ln) - ln)
    j = np.searchsorted(gap, np.asarray(ranks, np.int64), side="right")
    return np.asarray(ranks, np.int64) + np.concatenate(([0], np.cumsum(ln)))[j]


def test_full_size_128k_selection_bit_exact_and_output_close():
    """The Qwen3-8B batch-16 128K decode at full size (1024 clusters per KV
    head, top-32 + 512 samples): every head's selected set, n_exact and
    sample rows equal the oracle's; outputs of a head subset within
    max-abs 2e-2 / mean-abs 2e-3."""
    sh = QWEN3_8B_128K
    w = make_decode_workload(scaled_shape(sh, steps=1), device="cuda")
    labels = w.labels[:, :, :sh.sample_end].contiguous()
    summ = S.build_summary(w.keys, w.values, labels, sh.n_clusters, sample_end=sh.sample_end,
                           n_total=sh.context)
    q = w.queries[0].contiguous()
    kw = dict(mode="hybrid", n_total=sh.context, topk_clusters=sh.topk_clusters,
              samples=sh.samples, seed=21, step=3)
    sel, rows, n_exact = S.santa_decode_select(q, w.keys, w.values, summ, **kw)
    res = S.santa_decode(q, w.keys, w.values, summ, **kw)
    sel, rows, out = sel.cpu().numpy(), rows.cpu().numpy(), res.out.cpu().numpy()
    n_exact = n_exact.cpu().numpy()
    qn = q.cpu().numpy()
    lab_cpu = labels.cpu().numpy()
    del labels
    errs, loops = [], 0
    for b in range(sh.batch):
        for kv in range(sh.num_kv_heads):
            K = w.keys[b, kv].float().cpu().numpy()
            o = O.build_summary(K[:sh.sample_end], lab_cpu[b, kv], sh.n_clusters)
            V = None
            for hh in range(sh.group):
                h = kv * sh.group + hh
                chosen = O.select_topk(O.centroid_guess(o, qn[b, h], sh.scale), sh.topk_clusters)
                want = np.zeros(sh.n_clusters, np.uint8)
                want[chosen] = 1
                assert np.array_equal(sel[b, h], want), (b, h)
                assert int(n_exact[b, h]) == int(o.lengths[chosen].sum())
                n_rest = sh.sample_end - int(o.lengths[chosen].sum())
                ranks = O.philox_ranks(21, 3, b, h, sh.samples, n_rest)
                pos = _rest_positions(o, chosen, ranks)
                if loops < 4:  # the vectorised mapping is the oracle's loop
                    assert np.array_equal(pos, O.hybrid_positions(o, chosen, ranks))
                    loops += 1
                assert np.array_equal(rows[b, h], pos), (b, h)
                if (b * 3 + kv + hh) % 16 == 0:
                    if V is None:
                        V = w.values[b, kv].float().cpu().numpy()
                    r = O.decode_hybrid(qn[b, h], K, V, o, sh.sample_end, sh.topk_clusters,
                                        ranks, sh.scale)
                    errs.append(np.abs(out[b, h] - r.out))
    e = np.stack(errs)
    assert len(errs) >= 16
    assert e.max() < 2e-2 and e.mean() < 2e-3, (e.max(), e.mean())
