"""Host logic of the sequence-sharded decode, on CPU.

The shard bounds, the sample split and the Philox seeds are checked
directly; the two exchanges run on two and on four gloo ranks with the kernels replaced
by their oracle restatements (``shard_candidate_keys``, ``keys_threshold``,
``hybrid_shard_partial``, ``merge_shard_partials``), and the merged result
is compared with the oracle's sharded estimator over every shard's data.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import santa_oracle as O
from santapp_b200.attention.sharded import ShardExchange, shard_bounds, shard_seed, split_counts
from santapp_b200.synthetic import QWEN7B_32K, make_shard_workload, scaled_shape

SMALL = scaled_shape(QWEN7B_32K, name="shard-test", batch=1, num_query_heads=4, num_kv_heads=1,
                     head_dim=64, context=600, true_clusters=12, n_clusters=12,
                     topk_clusters=3, samples=20, recent_window=24, steps=1)


def test_shard_bounds_cover_and_balance():
    for n, k in [(10, 1), (10, 3), (32704, 8), (7, 7), (100, 6)]:
        b = shard_bounds(n, k)
        assert b[0][0] == 0 and b[-1][1] == n
        assert all(b[i][1] == b[i + 1][0] for i in range(k - 1))
        sizes = [e - s for s, e in b]
        assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    with pytest.raises(ValueError):
        shard_bounds(3, 4)


def test_split_counts_is_proportional_and_exact():
    assert split_counts(256, [1, 1, 1]) == [86, 85, 85]
    assert split_counts(7, [5, 0, 5]) == [4, 0, 3]
    rs = np.random.RandomState(0)
    for _ in range(200):
        w = rs.randint(0, 50, rs.randint(1, 9)).tolist()
        if sum(w) == 0:
            continue
        t = int(rs.randint(0, 1000))
        c = split_counts(t, w)
        assert sum(c) == t
        assert all(abs(ci - t * wi / sum(w)) < 1.0 for ci, wi in zip(c, w))


def test_shard_seeds_are_distinct():
    seeds = {shard_seed(s, r) for s in range(4) for r in range(32)}
    assert len(seeds) == 4 * 32
    assert shard_seed(5, 0) == 5


def test_shard_workload_partition():
    parts = [make_shard_workload(SMALL, r, 3) for r in range(3)]
    assert sum(p.sample_end for p in parts) == SMALL.sample_end
    assert sum(p.samples for p in parts) == SMALL.samples
    assert [p.cluster_base for p in parts] == [0, 4, 8]
    assert parts[-1].n_total == parts[-1].sample_end + SMALL.recent_window
    assert all(p.n_total == p.sample_end for p in parts[:-1])
    assert all(torch.equal(p.queries, parts[0].queries) for p in parts)


def _oracle_shard(p, b, kv):
    se = p.sample_end
    K = p.keys[b, kv].float().numpy()
    V = p.values[b, kv].float().numpy()
    summ = O.build_summary(K[:se], p.labels[b, kv].numpy(), p.n_clusters)
    return K, V, summ


def _ranks(p, summ, sel, h):
    n_rest = p.sample_end - int(sum(summ.lengths[c] for c in sel))
    rs = np.random.RandomState(1000 + h)
    return rs.randint(0, max(n_rest, 1), p.samples) if n_rest > 0 else np.zeros(0, np.int64)


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = SMALL
        parts = [make_shard_workload(sh, r, world) for r in range(world)]
        me = parts[rank]
        Hq, k, D = sh.num_query_heads, sh.topk_clusters, sh.head_dim
        ex = ShardExchange(rows=Hq, topk=k, head_dim=D, shard_index=rank, num_shards=world,
                           device="cpu")
        K, V, summ = _oracle_shard(me, 0, 0)
        qv = me.queries[0, 0].numpy()
        keys = np.concatenate([O.shard_candidate_keys(summ, qv[h], sh.scale, k, me.cluster_base)
                               for h in range(Hq)])
        ex.keys.copy_(torch.from_numpy(keys.view(np.int64)))
        all_keys = ex.exchange_keys().numpy().view(np.uint64).reshape(world, Hq, k)
        for h in range(Hq):
            thr = O.keys_threshold(all_keys[:, h], k)
            sel = O.selected_by_threshold(summ, qv[h], sh.scale, thr, me.cluster_base)
            part = O.hybrid_shard_partial(qv[h], K, V, summ, me.sample_end, me.n_total, sel,
                                          _ranks(me, summ, sel, h), sh.scale)
            ex.partial[h, :6] = torch.tensor(part[:6], dtype=torch.float32)
            ex.partial[h, 8:] = torch.from_numpy(part[6].astype(np.float32))
        allp = ex.exchange_partials().numpy()
        outs = []
        for h in range(Hq):
            parts_h = [(float(allp[r, h, 0]), float(allp[r, h, 1]), float(allp[r, h, 2]),
                        float(allp[r, h, 3]), float(allp[r, h, 4]), int(allp[r, h, 5]),
                        allp[r, h, 8:].astype(np.float64)) for r in range(world)]
            outs.append(O.merge_shard_partials(parts_h))
        if rank == 0:
            # the oracle's sharded estimator over every shard's data
            shards = [(*_oracle_shard(p, 0, 0)[:2], _oracle_shard(p, 0, 0)[2], p.sample_end,
                       p.n_total) for p in parts]
            bases = [p.cluster_base for p in parts]
            worst = 0.0
            for h in range(Hq):
                sels = O.shard_topk([s[2] for s in shards], qv[h], sh.scale, k, bases)
                ranks = [_ranks(p, s[2], sl, h) for p, s, sl in zip(parts, shards, sels)]
                ref = O.decode_hybrid_sharded(qv[h], shards, k, ranks, sh.scale, bases)
                out, lse, ess = outs[h]
                worst = max(worst, float(np.abs(out - ref.out).max()), abs(lse - ref.lse),
                            abs(ess - ref.ess))
            q.put(worst)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_exchange_and_merge_match_the_sharded_oracle(world):
    """Two ranks, and four (the shard count of the 4-GPU scaling run: every
    rank's keys in the threshold, the recent window on the last rank only)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    worst = q.get(timeout=5)
    # fp32 exchange buffers around float64 oracle partials
    assert worst < 1e-5, worst


def test_sharded_oracle_with_one_shard_is_the_hybrid_oracle():
    p = make_shard_workload(SMALL, 0, 1)
    K, V, summ = _oracle_shard(p, 0, 0)
    qv = p.queries[0, 0, 0].numpy()
    sel = O.select_topk(O.centroid_guess(summ, qv, SMALL.scale), SMALL.topk_clusters)
    ranks = _ranks(p, summ, sel, 0)
    a = O.decode_hybrid_sharded(qv, [(K, V, summ, p.sample_end, p.n_total)], SMALL.topk_clusters,
                                [ranks], SMALL.scale, [0])
    b = O.decode_hybrid(qv, K, V, summ, p.sample_end, SMALL.topk_clusters, ranks, SMALL.scale)
    assert np.allclose(a.out, b.out, atol=1e-12) and math.isclose(a.lse, b.lse, abs_tol=1e-12)
    assert math.isclose(a.ess, b.ess, rel_tol=1e-12)


def test_threshold_selection_lies_in_the_shards_own_candidates():
    """The threshold selection takes a shard's clusters from its own top-k
    candidate keys in the gathered list instead of scoring every centroid
    again.  The invariant behind it: a local cluster whose key reaches the
    global k-th key has fewer than k larger keys anywhere, so it is among the
    shard's own top-k.  Checked on random shards, with tied guesses (clusters
    that copy their neighbour's rows) broken by the lowest global id."""
    rng = np.random.default_rng(7)
    D, scale = 16, 0.25
    for _ in range(40):
        n, k = int(rng.integers(2, 6)), int(rng.integers(1, 9))
        summaries, bases, base = [], [], 0
        for _r in range(n):
            G = int(rng.integers(1, 14))
            rows = [rng.standard_normal((int(c), D)).astype(np.float32)
                    for c in rng.integers(1, 6, size=G)]
            for j in range(1, G):
                if rng.random() < 0.3:
                    rows[j] = rows[j - 1].copy()
            labels = np.repeat(np.arange(G), [len(x) for x in rows])
            summaries.append(O.build_summary(np.concatenate(rows), labels, G))
            bases.append(base)
            base += G
        q = rng.standard_normal(D).astype(np.float32)
        cands = [O.shard_candidate_keys(s, q, scale, k, b) for s, b in zip(summaries, bases)]
        thr = O.keys_threshold(np.stack(cands), k)
        want = O.shard_topk(summaries, q, scale, k, bases)
        for r, (s, b) in enumerate(zip(summaries, bases)):
            full = O.selected_by_threshold(s, q, scale, thr, b)
            own = sorted(0xFFFFFFFF - (int(x) & 0xFFFFFFFF) - b
                         for x in cands[r] if int(x) and int(x) >= thr)
            assert np.array_equal(full, want[r])
            assert own == full.tolist()
