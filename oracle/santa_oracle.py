"""CPU restatement (numpy + the C helpers in santa_oracle.c) of the SANTA++ path.

TEST INFRASTRUCTURE ONLY.  This module is the oracle the CUDA library is
checked against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` import it; the product package never does.

What it restates (reference = santapp-ruler-bench/src/santapp_ruler):

* ``MiniBatchKMeansOracle.fit_predict``  attention/minibatch_kmeans.py:128-334,
  including greedy k-means++ (73-126), the numpy ``RandomState`` stream, the
  online means (226-239), low-count reassignment (241-267) and EWA early
  stopping (278-315).  The host-side control flow and every random draw are
  the reference's own; distances and sums follow the defined arithmetic of
  santa_oracle.c.
* ``build_summary``  attention/santapp.py:508-540 with a stable member sort.
* ``decode_topk``    attention/santapp.py:395-427 (budget walk, plain softmax).
* ``decode_guided``  attention/santapp.py:429-449 + 472-506 (IS combine).
* ``decode_uniform`` attention/santapp.py:459-468 + 472-506.
* ``decode_santa``   attention/santapp.py:450-458 + 472-506.
* ``decode_hybrid``  the "top-k clusters plus sampled tokens" estimator: exact
  softmax terms over the k highest-guess clusters (the topk ordering of
  santapp.py:397-401) and the recent window, plus uniform importance samples
  over the remaining old-prefix tokens with ``log r = -log(n_rest)`` (the
  uniform-mode weight of santapp.py:463-467 and the combine of 472-506).
* ``decode_hybrid_sharded`` the same estimator over contiguous sequence
  shards: one global top-k over all shards' clusters (``shard_topk``) and
  the sample budget stratified over the shards (the reference itself is
  single-GPU; this is the sharded decode's definition).
* ``fingerprints``   the clustering features of santapp.py:672-691 (key . probe
  query / sqrt(d), then a per-column z-score) under defined arithmetic.
* ``prefill_causal`` dense causal softmax attention (santapp.py:337-346 calls
  torch SDPA with is_causal=True).

Floating-point attention outputs are computed in float64 here; the CUDA path
computes in fp32 and is compared with a stated tolerance.  Cluster labels,
selections and sample positions are compared bit for bit.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libsanta_oracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")


def build_oracle() -> str:
    """Compile santa_oracle.c (gcc, oracle/Makefile) if it is not built."""
    src = os.path.join(_HERE, "santa_oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build_oracle()
        L = ctypes.CDLL(_LIB_PATH)
        i64, c_int, c_float = ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.or_fx_sum.argtypes = [_f32p, i64]
        L.or_fx_sum.restype = c_float
        L.or_fx_cumsum.argtypes = [_f32p, i64, _f32p]
        L.or_sqnorm.argtypes = [_f32p, i64, c_int, _f32p]
        L.or_assign.argtypes = [_f32p, _f32p, i64, _f32p, _f32p, c_int, c_int,
                                _i32p, _f32p]
        L.or_assign.restype = c_float
        L.or_kmeans_pp.argtypes = [_f32p, i64, c_int, c_int, c_int, i64, _f64p,
                                   _f32p, _i64p]
        L.or_minibatch_update.argtypes = [_f32p, _i32p, i64, c_int, c_int, _f32p,
                                          _f32p, _f32p, _f32p]
        L.or_cluster_means.argtypes = [_f32p, _i32p, i64, c_int, c_int, _f32p, _i64p]
        L.or_centroid_guess.argtypes = [_f32p, _f32p, c_int, c_int, _f32p, c_float,
                                        _f32p]
        L.or_philox4x32.argtypes = [_u32p, _u32p, _u32p]
        L.or_fingerprints.argtypes = [_f32p, i64, c_int, _f32p, i64, c_int, _i64p, c_int,
                                      c_float, _f32p]
        L.or_zscore.argtypes = [_f32p, i64, c_int]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# defined arithmetic helpers
# ---------------------------------------------------------------------------

def fx_sum(v) -> np.float32:
    v = _f32(v).ravel()
    return np.float32(lib().or_fx_sum(v, v.size))


def fx_cumsum(v) -> np.ndarray:
    v = _f32(v).ravel()
    out = np.empty_like(v)
    lib().or_fx_cumsum(v, v.size, out)
    return out


def sqnorm(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape[0], np.float32)
    lib().or_sqnorm(x, x.shape[0], x.shape[1], out)
    return out


def assign(x, centers, xx=None):
    """labels (int32), per-row minimum distance, fixed-point inertia (fp32)."""
    x = _f32(x)
    centers = _f32(centers)
    if xx is None:
        xx = sqnorm(x)
    cc = sqnorm(centers)
    labels = np.empty(x.shape[0], np.int32)
    mind = np.empty(x.shape[0], np.float32)
    inertia = lib().or_assign(x, _f32(xx), x.shape[0], centers, cc, centers.shape[0],
                              x.shape[1], labels, mind)
    return labels, mind, np.float32(inertia)


def philox4x32(counter, key) -> np.ndarray:
    out = np.empty(4, np.uint32)
    lib().or_philox4x32(np.asarray(counter, np.uint32), np.asarray(key, np.uint32), out)
    return out


# ---------------------------------------------------------------------------
# MiniBatchKMeans (minibatch_kmeans.py:32-334)
# ---------------------------------------------------------------------------

class MiniBatchKMeansOracle:
    """Host control flow and RNG stream of SklearnLikeTorchMiniBatchKMeans."""

    def __init__(self, n_clusters, *, batch_size=4096, n_init=1, max_iter=100,
                 tol=0.0, max_no_improvement=10, init_size=None,
                 reassignment_ratio=0.01, random_state=0):
        self.n_clusters = int(n_clusters)
        self.batch_size = int(batch_size)
        self.n_init = int(n_init)
        self.max_iter = int(max_iter)
        self.tol = float(tol)
        self.max_no_improvement = max_no_improvement
        self.init_size = init_size
        self.reassignment_ratio = float(reassignment_ratio)
        self.random_state = random_state

    def _kmeans_pp(self, x, rng):
        n, d = x.shape
        k = self.n_clusters
        trials = 2 + int(np.log(k))
        p = np.ones(n, dtype=np.float32)
        p /= p.sum(dtype=np.float32)
        first_id = int(rng.choice(n, p=p))
        uniforms = rng.uniform(size=(k - 1) * trials).astype(np.float64)
        centers = np.empty((k, d), np.float32)
        ids = np.empty(k, np.int64)
        lib().or_kmeans_pp(_f32(x), n, d, k, trials, first_id,
                           np.ascontiguousarray(uniforms), centers, ids)
        self.init_ids_ = ids
        return centers

    def fit_predict(self, x):
        x = _f32(x)
        if x.ndim != 2:
            raise ValueError(f"Expected [samples, features], got {tuple(x.shape)}")
        n = x.shape[0]
        k = self.n_clusters
        if n < k:
            raise ValueError(f"n_samples={n} must be >= n_clusters={k}")
        batch_size = min(self.batch_size, n)
        init_size = self.init_size
        if init_size is None:
            init_size = 3 * batch_size
            if init_size < k:
                init_size = 3 * k
        elif init_size < k:
            init_size = 3 * k
        init_size = min(int(init_size), n)

        rng = np.random.RandomState(self.random_state)
        validation_ids = rng.randint(0, n, init_size)
        x_valid = x[validation_ids]
        best_centers = None
        best_vi = None
        for _ in range(self.n_init):
            if init_size < n:
                init_ids = rng.randint(0, n, init_size)
                x_init = x[init_ids]
            else:
                x_init = x
            centers = self._kmeans_pp(x_init, rng)
            if self.n_init == 1:
                best_centers = centers
            else:
                _, _, vi = assign(x_valid, centers)
                vi = float(vi)
                if best_vi is None or vi < best_vi:
                    best_vi = vi
                    best_centers = centers.copy()
        centers = best_centers
        counts = np.zeros(k, np.float32)
        scaled_tol = (float(x.astype(np.float64).var(axis=0).mean()) * self.tol
                      if self.tol > 0.0 else 0.0)

        n_steps = (self.max_iter * n) // batch_size
        ewa = None
        ewa_min = None
        no_improvement = 0
        since = 0
        xx_all = sqnorm(x)
        step = -1
        self.reassign_steps_ = []
        for step in range(n_steps):
            since += batch_size
            random_reassign = bool((counts == 0).any() or since >= 10 * k)
            if random_reassign:
                since = 0
            batch_ids = rng.randint(0, n, batch_size)
            xb = x[batch_ids]
            labels, _, batch_inertia = assign(xb, centers, xx_all[batch_ids])
            centers_new = np.empty_like(centers)
            lib().or_minibatch_update(xb, labels, batch_size, x.shape[1], k, centers,
                                      counts, centers_new, np.empty(k, np.float32))
            if random_reassign and self.reassignment_ratio > 0.0:
                thresh = np.float32(np.float32(self.reassignment_ratio) * counts.max())
                to_reassign = counts < thresh
                if int(to_reassign.sum()) > 0.5 * batch_size:
                    keep = np.argsort(counts, kind="stable")[int(0.5 * batch_size):]
                    to_reassign[keep] = False
                n_re = int(to_reassign.sum())
                if n_re:
                    rows = rng.choice(batch_size, replace=False, size=n_re)
                    centers_new[to_reassign] = xb[rows]
                    counts[to_reassign] = counts[~to_reassign].min()
                    self.reassign_steps_.append(step)
            if scaled_tol > 0.0:
                diff = float(((centers_new.astype(np.float64) - centers) ** 2).sum())
            else:
                diff = 0.0
            centers = centers_new
            if step == 0:
                continue
            mean_inertia = float(batch_inertia) / batch_size
            if ewa is None:
                ewa = mean_inertia
            else:
                alpha = min(batch_size * 2.0 / (n + 1), 1.0)
                ewa = ewa * (1.0 - alpha) + mean_inertia * alpha
            if scaled_tol > 0.0 and diff <= scaled_tol:
                break
            if ewa_min is None or ewa < ewa_min:
                ewa_min = ewa
                no_improvement = 0
            else:
                no_improvement += 1
            if self.max_no_improvement is not None and no_improvement >= self.max_no_improvement:
                break

        self.cluster_centers_ = centers
        self.counts_ = counts
        self.n_steps_ = step + 1
        self.n_iter_ = int(np.ceil(self.n_steps_ * batch_size / n))
        labels, _, inertia = assign(x, centers, xx_all)
        self.labels_ = labels.astype(np.int64)
        self.inertia_ = float(inertia)
        return self.labels_


# ---------------------------------------------------------------------------
# cluster summary (santapp.py:508-540)
# ---------------------------------------------------------------------------

@dataclass
class Summary:
    members: np.ndarray      # int64 [N] token ids, sorted by (cluster, token)
    starts: np.ndarray       # int64 [G'] start of each non-empty cluster in members
    lengths: np.ndarray      # int64 [G']
    centroids: np.ndarray    # fp32 [G', D]
    log_n: np.ndarray        # fp32 [G'] = fl32(log(fl64(n)))
    active: np.ndarray       # int64 [G'] original cluster id of each row

    @property
    def num_groups(self) -> int:
        return int(self.lengths.size)


def log_count(n) -> np.ndarray:
    return np.log(np.asarray(n, dtype=np.float64)).astype(np.float32)


def build_summary(keys, labels, n_clusters) -> Summary:
    keys = _f32(keys)
    labels = np.asarray(labels).astype(np.int64)
    counts = np.bincount(labels, minlength=n_clusters)
    active = np.nonzero(counts > 0)[0]
    members = np.argsort(labels, kind="stable").astype(np.int64)
    full_starts = np.concatenate(([0], np.cumsum(counts[:-1]))).astype(np.int64)
    sums = np.empty((n_clusters, keys.shape[1]), np.float32)
    cnt = np.empty(n_clusters, np.int64)
    lib().or_cluster_means(keys, labels.astype(np.int32), keys.shape[0], keys.shape[1],
                           n_clusters, sums, cnt)
    return Summary(
        members=members,
        starts=full_starts[active],
        lengths=counts[active].astype(np.int64),
        centroids=np.ascontiguousarray(sums[active]),
        log_n=log_count(counts[active]),
        active=active.astype(np.int64),
    )


# ---------------------------------------------------------------------------
# selection (santapp.py:397-411)
# ---------------------------------------------------------------------------

def centroid_guess(summary: Summary, q, scale) -> np.ndarray:
    q = _f32(q)
    out = np.empty(summary.num_groups, np.float32)
    lib().or_centroid_guess(summary.centroids, summary.log_n, summary.num_groups,
                            summary.centroids.shape[1], q, np.float32(scale), out)
    return out


def rank_clusters(guess) -> np.ndarray:
    """Descending order of guess; equal guesses keep ascending cluster order."""
    return np.argsort(-np.asarray(guess, np.float32), kind="stable")


def select_budget(summary: Summary, guess, budget) -> np.ndarray:
    """Shortest prefix of the ranking whose member count reaches budget."""
    order = rank_clusters(guess)
    csum = np.cumsum(summary.lengths[order])
    n = int(np.searchsorted(csum, budget, side="left")) + 1
    return order[: min(n, order.size)]


def select_topk(guess, k) -> np.ndarray:
    return rank_clusters(guess)[:k]


def hybrid_positions(summary: Summary, selected, ranks) -> np.ndarray:
    """Map ranks in [0, n_rest) to member positions outside the selected clusters.

    Positions of the non-selected clusters are enumerated in ascending position
    order; rank r is the r-th of them."""
    sel = np.sort(np.asarray(selected, np.int64))
    starts = summary.starts[sel]
    lens = summary.lengths[sel]
    out = np.empty(len(ranks), np.int64)
    for i, r in enumerate(np.asarray(ranks, np.int64)):
        p = int(r)
        for s, l in zip(starts, lens):
            if p >= s:
                p += int(l)
            else:
                break
        out[i] = p
    return out


# ---------------------------------------------------------------------------
# decode estimators (santapp.py:365-506)
# ---------------------------------------------------------------------------

@dataclass
class DecodeResult:
    out: np.ndarray          # float64 [D]
    lse: float               # log(numerator weight total), see module doc
    n_exact: int             # exact old-prefix tokens (topk / hybrid)
    n_samples: int
    ess: float | None
    selected: np.ndarray | None = None
    token_ids: np.ndarray | None = None


def _scores(K, q, scale, idx):
    rows = np.asarray(K[idx], np.float64)
    return rows @ np.asarray(q, np.float64) * float(scale)


def _combine(q, K, V, scale, exact_idx, samp_idx, samp_logr, recent):
    """Self-normalised combine of santapp.py:472-506 with exact terms."""
    S = len(samp_idx)
    s_ex = _scores(K, q, scale, exact_idx) if len(exact_idx) else np.zeros(0)
    s_rec = _scores(K, q, scale, recent) if len(recent) else np.zeros(0)
    if S:
        lw = _scores(K, q, scale, samp_idx) - np.asarray(samp_logr, np.float64)
    else:
        lw = np.zeros(0)
    allv = np.concatenate((s_ex, s_rec, lw))
    m = allv.max()
    w_ex = np.exp(s_ex - m)
    w_rec = np.exp(s_rec - m)
    w_s = np.exp(lw - m) / S if S else np.zeros(0)
    Vf = np.asarray(V, np.float64)
    num = np.zeros(V.shape[1])
    if len(exact_idx):
        num += w_ex @ Vf[exact_idx]
    if len(recent):
        num += w_rec @ Vf[recent]
    if S:
        num += w_s @ Vf[samp_idx]
    den = w_ex.sum() + w_rec.sum() + w_s.sum()
    ess = None
    if S:
        nw = np.exp(lw - lw.max())
        ess = float(nw.sum() ** 2 / (nw ** 2).sum() / S)
    return num / den, float(m + math.log(den)), ess


def _recent(sample_end, n_total):
    return np.arange(sample_end, n_total, dtype=np.int64)


def decode_topk(q, K, V, summary: Summary, sample_end, budget, scale) -> DecodeResult:
    guess = centroid_guess(summary, q, scale)
    sel = select_budget(summary, guess, budget)
    idx = np.concatenate([summary.members[summary.starts[g]: summary.starts[g] + summary.lengths[g]]
                          for g in sel]) if len(sel) else np.zeros(0, np.int64)
    out, lse, _ = _combine(q, K, V, scale, idx, [], [], _recent(sample_end, K.shape[0]))
    return DecodeResult(out, lse, int(idx.size), 0, None, sel, idx)


def group_probability(summary: Summary, q, scale) -> np.ndarray:
    g = centroid_guess(summary, q, scale).astype(np.float64)
    e = np.exp(g - g.max())
    return e / e.sum()


def decode_guided(q, K, V, summary: Summary, sample_end, groups, within, scale) -> DecodeResult:
    groups = np.asarray(groups, np.int64)
    within = np.asarray(within, np.int64)
    p = group_probability(summary, q, scale)
    pos = summary.starts[groups] + within
    idx = summary.members[pos]
    logr = np.log(p[groups]) - np.log(summary.lengths[groups].astype(np.float64))
    out, lse, ess = _combine(q, K, V, scale, [], idx, logr, _recent(sample_end, K.shape[0]))
    return DecodeResult(out, lse, 0, len(idx), ess, None, idx)


def decode_uniform(q, K, V, sample_end, idx, scale) -> DecodeResult:
    idx = np.asarray(idx, np.int64)
    logr = np.full(len(idx), -math.log(sample_end))
    out, lse, ess = _combine(q, K, V, scale, [], idx, logr, _recent(sample_end, K.shape[0]))
    return DecodeResult(out, lse, 0, len(idx), ess, None, idx)


def decode_santa(q, K, V, sample_end, idx, scale) -> DecodeResult:
    idx = np.asarray(idx, np.int64)
    old = _scores(K, q, scale, np.arange(sample_end))
    mx = old.max()
    lse_old = mx + math.log(np.exp(old - mx).sum())
    logr = old[idx] - lse_old
    out, lse, ess = _combine(q, K, V, scale, [], idx, logr, _recent(sample_end, K.shape[0]))
    return DecodeResult(out, lse, 0, len(idx), ess, None, idx)


def decode_hybrid(q, K, V, summary: Summary, sample_end, topk, ranks, scale) -> DecodeResult:
    """Exact top-k clusters + uniform samples (given as ranks) over the rest."""
    guess = centroid_guess(summary, q, scale)
    sel = select_topk(guess, topk)
    exact_pos = np.concatenate([np.arange(summary.starts[g], summary.starts[g] + summary.lengths[g])
                                for g in sel]) if len(sel) else np.zeros(0, np.int64)
    exact_idx = summary.members[exact_pos]
    n_rest = int(sample_end - exact_pos.size)
    ranks = np.asarray(ranks, np.int64)
    if n_rest > 0 and ranks.size:
        pos = hybrid_positions(summary, sel, ranks)
        samp_idx = summary.members[pos]
        logr = np.full(ranks.size, -math.log(n_rest))
    else:
        samp_idx = np.zeros(0, np.int64)
        logr = np.zeros(0)
    out, lse, ess = _combine(q, K, V, scale, exact_idx, samp_idx, logr,
                             _recent(sample_end, K.shape[0]))
    return DecodeResult(out, lse, int(exact_idx.size), int(samp_idx.size), ess, sel, samp_idx)


# ---------------------------------------------------------------------------
# hybrid decode over sequence shards
# ---------------------------------------------------------------------------

def shard_topk(summaries, q, scale, k, bases) -> list:
    """Global top-k over the clusters of all shards (cluster row c of shard r
    has global id bases[r] + c): guess descending, lowest global id first on
    ties, the ranking of select_topk over the concatenated clusters.  Returns
    the selected local rows of every shard, ascending."""
    keys = []
    for r, s in enumerate(summaries):
        gs = centroid_guess(s, q, scale)
        keys += [(float(gs[c]), int(bases[r]) + c, r, c) for c in range(s.num_groups)]
    keys.sort(key=lambda t: (-t[0], t[1]))
    top = keys[:k]
    return [np.array(sorted(c for (_, _, rr, c) in top if rr == r), np.int64)
            for r in range(len(summaries))]


def order_key(f) -> int:
    """Order-preserving 32-bit image of an fp32 value (-0 taken as +0)."""
    b = int(np.float32(np.float32(f) + np.float32(0.0)).view(np.uint32))
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def shard_candidate_keys(summary: Summary, q, scale, k, base) -> np.ndarray:
    """A shard's candidate keys for one query head, descending, 0-padded to
    k: order_key(guess) << 32 | (0xFFFFFFFF - global id)."""
    gs = centroid_guess(summary, q, scale)
    keys = sorted(((order_key(gs[c]) << 32) | (0xFFFFFFFF - (int(base) + c))
                   for c in range(summary.num_groups)), reverse=True)[:k]
    return np.array(keys + [0] * (k - len(keys)), np.uint64)


def keys_threshold(all_keys, k) -> int:
    """k-th largest of the gathered keys (every real key when fewer)."""
    real = sorted((int(x) for x in np.asarray(all_keys, np.uint64).ravel() if int(x)),
                  reverse=True)
    return real[k - 1] if len(real) >= k else 1


def selected_by_threshold(summary: Summary, q, scale, thr, base) -> np.ndarray:
    gs = centroid_guess(summary, q, scale)
    return np.array([c for c in range(summary.num_groups)
                     if ((order_key(gs[c]) << 32) | (0xFFFFFFFF - (int(base) + c))) >= thr],
                    np.int64)


def hybrid_shard_partial(q, K, V, summary: Summary, sample_end, n_total, selected, ranks, scale):
    """Shard partial (m, l, ms, e1, e2, n_samples, o[D]) in log2 units,
    float64: l = sum 2^(lw - m), o = sum 2^(lw - m) v over the shard's exact
    rows, recent rows and stratified samples (lw in log2 units)."""
    sel = np.asarray(selected, np.int64)
    pos = (np.concatenate([np.arange(summary.starts[g], summary.starts[g] + summary.lengths[g])
                           for g in sel]) if len(sel) else np.zeros(0, np.int64))
    ex = summary.members[pos]
    rec = _recent(sample_end, n_total)
    idx = np.concatenate([ex, rec]).astype(np.int64)
    lw = _scores(K, q, scale, idx) if idx.size else np.zeros(0)
    rk = np.asarray(ranks, np.int64)
    n_rest = int(sample_end - ex.size)
    slw = np.zeros(0)
    if n_rest > 0 and rk.size:
        sidx = summary.members[hybrid_positions(summary, sel, rk)]
        slw = _scores(K, q, scale, sidx) + math.log(n_rest) - math.log(rk.size)
        idx = np.concatenate([idx, sidx])
        lw = np.concatenate([lw, slw])
    lw2, slw2 = lw / math.log(2.0), slw / math.log(2.0)
    D = np.asarray(V).shape[1]
    if lw2.size == 0:
        return (-math.inf, 0.0, -math.inf, 0.0, 0.0, int(rk.size if n_rest > 0 else 0),
                np.zeros(D))
    m = lw2.max()
    w = np.exp2(lw2 - m)
    o = w @ np.asarray(V, np.float64)[idx]
    ms, e1, e2 = -math.inf, 0.0, 0.0
    if slw2.size:
        ms = slw2.max()
        we = np.exp2(slw2 - ms)
        e1, e2 = float(we.sum()), float((we ** 2).sum())
    return (float(m), float(w.sum()), float(ms), e1, e2, int(slw2.size), o)


def merge_shard_partials(parts):
    """LSE merge of hybrid_shard_partial results -> (out, lse, ess)."""
    M = max((p[0] for p in parts if p[1] > 0), default=-math.inf)
    L, o = 0.0, 0.0
    for p in parts:
        if p[1] > 0:
            f = 2.0 ** (p[0] - M)
            L += p[1] * f
            o = o + p[6] * f
    MS = max((p[2] for p in parts if p[3] > 0), default=-math.inf)
    E1 = sum(p[3] * 2.0 ** (p[2] - MS) for p in parts if p[3] > 0)
    E2 = sum(p[4] * 4.0 ** (p[2] - MS) for p in parts if p[3] > 0)
    ns = sum(p[5] for p in parts)
    out = o / L if L > 0 else np.zeros_like(parts[0][6])
    lse = (M + math.log2(L)) * math.log(2.0) if L > 0 else -math.inf
    ess = (E1 * E1 / E2) / ns if ns > 0 and E2 > 0 else 0.0
    return out, lse, ess


def decode_hybrid_sharded(q, shards, k, ranks, scale, bases) -> DecodeResult:
    """The hybrid estimator with the sample budget stratified over shards.

    shards[r] = (K_r, V_r, summary_r, sample_end_r, n_total_r): shard r's
    token rows, its summary and its old-prefix / total lengths.  ranks[r] are
    shard r's sample ranks in [0, n_rest_r); a sample of shard r weighs
    n_rest_r / len(ranks[r]) (log r = log(S_r) - log(n_rest_r)).  Exact terms:
    the global top-k clusters (shard_topk) and every shard's recent rows."""
    sel = shard_topk([s[2] for s in shards], q, scale, k, bases)
    terms_s, terms_v, samp_lw = [], [], []
    n_exact = 0
    for r, (K, V, summ, se, nt) in enumerate(shards):
        sr = sel[r]
        pos = (np.concatenate([np.arange(summ.starts[g], summ.starts[g] + summ.lengths[g])
                               for g in sr]) if len(sr) else np.zeros(0, np.int64))
        ex = summ.members[pos]
        n_exact += ex.size
        rec = _recent(se, nt)
        for idx in (ex, rec):
            if len(idx):
                terms_s.append(_scores(K, q, scale, idx))
                terms_v.append(np.asarray(V, np.float64)[idx])
        rk = np.asarray(ranks[r], np.int64)
        n_rest = int(se - ex.size)
        if n_rest > 0 and rk.size:
            sidx = summ.members[hybrid_positions(summ, sr, rk)]
            lw = _scores(K, q, scale, sidx) + math.log(n_rest) - math.log(rk.size)
            terms_s.append(lw)
            terms_v.append(np.asarray(V, np.float64)[sidx])
            samp_lw.append(lw)
    s_all = np.concatenate(terms_s)
    v_all = np.concatenate(terms_v)
    m = s_all.max()
    w = np.exp(s_all - m)
    out = w @ v_all / w.sum()
    ess = None
    if samp_lw:
        lw = np.concatenate(samp_lw)
        nw = np.exp(lw - lw.max())
        ess = float(nw.sum() ** 2 / (nw ** 2).sum() / lw.size)
    return DecodeResult(out, float(m + math.log(w.sum())), n_exact,
                        int(sum(len(x) for x in samp_lw)), ess, sel, None)


# ---------------------------------------------------------------------------
# on-device sampler restatement (Philox4x32-10)
# ---------------------------------------------------------------------------

def philox_ranks(seed: int, step: int, b: int, h: int, n_samples: int, n_rest: int) -> np.ndarray:
    """Sample ranks the CUDA sampler draws for (seed, step, batch b, q-head h):
    word i of the stream is word (i % 4) of Philox4x32-10 with counter
    (i // 4, h, b, step) and key (seed lo, seed hi); rank = (word * n_rest) >> 32."""
    key = np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], np.uint32)
    out = np.empty(n_samples, np.int64)
    for blk in range((n_samples + 3) // 4):
        w = philox4x32(np.array([blk, h, b, step], np.uint32), key)
        for j in range(4):
            i = blk * 4 + j
            if i < n_samples:
                out[i] = (int(w[j]) * int(n_rest)) >> 32
    return out


# ---------------------------------------------------------------------------
# key fingerprints (santapp.py:598-690)
# ---------------------------------------------------------------------------

def fingerprints(keys, q_group, probes, normalize=True) -> np.ndarray:
    """keys [N, D], q_group [g, T, D] rotated fp32 queries of the KV head's
    query heads, probes [P] -> [N, g*P] (z-scored per column if normalize)."""
    keys = _f32(keys)
    q_group = _f32(q_group)
    probes = np.ascontiguousarray(np.asarray(probes, np.int64))
    n, d = keys.shape
    g, T, _ = q_group.shape
    out = np.empty((n, g * probes.size), np.float32)
    lib().or_fingerprints(keys, n, d, q_group, T * d, g, probes, probes.size,
                          np.float32(math.sqrt(d)), out)
    if normalize:
        lib().or_zscore(out, n, out.shape[1])
    return out


# ---------------------------------------------------------------------------
# dense causal prefill (santapp.py:337-346 -> torch SDPA, is_causal=True)
# ---------------------------------------------------------------------------

def prefill_causal(q, k, v, scale) -> np.ndarray:
    """q [Hq,T,D], k/v [Hkv,T,D] -> out [Hq,T,D] float64 (GQA by head // group)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    Hq, T, _ = q.shape
    g = Hq // k.shape[0]
    out = np.empty_like(q)
    mask = np.triu(np.ones((T, T), bool), 1)
    for h in range(Hq):
        s = q[h] @ k[h // g].T * scale
        s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[h] = p @ v[h // g]
    return out
