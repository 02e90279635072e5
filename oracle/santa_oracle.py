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
