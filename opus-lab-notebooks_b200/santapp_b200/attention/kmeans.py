"""MiniBatchKMeans on the sm_100a kernels of libsanta_b200.so.

Host-side mirror of ``SklearnLikeTorchMiniBatchKMeans`` and
``gpu_minibatch_labels`` (santapp_ruler/attention/minibatch_kmeans.py:32-347):
same constructor, same attributes after ``fit_predict``.  The control flow
and every random draw are the reference's (numpy ``RandomState``, in the
reference's order); the arithmetic that depends on the data — squared norms,
nearest-centre assignment and inertia, greedy k-means++, the mini-batch
centre update, the low-count reassignment — runs in the CUDA kernels
(include/santa_b200.h, csrc/kmeans.cu) under defined arithmetic, so labels
and centres are reproducible bit for bit.

Per mini-batch step the host uploads the step's batch ids and reads back the
counts and the batch inertia into pinned memory, waiting on an event behind
the copies (the early-stopping rule and the reassignment rule of
minibatch_kmeans.py:241-315 need them before the next step's draws), as the
reference's control flow requires.  The greedy k-means++ seeding runs on
the device with no host round trip (two launches per centre).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _lib
from .santapp import _require_cuda

__all__ = ["SklearnLikeTorchMiniBatchKMeans", "gpu_minibatch_labels"]


def _fx_value(words: np.ndarray) -> float:
    """fl32(fl64(hi) + fl64(lo) * 2^-64) of a Q64.64 sum held as (lo, hi)."""
    lo, hi = int(words[0]), int(words[1])
    return float(np.float32(float(hi) + float(lo) * 2.0 ** -64))


class SklearnLikeTorchMiniBatchKMeans:
    def __init__(self, n_clusters, *, batch_size=4096, n_init=1, max_iter=100, tol=0.0,
                 max_no_improvement=10, init_size=None, reassignment_ratio=0.01,
                 random_state=0, verbose=False):
        self.n_clusters = int(n_clusters)
        self.batch_size = int(batch_size)
        self.n_init = int(n_init)
        self.max_iter = int(max_iter)
        self.tol = float(tol)
        self.max_no_improvement = max_no_improvement
        self.init_size = init_size
        self.reassignment_ratio = float(reassignment_ratio)
        self.random_state = random_state
        self.verbose = bool(verbose)

    # ---- kernel calls ------------------------------------------------------
    def _sqnorm(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
        _lib.check("santa_kmeans_sqnorm", self._lib.santa_kmeans_sqnorm(
            x.data_ptr(), x.shape[0], x.shape[1], out.data_ptr(), _lib.stream_handle()))
        return out

    def _assign(self, x, rows, xx, n, centers, labels=None):
        """Labels (int32, device) and the fixed-point inertia (host float)."""
        cc = self._sqnorm(centers)
        if labels is None:
            labels = torch.empty(n, dtype=torch.int32, device=x.device)
        self._fx.zero_()
        _lib.check("santa_kmeans_assign", self._lib.santa_kmeans_assign(
            x.data_ptr(), _lib.ptr(rows), xx.data_ptr(), n, x.shape[1], centers.data_ptr(),
            cc.data_ptr(), self.n_clusters, labels.data_ptr(), None, self._fx.data_ptr(),
            _lib.stream_handle()))
        return labels

    def _kmeans_pp(self, x, rows, xx, n, rng):
        """_greedy_kmeans_plus_plus (minibatch_kmeans.py:73-126): the draws
        here, the distances and potentials on the device."""
        k, d = self.n_clusters, x.shape[1]
        trials = 2 + int(np.log(k))
        p = np.ones(n, dtype=np.float32)
        p /= p.sum(dtype=np.float32)
        first_id = int(rng.choice(n, p=p))
        uniforms = rng.uniform(size=(k - 1) * trials).astype(np.float64)
        u_dev = torch.from_numpy(np.ascontiguousarray(uniforms) if uniforms.size
                                 else np.zeros(1)).to(x.device)
        centers = torch.empty(k, d, dtype=torch.float32, device=x.device)
        chosen = torch.empty(k, dtype=torch.int64, device=x.device)
        nbytes = ctypes.c_size_t()
        _lib.check("santa_kmeans_plusplus_workspace_bytes",
                   self._lib.santa_kmeans_plusplus_workspace_bytes(n, trials,
                                                                  ctypes.byref(nbytes)))
        ws = torch.empty(max(1, nbytes.value), dtype=torch.uint8, device=x.device)
        _lib.check("santa_kmeans_plusplus", self._lib.santa_kmeans_plusplus(
            x.data_ptr(), _lib.ptr(rows), xx.data_ptr(), n, d, k, trials, first_id,
            u_dev.data_ptr(), centers.data_ptr(), chosen.data_ptr(), ws.data_ptr(),
            nbytes.value, _lib.stream_handle()))
        self.init_ids_ = chosen
        return centers

    # ---- fit ---------------------------------------------------------------
    def fit_predict(self, x: torch.Tensor) -> torch.Tensor:
        """Labels of every row of ``x`` ([samples, features] CUDA tensor)."""
        _require_cuda("x", x)
        if x.ndim != 2:
            raise ValueError(f"Expected [samples, features], got {tuple(x.shape)}")
        if x.dtype != torch.float32:
            x = x.float()
        x = x.contiguous()
        d_in = x.shape[1]
        if d_in % 4:
            # zero feature columns leave every dot, norm and sum unchanged
            # (fmaf(0, 0, acc) == acc); the assignment kernel reads float4
            x = torch.nn.functional.pad(x, (0, 4 - d_in % 4))
        self._lib = _lib.load()
        dev = x.device
        n, d = x.shape
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

        self._fx = torch.zeros(2, dtype=torch.int64, device=dev)
        rng = np.random.RandomState(self.random_state)
        validation_ids = rng.randint(0, n, init_size)
        xx_all = self._sqnorm(x)
        best_centers, best_vi = None, None
        for _ in range(self.n_init):
            if init_size < n:
                init_ids = torch.from_numpy(rng.randint(0, n, init_size).astype(np.int64))
                centers = self._kmeans_pp(x, init_ids.to(dev), xx_all, init_size, rng)
            else:
                centers = self._kmeans_pp(x, None, xx_all, n, rng)
            if self.n_init == 1:
                best_centers = centers
            else:
                vid = torch.from_numpy(validation_ids.astype(np.int64)).to(dev)
                self._assign(x, vid, xx_all, init_size, centers)
                vi = _fx_value(self._fx.cpu().numpy().view(np.uint64))
                if best_vi is None or vi < best_vi:
                    best_vi, best_centers = vi, centers.clone()
        centers = best_centers
        centers_new = torch.empty_like(centers)
        counts = torch.zeros(k, dtype=torch.float32, device=dev)
        counts_host = np.zeros(k, np.float32)
        scaled_tol = 0.0
        if self.tol > 0.0:
            scaled_tol = float(x[:, :d_in].double().var(dim=0, unbiased=False).mean().item()) \
                * self.tol

        ub = ctypes.c_size_t()
        _lib.check("santa_kmeans_update_workspace_bytes",
                   self._lib.santa_kmeans_update_workspace_bytes(batch_size, k, ctypes.byref(ub)))
        uws = torch.empty(max(1, ub.value), dtype=torch.uint8, device=dev)
        ids_host = torch.empty(batch_size, dtype=torch.int64).pin_memory()
        ids_dev = torch.empty(batch_size, dtype=torch.int64, device=dev)
        labels_b = torch.empty(batch_size, dtype=torch.int32, device=dev)
        back = torch.empty(k + 4, dtype=torch.float32).pin_memory()
        landed = torch.cuda.Event()  # the step's read-back is in pinned memory
        stream = _lib.stream_handle()

        n_steps = (self.max_iter * n) // batch_size
        ewa = ewa_min = None
        no_improvement = 0
        since = 0
        step = -1
        self.reassign_steps_ = []
        for step in range(n_steps):
            since += batch_size
            random_reassign = bool((counts_host == 0).any() or since >= 10 * k)
            if random_reassign:
                since = 0
            ids_host.numpy()[:] = rng.randint(0, n, batch_size)
            ids_dev.copy_(ids_host, non_blocking=True)
            self._assign(x, ids_dev, xx_all, batch_size, centers, labels_b)
            _lib.check("santa_kmeans_update", self._lib.santa_kmeans_update(
                x.data_ptr(), ids_dev.data_ptr(), batch_size, d, labels_b.data_ptr(), k,
                centers.data_ptr(), counts.data_ptr(), centers_new.data_ptr(), None,
                uws.data_ptr(), ub.value, stream))
            back[:k].copy_(counts, non_blocking=True)
            back[k:].copy_(self._fx.view(torch.float32), non_blocking=True)
            landed.record()
            landed.synchronize()
            counts_host = back[:k].numpy().copy()
            batch_inertia = _fx_value(back[k:].numpy().view(np.uint64))
            if random_reassign and self.reassignment_ratio > 0.0:
                thresh = np.float32(np.float32(self.reassignment_ratio) * counts_host.max())
                to_reassign = counts_host < thresh
                if int(to_reassign.sum()) > 0.5 * batch_size:
                    keep = np.argsort(counts_host, kind="stable")[int(0.5 * batch_size):]
                    to_reassign[keep] = False
                n_re = int(to_reassign.sum())
                if n_re:
                    rows = rng.choice(batch_size, replace=False, size=n_re)
                    new_count = np.float32(counts_host[~to_reassign].min())
                    cl = torch.from_numpy(np.nonzero(to_reassign)[0].astype(np.int32)).to(dev)
                    br = torch.from_numpy(rows.astype(np.int32)).to(dev)
                    _lib.check("santa_kmeans_reassign", self._lib.santa_kmeans_reassign(
                        x.data_ptr(), ids_dev.data_ptr(), br.data_ptr(), cl.data_ptr(), n_re, d,
                        centers_new.data_ptr(), counts.data_ptr(), float(new_count), stream))
                    counts_host[to_reassign] = new_count
                    self.reassign_steps_.append(step)
            if scaled_tol > 0.0:
                diff = float(((centers_new.double() - centers.double()) ** 2).sum().item())
            else:
                diff = 0.0
            centers, centers_new = centers_new, centers
            if step == 0:
                continue
            mean_inertia = batch_inertia / batch_size
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

        self.cluster_centers_ = centers[:, :d_in].contiguous()
        self.counts_ = counts
        self.n_steps_ = step + 1
        self.n_iter_ = int(np.ceil(self.n_steps_ * batch_size / n))
        labels = self._assign(x, None, xx_all, n, centers)
        self.labels_ = labels.long()
        self.inertia_ = _fx_value(self._fx.cpu().numpy().view(np.uint64))
        if self.verbose:
            print(f"GPU MiniBatchKMeans: {self.n_steps_} mini-batches, "
                  f"{self.n_iter_} effective epochs")
        return self.labels_


def gpu_minibatch_labels(x: torch.Tensor, n_clusters: int, seed: int) -> torch.Tensor:
    """The notebook's sklearn parameters (minibatch_kmeans.py:337-347)."""
    return SklearnLikeTorchMiniBatchKMeans(
        n_clusters=n_clusters, batch_size=4096, n_init=1, max_iter=100, tol=0.0,
        max_no_improvement=10, init_size=None, reassignment_ratio=0.01,
        random_state=seed).fit_predict(x)
