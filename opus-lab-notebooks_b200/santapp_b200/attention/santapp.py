"""SANTA++ attention entry points backed by the sm_100a CUDA library.

Host-side mirror of santapp_ruler/attention/santapp.py for the hot path:

* ``ClusterSummary`` / ``build_summary`` replace ``ClusterSummary`` and
  ``SantaPlusEngine._build_summary`` (santapp.py:53-63, 508-540), batched over
  (batch, KV head) and extended with the cluster-sorted K/V copy the decode
  kernel streams from.
* ``santa_decode`` replaces ``SantaPlusEngine._approximate_attention``
  (santapp.py:365-506) for every (batch, query head) of a decode step in one
  call, in the reference's modes ``topk``, ``guided``, ``uniform``, ``santa``
  and the ``hybrid`` estimator (exact top-k clusters + uniform samples of
  the remaining prefix).
* ``DecodeTrafficTracker`` keeps the reference's draw-count accounting
  (santapp.py:80-142).

Every function runs on CUDA tensors only and raises on anything else; the
work happens in libsanta_b200.so (include/santa_b200.h).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _lib
from .paged import PagedKVCache

__all__ = [
    "ClusterSummary", "build_summary", "santa_decode", "DecodeResult", "DecodeWorkspace",
    "DecodeTrafficTracker", "santa_decode_select", "allocate_summary", "DecodeStep",
    "GraphedDecodeStep",
]


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (the SANTA++ kernels have no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _kv_dtype(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    raise ValueError(f"KV cache dtype {t.dtype} unsupported (bf16 or fp32)")


def _kv(key_cache, value_cache) -> tuple[torch.Tensor, torch.Tensor]:
    """The K and V tensors handed to the C ABI: contiguous caches, or the page
    pools of a PagedKVCache (passed as ``key_cache`` with ``value_cache``
    None)."""
    if isinstance(key_cache, PagedKVCache):
        if value_cache is not None and value_cache is not key_cache:
            raise ValueError("with a PagedKVCache, pass value_cache=None")
        return key_cache.key_pool, key_cache.value_pool
    _require_cuda("key_cache", key_cache)
    _require_cuda("value_cache", value_cache)
    if value_cache.shape != key_cache.shape or value_cache.dtype != key_cache.dtype:
        raise ValueError("key and value caches must have the same shape and dtype")
    return key_cache, value_cache


def _geometry(key_cache, num_query_heads: int, n_total: int,
              sample_end: int) -> _lib.SantaGeometry:
    """SantaGeometry of a contiguous ``[B, Hkv, capacity, D]`` cache or of a
    PagedKVCache (the table pointer is set from the cache object)."""
    paged = isinstance(key_cache, PagedKVCache)
    if not paged and key_cache.dim() != 4:
        raise ValueError("key/value cache must be [batch, kv_heads, capacity, head_dim]")
    B, Hkv, cap, D = key_cache.shape
    if num_query_heads % Hkv:
        raise ValueError("Query heads must be divisible by KV heads.")
    if not 0 < sample_end <= n_total:
        raise RuntimeError(
            f"Invalid sampled-prefix boundary {sample_end} for cache length {n_total}.")
    if n_total > cap:
        raise RuntimeError(f"cache length {n_total} exceeds capacity {cap}")
    geo = _lib.SantaGeometry(B, Hkv, num_query_heads // Hkv, D, cap, n_total, sample_end,
                             _kv_dtype(key_cache.key_pool if paged else key_cache))
    if paged:
        key_cache.fill_geometry(geo)
    return geo


# ---------------------------------------------------------------------------
# cluster summary
# ---------------------------------------------------------------------------

@dataclass
class ClusterSummary:
    """Cluster layout of the old prefix for every (batch, KV head).

    Row ``i < n_groups[b, kv]`` of ``starts`` / ``lengths_long`` /
    ``key_centroids`` describes the i-th non-empty cluster in ascending
    cluster id, as in the reference.  ``sorted_key`` / ``sorted_value`` hold
    the prefix rows in ``members`` order, so cluster i is the contiguous run
    ``[starts[i], starts[i] + lengths[i])``."""

    members: torch.Tensor        # [B, Hkv, N] int32 token ids
    positions: torch.Tensor      # [B, Hkv, N] int32 position of each token in members
    starts: torch.Tensor         # [B, Hkv, G] int32
    lengths_long: torch.Tensor   # [B, Hkv, G] int32
    log_n: torch.Tensor          # [B, Hkv, G] fp32
    key_centroids: torch.Tensor  # [B, Hkv, G, D] fp32
    n_groups: torch.Tensor       # [B, Hkv] int32
    sorted_key: torch.Tensor     # [B, Hkv, N, D]
    sorted_value: torch.Tensor   # [B, Hkv, N, D]
    max_groups: int
    sample_end: int

    @property
    def lengths_float(self) -> torch.Tensor:
        return self.lengths_long.float()

    def as_c(self) -> _lib.SantaSummary:
        return _lib.SantaSummary(
            self.members.data_ptr(), self.positions.data_ptr(), self.starts.data_ptr(),
            self.lengths_long.data_ptr(), self.log_n.data_ptr(), self.key_centroids.data_ptr(),
            self.n_groups.data_ptr(), self.sorted_key.data_ptr(), self.sorted_value.data_ptr(),
            self.max_groups)

    def head(self, b: int, kv: int) -> dict:
        """Reference-shaped fields of one (batch, KV head) (int64 like santapp.py:511-540)."""
        n = int(self.n_groups[b, kv])
        return {
            "members": self.members[b, kv].long(),
            "starts": self.starts[b, kv, :n].long(),
            "lengths_long": self.lengths_long[b, kv, :n].long(),
            "lengths_float": self.lengths_long[b, kv, :n].float(),
            "key_centroids": self.key_centroids[b, kv, :n],
        }

    def segment(self, b: int, kv: int) -> "ClusterSummary":
        """The summary of one (batch, KV head) as a one-segment summary
        (views, no copy), for a decode call on that head alone."""
        sl = (slice(b, b + 1), slice(kv, kv + 1))
        return ClusterSummary(
            members=self.members[sl], positions=self.positions[sl], starts=self.starts[sl],
            lengths_long=self.lengths_long[sl], log_n=self.log_n[sl],
            key_centroids=self.key_centroids[sl], n_groups=self.n_groups[sl],
            sorted_key=self.sorted_key[sl], sorted_value=self.sorted_value[sl],
            max_groups=self.max_groups, sample_end=self.sample_end)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (
            self.members, self.positions, self.starts, self.lengths_long, self.log_n,
            self.key_centroids, self.n_groups, self.sorted_key, self.sorted_value))


def allocate_summary(batch: int, num_kv_heads: int, sample_end: int, head_dim: int,
                     n_clusters: int, kv_dtype: torch.dtype, device) -> ClusterSummary:
    B, H, N, D, G = batch, num_kv_heads, sample_end, head_dim, n_clusters
    i32 = dict(dtype=torch.int32, device=device)
    return ClusterSummary(
        members=torch.empty(B, H, N, **i32),
        positions=torch.empty(B, H, N, **i32),
        starts=torch.empty(B, H, G, **i32),
        lengths_long=torch.empty(B, H, G, **i32),
        log_n=torch.empty(B, H, G, dtype=torch.float32, device=device),
        key_centroids=torch.zeros(B, H, G, D, dtype=torch.float32, device=device),
        n_groups=torch.empty(B, H, **i32),
        sorted_key=torch.empty(B, H, N, D, dtype=kv_dtype, device=device),
        sorted_value=torch.empty(B, H, N, D, dtype=kv_dtype, device=device),
        max_groups=G,
        sample_end=N,
    )


def build_summary(key_cache: torch.Tensor, value_cache: torch.Tensor, labels: torch.Tensor,
                  n_clusters: int, *, sample_end: int, n_total: int | None = None,
                  out: ClusterSummary | None = None, stream=None) -> ClusterSummary:
    """Cluster summary of the prefix ``[0, sample_end)`` from per-token labels.

    key_cache / value_cache: ``[B, Hkv, capacity, D]`` (bf16 or fp32), or a
    PagedKVCache as ``key_cache`` with ``value_cache`` None.
    labels: ``[B, Hkv, sample_end]`` integer cluster ids in ``[0, n_clusters)``.
    """
    kt, vt = _kv(key_cache, value_cache)
    B, Hkv, cap, D = key_cache.shape
    n_total = cap if n_total is None else n_total
    geo = _geometry(key_cache, Hkv, n_total, sample_end)
    if labels.shape != (B, Hkv, sample_end):
        raise ValueError(f"labels must be [{B}, {Hkv}, {sample_end}], got {tuple(labels.shape)}")
    labels = labels.to(device=kt.device, dtype=torch.int32).contiguous()
    if out is None:
        out = allocate_summary(B, Hkv, sample_end, D, n_clusters, kt.dtype, kt.device)
    lib = _lib.load()
    nbytes = ctypes.c_size_t()
    _lib.check("santa_build_summary_workspace_bytes",
               lib.santa_build_summary_workspace_bytes(ctypes.byref(geo), n_clusters,
                                                       ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=kt.device)
    c = out.as_c()
    _lib.check("santa_build_summary", lib.santa_build_summary(
        ctypes.byref(geo), kt.data_ptr(), vt.data_ptr(), labels.data_ptr(),
        n_clusters, ctypes.byref(c), ws.data_ptr(), nbytes.value, _lib.stream_handle(stream)))
    out._workspace = ws  # keeps the error flag readable; see summary_flag()
    return out


# ---------------------------------------------------------------------------
# sparse decode
# ---------------------------------------------------------------------------

@dataclass
class DecodeResult:
    out: torch.Tensor               # [B, Hq, D] fp32
    lse: torch.Tensor               # [B, Hq] fp32
    n_exact: torch.Tensor | None    # [B, Hq] int32
    ess: torch.Tensor | None        # [B, Hq] fp32


class DecodeWorkspace:
    """Reusable scratch buffer for ``santa_decode`` (grown on demand)."""

    def __init__(self):
        self.buffer: torch.Tensor | None = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buffer is None or self.buffer.numel() < nbytes or self.buffer.device != device:
            self.buffer = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        return self.buffer


_default_ws: dict = {}


def _check_injected_draws(lib, geo, ws: torch.Tensor, nbytes: int, stream=None) -> None:
    """Raise if an injected draw was out of range (the kernel clamps it)."""
    n = ctypes.c_int32()
    _lib.check("santa_decode_bad_draws", lib.santa_decode_bad_draws(
        ctypes.byref(geo), ws.data_ptr(), nbytes, ctypes.byref(n), _lib.stream_handle(stream)))
    if n.value:
        raise ValueError(f"injected sample draws out of range in {n.value} (batch, KV head) "
                         "segments")


def decode_params(mode: str, *, topk_clusters: int = 0, token_budget: int = 0, samples: int = 0,
                  scale: float, injected: bool = False, seed: int = 0, step: int = 0,
                  num_splits: int = 0) -> _lib.SantaDecodeParams:
    if mode not in _lib.MODES:
        raise ValueError(f"Unknown SANTA++ mode: {mode!r}")
    return _lib.SantaDecodeParams(
        _lib.MODES[mode], int(topk_clusters), int(token_budget), int(samples), float(scale),
        _lib.SAMPLES_INJECTED if injected else _lib.SAMPLES_DEVICE,
        int(seed) & 0xFFFFFFFFFFFFFFFF, int(step) & 0xFFFFFFFFFFFFFFFF, int(num_splits))


def santa_decode(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 summary: ClusterSummary, *, mode: str = "hybrid", n_total: int,
                 sample_end: int | None = None, topk_clusters: int = 0, token_budget: int = 0,
                 samples: int = 0, scale: float | None = None,
                 sample_a: torch.Tensor | None = None, sample_b: torch.Tensor | None = None,
                 seed: int = 0, step: int = 0, num_splits: int = 0,
                 out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                 with_stats: bool = False, workspace: DecodeWorkspace | None = None,
                 stream=None) -> DecodeResult:
    """One SANTA++ decode step for all (batch, query head) pairs.

    q: ``[B, Hq, D]`` fp32 (RoPE applied).  ``mode`` is one of the reference's
    ``topk`` (budget walk with ``token_budget`` tokens), ``guided``,
    ``uniform``, ``santa`` (``samples`` draws) or ``hybrid`` (exact
    ``topk_clusters`` clusters plus ``samples`` uniform draws of the rest).
    ``sample_a`` / ``sample_b`` inject the random draws instead of the
    on-device Philox sampler (see include/santa_b200.h).  ``key_cache`` may
    be a PagedKVCache (``value_cache`` None)."""
    _require_cuda("q", q)
    kt, vt = _kv(key_cache, value_cache)
    if q.dtype != torch.float32 or q.dim() != 3:
        raise ValueError("q must be [batch, query_heads, head_dim] fp32")
    B, Hq, D = q.shape
    sample_end = summary.sample_end if sample_end is None else sample_end
    geo = _geometry(key_cache, Hq, n_total, sample_end)
    if key_cache.shape[0] != B or key_cache.shape[3] != D:
        raise ValueError("q and cache disagree on batch or head_dim")
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    injected = sample_a is not None
    if injected:
        for name, t in (("sample_a", sample_a), ("sample_b", sample_b)):
            if t is not None:
                _require_cuda(name, t)
                if t.dtype != torch.int32 or t.shape != (B, Hq, samples):
                    raise ValueError(f"{name} must be int32 [{B}, {Hq}, {samples}]")
    p = decode_params(mode, topk_clusters=topk_clusters, token_budget=token_budget,
                      samples=samples, scale=scale, injected=injected, seed=seed, step=step,
                      num_splits=num_splits)
    lib = _lib.load()
    nbytes = ctypes.c_size_t()
    _lib.check("santa_decode_workspace_bytes", lib.santa_decode_workspace_bytes(
        ctypes.byref(geo), ctypes.byref(p), summary.max_groups, ctypes.byref(nbytes)))
    if workspace is None:
        workspace = _default_ws.setdefault(q.device, DecodeWorkspace())
    ws = workspace.get(nbytes.value, q.device)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    if lse is None:
        lse = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
    n_exact = torch.empty(B, Hq, dtype=torch.int32, device=q.device) if with_stats else None
    ess = torch.empty(B, Hq, dtype=torch.float32, device=q.device) if with_stats else None
    c = summary.as_c()
    _lib.check("santa_decode", lib.santa_decode(
        ctypes.byref(geo), ctypes.byref(p), q.data_ptr(), kt.data_ptr(),
        vt.data_ptr(), ctypes.byref(c), _lib.ptr(sample_a), _lib.ptr(sample_b),
        out.data_ptr(), lse.data_ptr(), _lib.ptr(n_exact), _lib.ptr(ess), ws.data_ptr(),
        nbytes.value, _lib.stream_handle(stream)))
    if injected:
        _check_injected_draws(lib, geo, ws, nbytes.value, stream)
    return DecodeResult(out, lse, n_exact, ess)


class DecodeStep:
    """A decode call pre-bound to one cache, summary and parameter set.

    The geometry, parameter and summary structs and the workspace are built
    once, so a decode step costs two C ABI calls (``plan`` then ``execute``)
    and no allocation.  Used by the model-level decode loop and the bench."""

    def __init__(self, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 summary: ClusterSummary, *, num_query_heads: int, mode: str = "hybrid",
                 n_total: int, topk_clusters: int = 0, token_budget: int = 0, samples: int = 0,
                 scale: float | None = None, seed: int = 0, num_splits: int = 0,
                 injected: bool = False, with_stats: bool = False):
        self.kv_args = (key_cache, value_cache)   # as given (a PagedKVCache stays alive)
        self.key_cache, self.value_cache = _kv(key_cache, value_cache)
        self.summary = summary
        B, Hkv, _, D = key_cache.shape
        self.geo = _geometry(key_cache, num_query_heads, n_total, summary.sample_end)
        self.scale = 1.0 / math.sqrt(D) if scale is None else scale
        self.mode = mode
        self.p = decode_params(mode, topk_clusters=topk_clusters, token_budget=token_budget,
                               samples=samples, scale=self.scale, injected=injected, seed=seed,
                               num_splits=num_splits)
        self.c = summary.as_c()
        self.lib = _lib.load()
        nbytes = ctypes.c_size_t()
        _lib.check("santa_decode_workspace_bytes", self.lib.santa_decode_workspace_bytes(
            ctypes.byref(self.geo), ctypes.byref(self.p), summary.max_groups,
            ctypes.byref(nbytes)))
        self.ws_bytes = nbytes.value
        dev = self.key_cache.device
        self.ws = torch.empty(max(1, self.ws_bytes), dtype=torch.uint8, device=dev)
        self.out = torch.empty(B, num_query_heads, D, dtype=torch.float32, device=dev)
        self.lse = torch.empty(B, num_query_heads, dtype=torch.float32, device=dev)
        self.n_exact = (torch.empty(B, num_query_heads, dtype=torch.int32, device=dev)
                        if with_stats else None)
        self.ess = (torch.empty(B, num_query_heads, dtype=torch.float32, device=dev)
                    if with_stats else None)
        self._q = None
        self._refs = (ctypes.byref(self.geo), ctypes.byref(self.p), ctypes.byref(self.c))

    def plan(self, q: torch.Tensor, step: int = 0, sample_a=None, sample_b=None, stream=None):
        self.p.step = int(step) & 0xFFFFFFFFFFFFFFFF
        self._q = q
        g, p, c = self._refs
        _lib.check("santa_decode_plan", self.lib.santa_decode_plan(
            g, p, q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(), c,
            _lib.ptr(sample_a), _lib.ptr(sample_b), _lib.ptr(self.n_exact), self.ws.data_ptr(),
            self.ws_bytes, _lib.stream_handle(stream)))
        if sample_a is not None:
            _check_injected_draws(self.lib, self.geo, self.ws, self.ws_bytes, stream)

    def execute(self, stream=None) -> torch.Tensor:
        g, p, c = self._refs
        _lib.check("santa_decode_execute", self.lib.santa_decode_execute(
            g, p, self._q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(),
            c, self.out.data_ptr(), self.lse.data_ptr(), _lib.ptr(self.ess), self.ws.data_ptr(),
            self.ws_bytes, _lib.stream_handle(stream)))
        return self.out

    def __call__(self, q: torch.Tensor, step: int = 0, stream=None) -> torch.Tensor:
        self.plan(q, step, stream=stream)
        return self.execute(stream)

    @property
    def kernels_per_call(self) -> int:
        """Kernels of this library launched per step: select and attend, plus
        the old-prefix LSE pass in santa mode."""
        return 2 + (1 if self.mode == "santa" else 0)

    def graphed(self, q_host: torch.Tensor, out_host: torch.Tensor) -> "GraphedDecodeStep":
        """This step captured once in a CUDA graph together with its host
        transfers (see ``GraphedDecodeStep``)."""
        return GraphedDecodeStep(self, q_host, out_host)


class GraphedDecodeStep:
    """A ``DecodeStep`` and its host transfers as one CUDA graph.

    Per ``run(step)`` the graph copies the queries in from the pinned host
    buffer ``q_host`` ([B, Hq, D] fp32) together with the Philox step
    counter (a device word the selection kernel reads in place of the
    parameter, so each replay draws the samples of its own step), runs the
    selection and the attention, and copies the output into the pinned
    ``out_host``.  One graph launch per decode step instead of four API
    calls; the output is in ``out_host`` once the stream is synchronised.
    Write a step's queries into ``q_host`` only after the previous step's
    output was read (the graph reads the buffer when it runs)."""

    def __init__(self, step: DecodeStep, q_host: torch.Tensor, out_host: torch.Tensor):
        for name, t in (("q_host", q_host), ("out_host", out_host)):
            if t.device.type != "cpu" or not t.is_pinned() or t.dtype != torch.float32:
                raise ValueError(f"{name} must be a pinned fp32 host tensor")
            if tuple(t.shape) != tuple(step.out.shape):
                raise ValueError(f"{name} must be {tuple(step.out.shape)}")
        if step.p.sample_source != _lib.SAMPLES_DEVICE:
            raise ValueError("a graphed step draws its samples on the device")
        self.step, self.q_host, self.out_host = step, q_host, out_host
        dev = step.out.device
        self.q_dev = torch.empty(q_host.shape, dtype=torch.float32, device=dev)
        self.step_host = torch.zeros(1, dtype=torch.int64).pin_memory()
        self.step_dev = torch.zeros(1, dtype=torch.int64, device=dev)
        # the step's parameters with the counter read from the device word
        self.p = _lib.SantaDecodeParams.from_buffer_copy(step.p)
        self.p.step_dev = self.step_dev.data_ptr()
        self._refs = (ctypes.byref(step.geo), ctypes.byref(self.p), ctypes.byref(step.c))
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            for _ in range(2):   # first launches (function attributes) outside the capture
                self._body()
        stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self._body()
        torch.cuda.synchronize(dev)

    def _body(self) -> None:
        st = self.step
        g, p, c = self._refs
        self.q_dev.copy_(self.q_host, non_blocking=True)
        self.step_dev.copy_(self.step_host, non_blocking=True)
        _lib.check("santa_decode_plan", st.lib.santa_decode_plan(
            g, p, self.q_dev.data_ptr(), st.key_cache.data_ptr(), st.value_cache.data_ptr(), c,
            None, None, _lib.ptr(st.n_exact), st.ws.data_ptr(), st.ws_bytes,
            _lib.stream_handle()))
        _lib.check("santa_decode_execute", st.lib.santa_decode_execute(
            g, p, self.q_dev.data_ptr(), st.key_cache.data_ptr(), st.value_cache.data_ptr(), c,
            st.out.data_ptr(), st.lse.data_ptr(), _lib.ptr(st.ess), st.ws.data_ptr(),
            st.ws_bytes, _lib.stream_handle()))
        self.out_host.copy_(st.out, non_blocking=True)

    def run(self, step: int) -> None:
        """Enqueue decode step ``step`` on the current stream (not synchronised)."""
        self.step_host[0] = int(step) & 0x7FFFFFFFFFFFFFFF
        self.graph.replay()

    @property
    def kernels_per_call(self) -> int:
        return self.step.kernels_per_call


def santa_decode_select(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                        summary: ClusterSummary, *, mode: str = "hybrid", n_total: int,
                        sample_end: int | None = None, topk_clusters: int = 0,
                        token_budget: int = 0, samples: int = 0, scale: float | None = None,
                        sample_a: torch.Tensor | None = None,
                        sample_b: torch.Tensor | None = None, seed: int = 0, step: int = 0,
                        workspace: DecodeWorkspace | None = None, stream=None):
    """Selection part of ``santa_decode`` read out per query head.

    Returns ``(selected [B, Hq, G] uint8, sample_rows [B, Hq, S] int32,
    n_exact [B, Hq] int32)``; ``sample_rows`` index the cluster-sorted copy."""
    _require_cuda("q", q)
    kt, vt = _kv(key_cache, value_cache)
    B, Hq, D = q.shape
    sample_end = summary.sample_end if sample_end is None else sample_end
    geo = _geometry(key_cache, Hq, n_total, sample_end)
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    p = decode_params(mode, topk_clusters=topk_clusters, token_budget=token_budget,
                      samples=samples, scale=scale, injected=sample_a is not None, seed=seed,
                      step=step)
    lib = _lib.load()
    nbytes = ctypes.c_size_t()
    _lib.check("santa_decode_workspace_bytes", lib.santa_decode_workspace_bytes(
        ctypes.byref(geo), ctypes.byref(p), summary.max_groups, ctypes.byref(nbytes)))
    if workspace is None:
        workspace = _default_ws.setdefault(q.device, DecodeWorkspace())
    ws = workspace.get(nbytes.value, q.device)
    selected = torch.empty(B, Hq, summary.max_groups, dtype=torch.uint8, device=q.device)
    rows = torch.empty(B, Hq, max(samples, 1), dtype=torch.int32, device=q.device)
    n_exact = torch.empty(B, Hq, dtype=torch.int32, device=q.device)
    c = summary.as_c()
    _lib.check("santa_decode_select", lib.santa_decode_select(
        ctypes.byref(geo), ctypes.byref(p), q.data_ptr(), kt.data_ptr(),
        vt.data_ptr(), ctypes.byref(c), _lib.ptr(sample_a), _lib.ptr(sample_b),
        selected.data_ptr(), rows.data_ptr(), n_exact.data_ptr(), ws.data_ptr(), nbytes.value,
        _lib.stream_handle(stream)))
    if sample_a is not None:
        _check_injected_draws(lib, geo, ws, nbytes.value, stream)
    return selected, rows[..., :samples], n_exact


# ---------------------------------------------------------------------------
# traffic accounting (santapp.py:80-142)
# ---------------------------------------------------------------------------

@dataclass
class DecodeTrafficTracker:
    """Decode-time attention row reads over all layers and heads."""

    head_calls: int = 0
    dense_kv_vectors: int = 0
    kv_vectors_read: int = 0
    metadata_key_vectors_read: int = 0
    sampled_token_draws: int = 0
    recent_token_reads: int = 0
    total_tokens_summed: int = 0
    ess_ratios: list = field(default_factory=list)

    def record_step(self, *, mode: str, n_total: int, sample_end: int, n_exact: np.ndarray,
                    samples: int, n_groups: np.ndarray, ess: np.ndarray | None = None) -> None:
        """Account one batched decode step (one call per query head in the
        reference: santapp.py:419-426 for topk, 498-505 otherwise)."""
        recent = n_total - sample_end
        n_exact = np.asarray(n_exact).reshape(-1)
        n_groups = np.asarray(n_groups).reshape(-1)
        calls = n_exact.size
        g = calls // max(1, n_groups.size)
        meta = np.repeat(n_groups, g) if n_groups.size else np.zeros(calls, np.int64)
        self.head_calls += calls
        self.dense_kv_vectors += 2 * n_total * calls
        self.recent_token_reads += recent * calls
        self.total_tokens_summed += n_total * calls
        if mode == "topk":
            self.kv_vectors_read += int(2 * (n_exact.sum() + recent * calls))
            self.sampled_token_draws += int(n_exact.sum())
            self.metadata_key_vectors_read += int(meta.sum())
        elif mode == "santa":
            self.kv_vectors_read += (sample_end + samples + 2 * recent) * calls
            self.sampled_token_draws += samples * calls
        else:
            exact = n_exact.sum() if mode == "hybrid" else 0
            self.kv_vectors_read += int(2 * (samples * calls + exact + recent * calls))
            self.sampled_token_draws += samples * calls
            if mode in ("guided", "hybrid"):
                self.metadata_key_vectors_read += int(meta.sum())
        if ess is not None and mode != "topk":
            self.ess_ratios.extend(float(x) for x in np.asarray(ess).reshape(-1))

    def as_dict(self) -> dict:
        dense = self.dense_kv_vectors
        calls = self.head_calls
        equivalent = self.kv_vectors_read + self.metadata_key_vectors_read
        return {
            "decode_attention_head_calls": calls,
            "decode_dense_kv_vectors": dense,
            "decode_kv_vectors_read": self.kv_vectors_read,
            "decode_metadata_key_vectors_read": self.metadata_key_vectors_read,
            "decode_kv_access_pct": 100.0 * self.kv_vectors_read / dense if dense else 0.0,
            "decode_read_equivalent_pct": 100.0 * equivalent / dense if dense else 0.0,
            "decode_metadata_equivalent_pct": (100.0 * self.metadata_key_vectors_read / dense
                                               if dense else 0.0),
            "mean_sampled_token_draws_per_head_call": (self.sampled_token_draws / calls
                                                       if calls else 0.0),
            "mean_recent_tokens_per_head_call": self.recent_token_reads / calls if calls else 0.0,
            "mean_total_tokens_per_head_call": self.total_tokens_summed / calls if calls else 0.0,
            "mean_ess_over_samples": float(np.mean(self.ess_ratios)) if self.ess_ratios else None,
        }
