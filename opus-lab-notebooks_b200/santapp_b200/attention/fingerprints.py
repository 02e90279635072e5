"""Key fingerprints for clustering, on the sm_100a kernels.

Host-side mirror of the clustering input of
``SantaPlusEngine._dense_prefill_and_cluster`` (santapp_ruler/attention/
santapp.py:598-691): probe positions chosen by ``probe_strategy`` with the
reference's numpy draws, then per (layer, KV head) the fingerprints
``concat_h(K_prefix @ q_h[probes].T / sqrt(d))`` z-scored per column
(population std + 1e-6).  The arithmetic runs in ``santa_fingerprints``
(csrc/fingerprint.cu) with order-independent exact column sums, so the
features, and the k-means labels computed from them, are reproducible bit
for bit.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from .. import _lib
from .santapp import _require_cuda

__all__ = ["probe_positions", "cluster_count", "build_fingerprints"]


def probe_positions(strategy: str, prompt_tokens: int, n_probes: int, *,
                    region_start_fraction: float = 0.75, probe_seed: int = 0) -> np.ndarray:
    """Probe query positions (santapp.py:598-642)."""
    max_idx = prompt_tokens - 1
    if strategy == "end_quarter":
        probe_start = int(region_start_fraction * prompt_tokens)
        candidates = np.arange(probe_start, max_idx)
        if candidates.size < n_probes:
            raise ValueError(f"Only {candidates.size} probe positions available, "
                             f"need {n_probes}.")
        rng = np.random.RandomState(probe_seed)
        return np.sort(rng.choice(candidates, size=n_probes, replace=False))
    if strategy in ("start", "middle", "end", "random") and max_idx < n_probes:
        raise ValueError(f"Prompt too short ({max_idx} tokens) for {n_probes} probes.")
    if strategy == "start":
        return np.arange(0, n_probes)
    if strategy == "middle":
        mid = max_idx // 2
        start = max(0, mid - n_probes // 2)
        return np.arange(start, start + n_probes)
    if strategy == "end":
        return np.arange(max_idx - n_probes, max_idx)
    if strategy == "random":
        rng = np.random.RandomState(probe_seed)
        return np.sort(rng.choice(max_idx, size=n_probes, replace=False))
    raise ValueError(f"Unknown probe strategy: {strategy!r}")


def cluster_count(sample_end: int, group_size: int) -> int:
    """n_clusters of one (layer, KV head) (santapp.py:646-649)."""
    return min(sample_end, max(2, sample_end // group_size))


def build_fingerprints(key_prefix: torch.Tensor, query_rotated: torch.Tensor, kv_head: int,
                       group: int, probes, *, normalize: bool = True,
                       out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """key_prefix ``[N, D]`` (bf16 or fp32) and the layer's rotated queries
    ``[Hq, T, D]`` fp32 -> fingerprints ``[N, group * P]`` fp32."""
    _require_cuda("key_prefix", key_prefix)
    _require_cuda("query_rotated", query_rotated)
    if key_prefix.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("key_prefix must be bf16 or fp32")
    if query_rotated.dtype != torch.float32 or query_rotated.dim() != 3:
        raise ValueError("query_rotated must be [query_heads, T, D] fp32")
    N, D = key_prefix.shape
    Hq, T, Dq = query_rotated.shape
    if Dq != D or (kv_head + 1) * group > Hq:
        raise ValueError("query heads / head_dim do not match the keys")
    pr = torch.as_tensor(np.asarray(probes, np.int64), device=key_prefix.device)
    if pr.numel() == 0 or int(pr.min()) < 0 or int(pr.max()) >= T:
        raise ValueError("probe positions must lie in [0, T)")
    cols = group * pr.numel()
    if out is None:
        out = torch.empty(N, cols, dtype=torch.float32, device=key_prefix.device)
    lib = _lib.load()
    nbytes = ctypes.c_size_t()
    _lib.check("santa_fingerprints_workspace_bytes",
               lib.santa_fingerprints_workspace_bytes(cols, ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=key_prefix.device)
    dtype = _lib.DTYPE_BF16 if key_prefix.dtype == torch.bfloat16 else _lib.DTYPE_F32
    qg = query_rotated[kv_head * group:(kv_head + 1) * group]
    _lib.check("santa_fingerprints", lib.santa_fingerprints(
        key_prefix.data_ptr(), dtype, N, D, qg.data_ptr(), T * D, group, pr.data_ptr(),
        pr.numel(), float(np.float32(math.sqrt(D))), 1 if normalize else 0, out.data_ptr(),
        ws.data_ptr(), nbytes.value, _lib.stream_handle(stream)))
    return out
