"""Dense causal prefill attention on the sm_100a tcgen05 kernel.

Replaces the prefill branch of ``SantaPlusEngine._attention_forward``
(santapp_ruler/attention/santapp.py:320-346): the reference calls
``transformers.integrations.sdpa_attention.sdpa_attention_forward``, i.e.
``torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)``
over ``[B, H, T, D]`` bf16 tensors with GQA (query head ``h`` reads KV head
``h // (Hq // Hkv)``).  Here one call of ``santa_prefill`` (C ABI) does the
same with tcgen05 MMAs accumulating in TMEM.
"""

from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib
from .paged import PagedKVCache
from .santapp import _require_cuda

__all__ = ["santa_prefill"]


def santa_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
                  scale: float | None = None, out: torch.Tensor | None = None,
                  return_lse: bool = False, stream=None):
    """q ``[B, Hq, T, D]``, k / v ``[B, Hkv, C, D]`` (C >= T: a cache whose first
    T tokens are the prompt) bf16 CUDA tensors, or ``k`` a PagedKVCache
    holding the prompt (``v`` None) ->
    out ``[B, Hq, T, D]`` bf16 (and the natural-log softmax denominators
    ``[B, Hq, T]`` fp32 with ``return_lse``)."""
    paged = k if isinstance(k, PagedKVCache) else None
    if paged is not None:
        if v is not None:
            raise ValueError("with a PagedKVCache, pass v=None")
        k, v = paged.key_pool, paged.value_pool
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t)
        if t.dtype != torch.bfloat16 or t.dim() != 4:
            raise ValueError(f"{name} must be a [batch, heads, seq, head_dim] bf16 tensor")
    B, Hq, T, D = q.shape
    if paged is not None:
        Hkv, cap = paged.num_kv_heads, paged.capacity
        if paged.batch != B or paged.head_dim != D or cap < T:
            raise ValueError("the paged cache must hold batch x >= seq tokens of head_dim")
    else:
        Hkv, cap = k.shape[1], k.shape[2]
    if paged is None and (k.shape != (B, Hkv, cap, D) or v.shape != k.shape or cap < T):
        raise ValueError("k and v must be [batch, kv_heads, >= seq, head_dim] matching q "
                         "(a KV cache whose first seq tokens are used)")
    if Hq % Hkv:
        raise ValueError("Query heads must be divisible by KV heads.")
    shape = _lib.SantaPrefillShape(B, Hq, Hkv, T, D, 1.0 / math.sqrt(D) if scale is None
                                   else float(scale), 1 if causal else 0,
                                   0 if paged is not None else cap)
    lib = _lib.load()
    nbytes = ctypes.c_size_t()
    _lib.check("santa_prefill_workspace_bytes",
               lib.santa_prefill_workspace_bytes(ctypes.byref(shape), ctypes.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty(B, Hq, T, dtype=torch.float32, device=q.device) if return_lse else None
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    if paged is not None:
        _lib.check("santa_prefill_paged", lib.santa_prefill_paged(
            ctypes.byref(shape), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            paged.block_table.data_ptr(), paged.page_size, paged.max_pages, paged.num_pages,
            out.data_ptr(), _lib.ptr(lse), err.data_ptr(), ws.data_ptr(), nbytes.value,
            _lib.stream_handle(stream)))
    else:
        _lib.check("santa_prefill", lib.santa_prefill(
            ctypes.byref(shape), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            _lib.ptr(lse), err.data_ptr(), ws.data_ptr(), nbytes.value,
            _lib.stream_handle(stream)))
    out._santa_error_flag = err  # read by callers that check the kernel's bounded waits
    return (out, lse) if return_lse else out
