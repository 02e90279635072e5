"""Paged KV cache: the per-layer cache of the reference split into pages.

The reference keeps one preallocated ``[n_kv, capacity, d]`` tensor per layer
and sequence (``LayerCache``, santapp_ruler/attention/santapp.py:66-77) and
appends every step's keys and values at the current length
(``_append_cache``, :234-274).  Here a layer's K and V live in page pools
``[num_pages, Hkv, page_size, D]`` shared by all sequences of the batch;
sequence ``b``'s token ``p`` is in page ``block_table[b, p // page_size]``,
slot ``p % page_size``.  Pages are handed out on demand, so a batch of
sequences of different lengths holds only the pages it uses, and a sequence
grows by taking a free page.

Every kernel that reads the cache (summary build, selection, the recent
window of the attention kernel, the santa-mode old-prefix pass) resolves rows
through the same table (``cache_row`` in the CUDA sources), so a paged cache
and a contiguous cache with the same contents give bit-identical results.
The sequence-sharded entry points take contiguous caches only.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib


class PagedKVCache:
    """K/V page pools of one attention layer plus the batch's block table.

    ``key_pool`` / ``value_pool``: ``[num_pages, num_kv_heads, page_size,
    head_dim]`` (bf16 or fp32) on the GPU; ``block_table``: ``[batch,
    max_pages]`` int32 page ids, ``-1`` for pages not yet mapped.
    ``page_size`` must be a power of two."""

    def __init__(self, key_pool: torch.Tensor, value_pool: torch.Tensor,
                 block_table: torch.Tensor):
        for name, t in (("key_pool", key_pool), ("value_pool", value_pool),
                        ("block_table", block_table)):
            if not isinstance(t, torch.Tensor):
                raise TypeError(f"{name} must be a torch.Tensor")
            if t.device.type != "cuda":
                raise ValueError(f"{name} must be a CUDA tensor (the SANTA++ kernels have no "
                                 "CPU path)")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        if key_pool.dim() != 4 or value_pool.shape != key_pool.shape:
            raise ValueError("pools must be [num_pages, kv_heads, page_size, head_dim], K and V "
                             "alike")
        if value_pool.dtype != key_pool.dtype:
            raise ValueError("key and value pools must have the same dtype")
        if block_table.dim() != 2 or block_table.dtype != torch.int32:
            raise ValueError("block_table must be int32 [batch, max_pages]")
        page_size = key_pool.shape[2]
        if page_size <= 0 or page_size & (page_size - 1):
            raise ValueError(f"page_size {page_size} must be a power of two")
        self.key_pool, self.value_pool, self.block_table = key_pool, value_pool, block_table
        self._free: list[int] | None = None       # free page ids (allocate() only)
        self._host_table: torch.Tensor | None = None
        self._mapped = 0                            # pages mapped in every sequence

    # ---- shape ------------------------------------------------------------
    @property
    def num_pages(self) -> int:
        return self.key_pool.shape[0]

    @property
    def num_kv_heads(self) -> int:
        return self.key_pool.shape[1]

    @property
    def page_size(self) -> int:
        return self.key_pool.shape[2]

    @property
    def head_dim(self) -> int:
        return self.key_pool.shape[3]

    @property
    def batch(self) -> int:
        return self.block_table.shape[0]

    @property
    def max_pages(self) -> int:
        return self.block_table.shape[1]

    @property
    def capacity(self) -> int:
        """Tokens a sequence can hold (its block-table row times page_size)."""
        return self.max_pages * self.page_size

    @property
    def dtype(self) -> torch.dtype:
        return self.key_pool.dtype

    @property
    def device(self) -> torch.device:
        return self.key_pool.device

    @property
    def shape(self) -> tuple:
        """The contiguous cache shape this cache stands for."""
        return (self.batch, self.num_kv_heads, self.capacity, self.head_dim)

    # ---- construction ------------------------------------------------------
    @classmethod
    def allocate(cls, batch: int, num_kv_heads: int, head_dim: int, *, max_tokens: int,
                 page_size: int = 256, num_pages: int | None = None,
                 dtype: torch.dtype = torch.bfloat16, device="cuda",
                 page_order_seed: int | None = None) -> "PagedKVCache":
        """Empty pools and an unmapped table (every entry -1).  ``num_pages``
        defaults to enough pages for every sequence at ``max_tokens``.  The
        free list hands pages out in ascending order, or in a seeded random
        order with ``page_order_seed`` (a sequence's pages then lie scattered
        over the pool)."""
        if page_size <= 0 or page_size & (page_size - 1):
            raise ValueError(f"page_size {page_size} must be a power of two")
        max_pages = -(-max_tokens // page_size)
        if num_pages is None:
            num_pages = batch * max_pages
        shape = (num_pages, num_kv_heads, page_size, head_dim)
        kp = torch.zeros(shape, dtype=dtype, device=device)
        vp = torch.zeros(shape, dtype=dtype, device=device)
        table = torch.full((batch, max_pages), -1, dtype=torch.int32, device=device)
        cache = cls(kp, vp, table)
        order = torch.arange(num_pages)
        if page_order_seed is not None:
            order = order[torch.randperm(num_pages,
                                         generator=torch.Generator().manual_seed(page_order_seed))]
        cache._free = order.tolist()[::-1]   # pop() from the end hands out order[0] first
        cache._host_table = torch.full((batch, max_pages), -1, dtype=torch.int32)
        return cache

    def reserve(self, length: int) -> None:
        """Map pages so that every sequence holds tokens ``[0, length)``
        (pages already mapped stay); raises when the pool runs out."""
        if self._free is None:
            raise RuntimeError("reserve() needs a cache made by allocate()")
        need = -(-length // self.page_size)
        if need <= self._mapped:      # every sequence holds these pages already
            return
        if need > self.max_pages:
            raise ValueError(f"length {length} exceeds the capacity {self.capacity}")
        changed = False
        for b in range(self.batch):
            for i in range(need):
                if int(self._host_table[b, i]) < 0:
                    if not self._free:
                        raise RuntimeError("page pool exhausted")
                    self._host_table[b, i] = self._free.pop()
                    changed = True
        self._mapped = need
        if changed:
            self.block_table.copy_(self._host_table, non_blocking=False)

    def release(self, b: int) -> None:
        """Return sequence ``b``'s pages to the free list (its tokens are gone)."""
        if self._free is None:
            raise RuntimeError("release() needs a cache made by allocate()")
        for i in range(self.max_pages):
            page = int(self._host_table[b, i])
            if page >= 0:
                self._free.append(page)
                self._host_table[b, i] = -1
        self._mapped = 0
        self.block_table.copy_(self._host_table, non_blocking=False)

    @classmethod
    def from_contiguous(cls, key_cache: torch.Tensor, value_cache: torch.Tensor, *,
                        length: int, page_size: int = 256, num_pages: int | None = None,
                        page_order_seed: int | None = None) -> "PagedKVCache":
        """Pages holding tokens ``[0, length)`` of contiguous ``[B, Hkv, cap,
        D]`` caches (one gather copy per page on the device)."""
        B, Hkv, cap, D = key_cache.shape
        cache = cls.allocate(B, Hkv, D, max_tokens=cap, page_size=page_size,
                             num_pages=num_pages, dtype=key_cache.dtype,
                             device=key_cache.device, page_order_seed=page_order_seed)
        cache.reserve(length)
        n = -(-length // page_size)
        pages = cache.block_table[:, :n].long()                       # [B, n]
        for src, pool in ((key_cache, cache.key_pool), (value_cache, cache.value_pool)):
            padded = torch.zeros(B, Hkv, n * page_size, D, dtype=src.dtype, device=src.device)
            padded[:, :, :length] = src[:, :, :length]
            blocks = padded.view(B, Hkv, n, page_size, D).permute(0, 2, 1, 3, 4)
            pool[pages.reshape(-1)] = blocks.reshape(B * n, Hkv, page_size, D)
        return cache

    def to_contiguous(self, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Tokens ``[0, length)`` gathered back into ``[B, Hkv, length, D]``
        K and V tensors (unmapped pages read as page 0, as the kernels do)."""
        n = -(-length // self.page_size)
        pages = self.block_table[:, :n].long()
        pages = torch.where((pages >= 0) & (pages < self.num_pages), pages,
                            torch.zeros_like(pages))
        out = []
        for pool in (self.key_pool, self.value_pool):
            blocks = pool[pages.reshape(-1)].view(self.batch, n, self.num_kv_heads,
                                                  self.page_size, self.head_dim)
            full = blocks.permute(0, 2, 1, 3, 4).reshape(self.batch, self.num_kv_heads,
                                                         n * self.page_size, self.head_dim)
            out.append(full[:, :, :length].contiguous())
        return out[0], out[1]

    def slots(self, b: int, positions) -> tuple[torch.Tensor, torch.Tensor]:
        """(page ids, slots) of sequence ``b``'s token positions, from the
        host copy of the table: ``key_pool[pages, kv, slots]`` are the rows."""
        if self._host_table is None:
            raise RuntimeError("slots() needs a cache made by allocate()")
        pos = torch.as_tensor(positions, dtype=torch.long)
        pages = self._host_table[b].long()[pos // self.page_size]
        if (pages < 0).any():
            raise ValueError("position in an unmapped page")
        return pages.to(self.device), (pos % self.page_size).to(self.device)

    def tokens(self, b: int, kv: int, n: int, value: bool = False) -> torch.Tensor:
        """Tokens ``[0, n)`` of sequence ``b``, KV head ``kv`` as a contiguous
        ``[n, D]`` tensor (a gather over the sequence's pages, on the device)."""
        pages = self.block_table[b, : -(-n // self.page_size)].long()
        pool = self.value_pool if value else self.key_pool
        return pool[pages, kv].reshape(-1, self.head_dim)[:n]

    # ---- the C view ----------------------------------------------------------
    def fill_geometry(self, geo: "_lib.SantaGeometry") -> None:
        """Set the paged fields of a SantaGeometry (the table pointer stays
        valid while this object holds the table)."""
        geo.block_table = ctypes.c_void_p(self.block_table.data_ptr())
        geo.page_size = self.page_size
        geo.max_pages = self.max_pages
        geo.num_pages = self.num_pages

    def append(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor,
               sin: torch.Tensor, start: int, *, q_rot_bf16: torch.Tensor | None = None,
               q_rot_f32: torch.Tensor | None = None, stream=None) -> None:
        """RoPE + append of ``tokens`` new positions at ``start`` into the
        pages (``santa_rope_append_paged``); maps the pages it needs first.
        q ``[B, T, Hq, D]``, k / v ``[B, T, Hkv, D]``, cos / sin ``[B, T, D]``,
        all bf16; rotated queries out as ``[B, Hq, T, D]`` (bf16 and/or fp32)."""
        if self.dtype != torch.bfloat16:
            raise ValueError("the fused RoPE append writes bf16 pools")
        B, T, Hq, D = q.shape
        # pages are mapped only when the new tokens cross into an unmapped one
        if self._free is not None and start + T > self._mapped * self.page_size:
            self.reserve(start + T)
        lib = _lib.load()
        _lib.check("santa_rope_append_paged", lib.santa_rope_append_paged(
            B, T, Hq, self.num_kv_heads, D, q.data_ptr(), k.data_ptr(), v.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), self.key_pool.data_ptr(), self.value_pool.data_ptr(),
            self.block_table.data_ptr(), self.page_size, self.max_pages, self.num_pages, start,
            _lib.ptr(q_rot_bf16), _lib.ptr(q_rot_f32), _lib.stream_handle(stream)))
