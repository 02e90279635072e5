"""Sequence-sharded SANTA++ decode (hybrid estimator) over torch.distributed.

The reference decodes on one GPU (santapp_ruler README.md:355).  For long
contexts this module splits every sequence's clustered prefix ``[0,
sample_end)`` into contiguous shards, one per rank (one process per GPU).
Each shard clusters its own tokens, so a shard's summary lists its own
clusters and the cluster with row ``c`` on shard ``r`` has the global id
``cluster_base(r) + c``.  The recent window ``[sample_end, n_total)`` is
held by the last shard.  A decode step is

1. ``santa_shard_candidates``: each shard's top-k keys per (sequence, query
   head) (guess = log n + c.q*scale as in santapp.py:397-400, ranked
   descending with the lowest global id first on ties);
2. exchange 1: an all-gather of the keys (``B*Hq*k`` uint64 per rank);
3. ``santa_shard_plan``: every rank takes the same global top-k and selects
   its local clusters among them; it draws its share of the uniform samples
   from its own non-selected tokens (stratified: a sample of shard r weighs
   ``n_rest_r / samples_r``);
4. ``santa_shard_execute``: the gather attention over the shard's rows into
   an unnormalised partial ``(m, l, o)`` per (sequence, query head);
5. exchange 2: an all-gather of the partials (``B*Hq*(D+8)`` fp32 per rank);
6. ``santa_merge_shards``: the LSE merge, identical on every rank.

Both exchanges move a few hundred KB.  With ``transport="nccl"`` they are
NCCL all-gathers on the ranks' own buffers (six steps, four launches).  With
``transport="p2p"`` a step is two launches and no collective: the selection
launch scores the shard's clusters, stores its top-k keys straight into every
rank's exchange buffer (mapped through CUDA IPC) and reads every rank's keys
from its own buffer as they arrive (steps 1-3); the attention launch stores
the shard's partials the same way and merges every rank's in its tail (steps
4-6).  Each 8-byte word stored into a peer's buffer carries the step's epoch
beside its data, so the consumer polls its own memory and needs no flag or
fence; every wait is bounded, and a wait that runs out sets ``p2p_error``
and turns the step's outputs into NaN (``ShardedDecodeStep`` raises on the
next call).  Either way remote data lands in local memory before a kernel
reads it; no TMA or multicast is involved.  ``ShardExchange`` holds the host
logic (shard bounds, sample split, Philox seeds, exchange buffers and order)
apart from the kernel calls, so that it can be checked on CPU ranks.
"""

from __future__ import annotations

import ctypes
import math

import torch

from .. import _lib
from .santapp import ClusterSummary, _geometry, _require_cuda, decode_params

__all__ = ["shard_bounds", "split_counts", "shard_seed", "exchange_layout", "key_words",
           "partial_words", "ShardExchange", "ShardedDecodeStep"]

_GOLDEN = 0x9E3779B97F4A7C15


def shard_bounds(n: int, num_shards: int) -> list[tuple[int, int]]:
    """Contiguous ``[start, end)`` shards of ``[0, n)``; sizes differ by at
    most one, the larger ones first."""
    if num_shards < 1 or n < num_shards:
        raise ValueError(f"cannot split {n} tokens into {num_shards} non-empty shards")
    base, extra = divmod(n, num_shards)
    out, s = [], 0
    for r in range(num_shards):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


def split_counts(total: int, weights) -> list[int]:
    """Integers proportional to ``weights`` that sum to ``total`` (largest
    remainder; ties go to the lower index)."""
    weights = [int(w) for w in weights]
    wsum = sum(weights)
    if wsum <= 0:
        raise ValueError("weights must have a positive sum")
    exact = [total * w / wsum for w in weights]
    out = [int(math.floor(x)) for x in exact]
    left = total - sum(out)
    order = sorted(range(len(weights)), key=lambda i: (-(exact[i] - out[i]), i))
    for i in order[:left]:
        out[i] += 1
    return out


def shard_seed(seed: int, shard: int) -> int:
    """Philox key of shard ``shard``: independent draw streams per shard."""
    return (int(seed) + int(shard) * _GOLDEN) & 0xFFFFFFFFFFFFFFFF


def exchange_layout(num_shards: int, rows: int, topk: int, head_dim: int) -> dict:
    """Byte offsets of the regions of a peer-memory exchange buffer (the
    layout the kernels use): ``keys`` u64 [2 parities][num_shards][rows][topk],
    ``parts`` u64 [2][num_shards][rows][head_dim + 8] (one word per partial
    float), ``stage`` f32 [rows][head_dim + 8], ``bytes`` in all."""
    pf = _lib.partial_floats(head_dim)
    keys = 1024
    parts = (keys + 2 * num_shards * rows * topk * 8 + 255) // 256 * 256
    stage = parts + 2 * num_shards * rows * pf * 8
    return {"keys": keys, "parts": parts, "stage": stage, "bytes": stage + rows * pf * 4}


def key_words(keys: torch.Tensor, epoch: int) -> torch.Tensor:
    """Candidate keys (int64, as santa_shard_candidates writes them) as the
    words the peer-memory exchange stores for step ``epoch``: the tag
    ``epoch % 255 + 1`` in bits 24-31 of each key."""
    tag = epoch % 255 + 1
    # -0xFF000001 is the 64-bit mask 0xFFFFFFFF00FFFFFF as a signed integer
    return (keys & -0xFF000001) | (tag << 24)


def partial_words(partial: torch.Tensor, epoch: int) -> torch.Tensor:
    """Partials (fp32, as santa_shard_execute writes them) as the words the
    peer-memory exchange stores for step ``epoch``: ``epoch`` (32 bits) in
    the high half of each word, the float's bits in the low half."""
    bits = partial.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    tag = epoch & 0xFFFFFFFF
    if tag >= 1 << 31:
        tag -= 1 << 32
    return bits | (tag << 32)


class ShardExchange:
    """Exchange buffers and collectives of one rank (kernel calls elsewhere).

    ``group`` is a torch.distributed process group (or None with
    ``num_shards == 1``); the all-gathers run on the current stream."""

    def __init__(self, *, rows: int, topk: int, head_dim: int, shard_index: int,
                 num_shards: int, device, group=None):
        if not 0 <= shard_index < num_shards:
            raise ValueError("shard_index out of range")
        if num_shards > _lib.MAX_SHARDS or topk * num_shards > _lib.SHARD_MAX_KEYS:
            raise ValueError(f"{num_shards} shards x top-{topk} exceeds the candidate key limit "
                             f"({_lib.SHARD_MAX_KEYS})")
        self.rows, self.topk, self.head_dim = rows, topk, head_dim
        self.shard_index, self.num_shards, self.group = shard_index, num_shards, group
        pf = _lib.partial_floats(head_dim)
        self.keys = torch.zeros(rows * topk, dtype=torch.int64, device=device)
        self.all_keys = torch.zeros(num_shards, rows * topk, dtype=torch.int64, device=device)
        self.partial = torch.zeros(rows, pf, dtype=torch.float32, device=device)
        self.all_partials = torch.zeros(num_shards, rows, pf, dtype=torch.float32, device=device)

    def _all_gather(self, out: torch.Tensor, inp: torch.Tensor) -> None:
        if self.num_shards == 1:
            out[0].copy_(inp)
            return
        import torch.distributed as dist
        if not dist.is_initialized():
            raise RuntimeError("sharded decode over several ranks needs torch.distributed")
        dist.all_gather_into_tensor(out.view(-1), inp.reshape(-1), group=self.group)

    def exchange_keys(self) -> torch.Tensor:
        """Exchange 1: every shard's candidate keys, shard-major."""
        self._all_gather(self.all_keys, self.keys)
        return self.all_keys

    def exchange_partials(self) -> torch.Tensor:
        """Exchange 2: every shard's partials, shard-major."""
        self._all_gather(self.all_partials, self.partial)
        return self.all_partials


class ShardedDecodeStep(ShardExchange):
    """One rank's sequence shard of a hybrid SANTA++ decode step.

    key_cache / value_cache: ``[B, Hkv, capacity, D]`` bf16 cache of this
    shard's tokens (its old-prefix slice, plus the recent window on the last
    shard); ``summary`` this shard's cluster summary (local cluster rows,
    ``sample_end`` = the shard's old-prefix length); ``n_total`` the shard's
    token count; ``samples`` this shard's share of the per-head sample budget
    (``split_counts`` of the budget by shard token counts)."""

    def __init__(self, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 summary: ClusterSummary, *, num_query_heads: int, n_total: int,
                 topk_clusters: int, samples: int, shard_index: int, num_shards: int,
                 cluster_base: int, group=None, scale: float | None = None, seed: int = 0,
                 injected: bool = False, transport: str = "nccl", wait_limit_us: int = 0):
        _require_cuda("key_cache", key_cache)
        _require_cuda("value_cache", value_cache)
        if key_cache.dtype != torch.bfloat16:
            raise ValueError("sharded decode runs on bf16 caches")
        B, Hkv, _, D = key_cache.shape
        super().__init__(rows=B * num_query_heads, topk=topk_clusters, head_dim=D,
                         shard_index=shard_index, num_shards=num_shards,
                         device=key_cache.device, group=group)
        self.key_cache, self.value_cache, self.summary = key_cache, value_cache, summary
        self.geo = _geometry(key_cache, num_query_heads, n_total, summary.sample_end)
        self.scale = 1.0 / math.sqrt(D) if scale is None else scale
        self.p = decode_params("hybrid", topk_clusters=topk_clusters, samples=samples,
                               scale=self.scale, injected=injected,
                               seed=shard_seed(seed, shard_index))
        self.c = summary.as_c()
        self.lib = _lib.load()
        self.shard = _lib.SantaShard(shard_index, num_shards, int(cluster_base), 0,
                                     self.all_keys.data_ptr(), None)
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.wait_limit_us = int(wait_limit_us)
        self.epoch = 0
        self.p2p = None
        self._err_host = None
        self._err_event = None
        self._p2p_buffers: list[int] = []  # every rank's buffer as mapped here
        self._p2p_owned = False
        nbytes = ctypes.c_size_t()
        _lib.check("santa_decode_workspace_bytes", self.lib.santa_decode_workspace_bytes(
            ctypes.byref(self.geo), ctypes.byref(self.p), summary.max_groups,
            ctypes.byref(nbytes)))
        self.ws_bytes = nbytes.value
        dev = key_cache.device
        self.ws = torch.empty(max(1, self.ws_bytes), dtype=torch.uint8, device=dev)
        self.out = torch.empty(B, num_query_heads, D, dtype=torch.float32, device=dev)
        self.lse = torch.empty(B, num_query_heads, dtype=torch.float32, device=dev)
        self.ess = torch.empty(B, num_query_heads, dtype=torch.float32, device=dev)
        self._q = None
        self._refs = (ctypes.byref(self.geo), ctypes.byref(self.p), ctypes.byref(self.c),
                      ctypes.byref(self.shard))
        if transport == "p2p" and num_shards > 1:
            self._p2p_setup(group)

    # ---- peer-memory exchange (transport="p2p") -----------------------------
    def p2p_buffer_bytes(self) -> int:
        n = ctypes.c_size_t()
        _lib.check("santa_p2p_buffer_bytes", self.lib.santa_p2p_buffer_bytes(
            self.num_shards, self.rows, self.topk, self.head_dim, ctypes.byref(n)))
        return n.value

    def bind_p2p(self, buffers: list[int], *, owned: bool = False,
                 epoch_base: int | None = None) -> None:
        """Use the exchange buffers ``buffers`` (device addresses of every
        rank's buffer as mapped in this process, own one at shard_index).

        Every rank must bind at the same point, with the same
        ``epoch_base``: the first step then uses epoch ``epoch_base + 1``.
        Buffers fresh from ``santa_p2p_alloc`` (zeroed) work with any base;
        buffers that an earlier binding used need a base at or above that
        binding's last epoch (its ``epoch``), or a stale word of that run
        could pass for a new one."""
        dev = self.out.device
        self._p2p_buffers = list(buffers)
        self._p2p_owned = owned
        if epoch_base is not None:
            self.epoch = int(epoch_base)
        self._peer_table = torch.tensor(buffers, dtype=torch.int64, device=dev)
        self.p2p_error = torch.zeros(1, dtype=torch.int32, device=dev)
        self._err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._err_event = torch.cuda.Event()
        self._err_step = None
        self.p2p = _lib.SantaP2P(self._peer_table.data_ptr(), buffers[self.shard_index], 0,
                                 self.p2p_error.data_ptr(), self.rows, self.topk,
                                 _lib.partial_floats(self.head_dim), self.wait_limit_us)
        self.shard.p2p = ctypes.addressof(self.p2p)
        self.transport = "p2p"

    def check_p2p(self) -> None:
        """Raise if a peer-memory wait ran out (waits for the device)."""
        if self.p2p is not None and int(self.p2p_error.item()) != 0:
            raise RuntimeError("sequence-shard exchange: a wait for a peer rank ran out of time; "
                               "the outputs of that step and of later steps are NaN")

    def _poll_p2p_error(self, step: int, stream=None) -> None:
        """Cheap asynchronous check: the previous step's error flag, copied
        to pinned memory behind it, raises once it has landed; then this
        step's flag is queued the same way."""
        if self._err_step is not None and self._err_event.query() and int(self._err_host[0]):
            raise RuntimeError(f"sequence-shard exchange: a wait for a peer rank ran out of "
                               f"time at or before step {self._err_step}; its outputs are NaN")
        s = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            self._err_host.copy_(self.p2p_error, non_blocking=True)
            self._err_event.record(s)
        self._err_step = step

    def _p2p_setup(self, group) -> None:
        """Allocate this rank's exchange buffer, share its IPC handle through
        the process group, map the peers' buffers and check each mapping by
        reading a marker its owner wrote."""
        import torch.distributed as dist
        lib, dev = self.lib, self.out.device
        own = ctypes.c_void_p()
        _lib.check("santa_p2p_alloc", lib.santa_p2p_alloc(self.p2p_buffer_bytes(),
                                                          ctypes.byref(own)))
        handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        _lib.check("santa_p2p_ipc_handle", lib.santa_p2p_ipc_handle(own, handle))
        mine = torch.tensor(bytearray(handle), dtype=torch.uint8, device=dev)
        every = torch.empty(self.num_shards * _lib.IPC_HANDLE_BYTES, dtype=torch.uint8,
                            device=dev)
        dist.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().numpy().reshape(self.num_shards, _lib.IPC_HANDLE_BYTES)
        marker_off = 768  # unused bytes of the counter block
        _lib.check("santa_p2p_poke", lib.santa_p2p_poke(own.value + marker_off,
                                                        0x5A5A0000 + self.shard_index))
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)
        buffers = []
        for r in range(self.num_shards):
            if r == self.shard_index:
                buffers.append(own.value)
                continue
            mapped = ctypes.c_void_p()
            h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)(*every[r].tolist())
            _lib.check("santa_p2p_ipc_open", lib.santa_p2p_ipc_open(h, ctypes.byref(mapped)))
            seen = ctypes.c_uint64()
            _lib.check("santa_p2p_peek", lib.santa_p2p_peek(mapped.value + marker_off,
                                                            ctypes.byref(seen)))
            if seen.value != 0x5A5A0000 + r:
                raise RuntimeError(f"exchange buffer of rank {r} is not mapped correctly")
            buffers.append(mapped.value)
        dist.barrier(group=group)
        self.bind_p2p(buffers, owned=True)

    def close(self) -> None:
        """Unmap the peers' exchange buffers and free this rank's."""
        if self._p2p_owned and self._p2p_buffers:
            for r, ptr in enumerate(self._p2p_buffers):
                if r == self.shard_index:
                    self.lib.santa_p2p_free(ctypes.c_void_p(ptr))
                else:
                    self.lib.santa_p2p_ipc_close(ctypes.c_void_p(ptr))
        self._p2p_buffers = []
        self._p2p_owned = False

    # ---- the kernel calls -------------------------------------------------
    def begin(self, q: torch.Tensor, step: int = 0) -> None:
        """Start step ``step`` with queries ``q``: the Philox step counter and
        the exchange epoch (one per step, the same sequence on every rank)."""
        self.p.step = int(step) & 0xFFFFFFFFFFFFFFFF
        self._q = q
        self.epoch += 1
        if self.p2p is not None:
            self.p2p.epoch = self.epoch

    def candidates(self, q: torch.Tensor, step: int = 0, stream=None) -> torch.Tensor:
        """NCCL transport, step 1: this shard's top-k keys into ``keys``."""
        self.begin(q, step)
        if self.p2p is not None:
            raise RuntimeError("with the peer-memory exchange, plan() runs the candidates pass")
        g, p, c, s = self._refs
        _lib.check("santa_shard_candidates", self.lib.santa_shard_candidates(
            g, p, q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(), c, s,
            self.keys.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
            _lib.stream_handle(stream)))
        return self.keys

    def plan(self, sample_a: torch.Tensor | None = None, n_exact: torch.Tensor | None = None,
             stream=None) -> None:
        """Step 3 (NCCL: after exchange 1); with the peer-memory exchange
        steps 1-3 in one launch."""
        g, p, c, s = self._refs
        _lib.check("santa_shard_plan", self.lib.santa_shard_plan(
            g, p, self._q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(),
            c, s, _lib.ptr(sample_a), _lib.ptr(n_exact), self.ws.data_ptr(), self.ws_bytes,
            _lib.stream_handle(stream)))

    def execute(self, stream=None) -> torch.Tensor:
        """Step 4 (NCCL: the partial, returned); with the peer-memory
        exchange steps 4-6 in one launch (the merged output, returned)."""
        g, p, c, s = self._refs
        if self.p2p is not None:
            _lib.check("santa_shard_attend", self.lib.santa_shard_attend(
                g, p, self._q.data_ptr(), self.key_cache.data_ptr(),
                self.value_cache.data_ptr(), c, s, self.out.data_ptr(), self.lse.data_ptr(),
                self.ess.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
                _lib.stream_handle(stream)))
            return self.out
        _lib.check("santa_shard_execute", self.lib.santa_shard_execute(
            g, p, self._q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(),
            c, s, self.partial.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
            _lib.stream_handle(stream)))
        return self.partial

    def merge(self, stream=None) -> torch.Tensor:
        """Step 6 (NCCL transport; the peer-memory attention launch merged)."""
        if self.p2p is not None:
            return self.out
        _lib.check("santa_merge_shards", self.lib.santa_merge_shards(
            self.rows, self.head_dim, self.num_shards, self.all_partials.data_ptr(),
            self.out.data_ptr(), self.lse.data_ptr(), self.ess.data_ptr(),
            _lib.stream_handle(stream)))
        return self.out

    def exchange_keys(self) -> torch.Tensor:
        if self.p2p is not None:
            return self.all_keys  # the kernels exchanged them through peer memory
        return super().exchange_keys()

    def exchange_partials(self) -> torch.Tensor:
        if self.p2p is not None:
            return self.all_partials
        return super().exchange_partials()

    def select(self, sample_a: torch.Tensor | None = None):
        """Selection readout of the plan (after exchange 1): ``(selected
        [B, Hq, G_local] uint8, sample_rows [B, Hq, samples] int32, n_exact)``."""
        B, Hq = self.out.shape[:2]
        dev = self.out.device
        sel = torch.zeros(B, Hq, self.summary.max_groups, dtype=torch.uint8, device=dev)
        rows = torch.full((B, Hq, max(1, self.p.samples)), -1, dtype=torch.int32, device=dev)
        n_exact = torch.zeros(B, Hq, dtype=torch.int32, device=dev)
        g, p, c, s = self._refs
        _lib.check("santa_shard_select", self.lib.santa_shard_select(
            g, p, self._q.data_ptr(), self.key_cache.data_ptr(), self.value_cache.data_ptr(),
            c, s, _lib.ptr(sample_a), sel.data_ptr(), rows.data_ptr(), n_exact.data_ptr(),
            self.ws.data_ptr(), self.ws_bytes, _lib.stream_handle(None)))
        return sel, rows[..., : self.p.samples], n_exact

    # ---- one decode step --------------------------------------------------
    def __call__(self, q: torch.Tensor, step: int = 0, sample_a: torch.Tensor | None = None):
        """The whole step on the current stream; returns ``out [B, Hq, D]``
        (identical on every rank)."""
        if self.p2p is not None:
            self.begin(q, step)
            self.plan(sample_a)
            out = self.execute()
            self._poll_p2p_error(step)
            return out
        self.candidates(q, step)
        self.exchange_keys()
        self.plan(sample_a)
        self.execute()
        self.exchange_partials()
        return self.merge()

    @property
    def kernels_per_call(self) -> int:
        # peer memory: select, attend; NCCL: candidates, select, attend, merge
        return 2 if self.p2p is not None else 4
