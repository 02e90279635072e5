"""Seeded synthetic decode workloads with the shapes of the Qwen attention layers.

There is no model or dataset on the machines this runs on, so every workload is
a Gaussian-mixture key cache: per KV head, ``centers ~ N(0,1)[G_true, D]``,
``assign ~ randint(G_true)``, ``K = centers[assign] + sigma * N(0,1)``,
``V ~ N(0,1)`` and queries ``q ~ N(0,1)`` (optionally pre-scaled).  Draws come
from one ``torch.Generator`` seeded once, in the order centers -> assign ->
key noise -> values -> queries, so a workload is a pure function of its
parameters and seed.

The sampled old prefix is ``[0, sample_end)`` with ``sample_end = T - W``
(``W`` = recent window, 64 by default as in santapp_ruler/config.py:76); the
tokens ``[sample_end, T)`` are attended exactly.
"""

from __future__ import annotations

import hashlib
import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class DecodeShape:
    """Attention geometry of one decode workload."""

    name: str
    num_query_heads: int
    num_kv_heads: int
    head_dim: int
    batch: int
    context: int
    true_clusters: int
    sigma: float
    kv_dtype: torch.dtype
    n_clusters: int
    topk_clusters: int
    samples: int
    recent_window: int = 64
    query_scale: float = 1.0
    steps: int = 1

    @property
    def group(self) -> int:
        return self.num_query_heads // self.num_kv_heads

    @property
    def sample_end(self) -> int:
        return self.context - self.recent_window

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)


# Qwen2.5-0.5B attention shape, fp32, one decode step (CPU-runnable case).
QWEN05B_4K = DecodeShape(
    name="qwen2.5-0.5b-attn-ctx4096",
    num_query_heads=14, num_kv_heads=2, head_dim=64, batch=1, context=4096,
    true_clusters=64, sigma=0.3, kv_dtype=torch.float32, n_clusters=64,
    topk_clusters=8, samples=64, query_scale=1.0 / math.sqrt(64), steps=1,
)

# Qwen2.5-7B attention shape, bf16 K/V, batch 8 at 32K context, 128 steps.
QWEN7B_32K = DecodeShape(
    name="qwen2.5-7b-attn-ctx32768-b8",
    num_query_heads=28, num_kv_heads=4, head_dim=128, batch=8, context=32768,
    true_clusters=256, sigma=0.25, kv_dtype=torch.bfloat16, n_clusters=256,
    topk_clusters=16, samples=256, steps=128,
)

# Qwen3-8B attention shape, bf16 K/V, batch 16 at 128K context, 64 steps.
QWEN3_8B_128K = DecodeShape(
    name="qwen3-8b-attn-ctx131072-b16",
    num_query_heads=32, num_kv_heads=8, head_dim=128, batch=16, context=131072,
    true_clusters=1024, sigma=0.25, kv_dtype=torch.bfloat16, n_clusters=1024,
    topk_clusters=32, samples=512, steps=64,
)

SHAPES = {s.name: s for s in (QWEN05B_4K, QWEN7B_32K, QWEN3_8B_128K)}


def scaled_shape(base: DecodeShape, **changes) -> DecodeShape:
    """A copy of ``base`` with some fields replaced (smaller test cases)."""
    fields = {k: getattr(base, k) for k in base.__dataclass_fields__}
    fields.update(changes)
    return DecodeShape(**fields)


@dataclass
class DecodeWorkload:
    shape: DecodeShape
    keys: torch.Tensor        # [B, Hkv, T, D] kv_dtype
    values: torch.Tensor      # [B, Hkv, T, D] kv_dtype
    labels: torch.Tensor      # [B, Hkv, T] int64 ground-truth mixture component
    queries: torch.Tensor     # [steps, B, Hq, D] fp32


def make_decode_workload(shape: DecodeShape, seed: int = 0,
                         device: str | torch.device = "cpu") -> DecodeWorkload:
    """Draw the Gaussian-mixture K/V cache and the per-step queries."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    B, H, T, D, G = (shape.batch, shape.num_kv_heads, shape.context,
                     shape.head_dim, shape.true_clusters)
    f32 = torch.float32
    centers = torch.randn(B, H, G, D, generator=gen, device=device, dtype=f32)
    assign = torch.randint(0, G, (B, H, T), generator=gen, device=device)
    noise = torch.randn(B, H, T, D, generator=gen, device=device, dtype=f32)
    keys = torch.gather(centers, 2, assign[..., None].expand(B, H, T, D))
    keys = keys.add_(noise, alpha=shape.sigma)
    del noise
    values = torch.randn(B, H, T, D, generator=gen, device=device, dtype=f32)
    queries = torch.randn(shape.steps, B, shape.num_query_heads, D,
                          generator=gen, device=device, dtype=f32)
    if shape.query_scale != 1.0:
        queries.mul_(shape.query_scale)
    return DecodeWorkload(
        shape=shape,
        keys=keys.to(shape.kv_dtype),
        values=values.to(shape.kv_dtype),
        labels=assign,
        queries=queries,
    )


def tensor_digest(*tensors: torch.Tensor) -> str:
    """sha256 over the raw bytes of CPU tensors (fixture drift guard)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous().cpu()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()


@dataclass
class ShardWorkload:
    """One sequence shard of a decode workload (see ``make_shard_workload``)."""

    keys: torch.Tensor        # [B, Hkv, n_total, D] this shard's tokens
    values: torch.Tensor
    labels: torch.Tensor      # [B, Hkv, sample_end] local cluster of each old token
    queries: torch.Tensor     # [steps, B, Hq, D] fp32, identical on every shard
    sample_end: int           # this shard's old-prefix tokens
    n_total: int              # sample_end (+ the recent window on the last shard)
    n_clusters: int           # this shard's clusters per (sequence, KV head)
    cluster_base: int         # global id of its cluster 0
    samples: int              # its share of the per-head sample budget


def make_shard_workload(shape: DecodeShape, shard_index: int, num_shards: int, seed: int = 0,
                        device: str | torch.device = "cpu") -> ShardWorkload:
    """Shard ``shard_index`` of ``num_shards`` contiguous sequence shards.

    The old prefix ``[0, sample_end)`` of every sequence is split into
    contiguous shards; shard r holds its slice plus, on the last shard, the
    recent window.  The Gaussian mixture's ``true_clusters`` components are
    split across the shards too (a shard's tokens come from its own
    components, which are its clusters), and so is the sample budget, in
    proportion to the shards' token counts.  Each shard draws its cache from
    its own generator (seed, shard); the queries come from a generator seeded
    with ``seed`` alone, so every rank sees the same queries."""
    from .attention.sharded import shard_bounds, split_counts
    bounds = shard_bounds(shape.sample_end, num_shards)
    sizes = [e - s for s, e in bounds]
    clusters = split_counts(shape.true_clusters, [1] * num_shards)
    if min(clusters) < 1:
        raise ValueError("fewer mixture components than shards")
    r = shard_index
    old = sizes[r]
    n_total = old + (shape.recent_window if r == num_shards - 1 else 0)
    G = clusters[r]
    B, H, D = shape.batch, shape.num_kv_heads, shape.head_dim
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed) * 1_000_003 + 1 + r)
    f32 = torch.float32
    centers = torch.randn(B, H, G, D, generator=gen, device=device, dtype=f32)
    assign = torch.randint(0, G, (B, H, n_total), generator=gen, device=device)
    keys = torch.gather(centers, 2, assign[..., None].expand(B, H, n_total, D))
    keys.add_(torch.randn(B, H, n_total, D, generator=gen, device=device, dtype=f32),
              alpha=shape.sigma)
    values = torch.randn(B, H, n_total, D, generator=gen, device=device, dtype=f32)
    qgen = torch.Generator(device=device)
    qgen.manual_seed(int(seed))
    queries = torch.randn(shape.steps, B, shape.num_query_heads, D, generator=qgen,
                          device=device, dtype=f32)
    if shape.query_scale != 1.0:
        queries.mul_(shape.query_scale)
    return ShardWorkload(
        keys=keys.to(shape.kv_dtype), values=values.to(shape.kv_dtype),
        labels=assign[:, :, :old].to(torch.int32).contiguous(), queries=queries,
        sample_end=old, n_total=n_total, n_clusters=G, cluster_base=sum(clusters[:r]),
        samples=split_counts(shape.samples, sizes)[r])
