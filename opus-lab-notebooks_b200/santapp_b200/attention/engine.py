"""Model-level SANTA++ engine on the sm_100a kernels.

Host-side mirror of ``SantaPlusEngine`` (santapp_ruler/attention/
santapp.py:145-926) for Qwen2 causal LMs, batched over sequences (the
reference supports batch 1, :293-294):

* ``patched()`` installs the same instance-level attention patch as the
  reference (:201-227) and restores it afterwards;
* ``_attention_forward`` (:285-363) runs the projections of the model, then
  one fused kernel for RoPE and the cache append (``santa_rope_append``,
  LayerCache :66-77 / :234-274), then
    - prefill (query tokens == key tokens): the tcgen05 causal attention
      ``santa_prefill`` over the cache in place,
    - sparse decode (one query token): ``santa_decode`` for every (sequence,
      query head) at once, in the configured mode,
    - dense decode (the fidelity path): torch SDPA over the cache, as the
      reference's dense branch does;
* ``_dense_prefill_and_cluster`` (:542-722): prefill, then per (layer, KV
  head, sequence) fingerprints (``build_fingerprints``), MiniBatchKMeans
  (``SklearnLikeTorchMiniBatchKMeans``) and the cluster summary
  (``build_summary``, batched over the layer);
* ``generate`` (:794-908): prefill + clustering, trim the cache by one token,
  re-feed the last prompt token, greedy decoding;
* ``_approximate_attention`` (:365-506): the reference's per-head call
  (one query head of sequence 0), kept for callers that drive the engine
  head by head; it routes to ``santa_decode`` on that head's summary.

The engine takes the reference's own ``SantaPlusConfig`` (config.py:68-78,
a slotted dataclass) or ``SantaB200Config``: fields the reference's config
lacks (``topk_clusters``, ``n_clusters``, ``kv_page_size``) fall back to
their defaults.  With ``kv_page_size`` set, every layer's cache is a
``PagedKVCache`` (page pools + block table, pages mapped as the sequences
grow): the append, the prefill, the summary build and the sparse decode all
read and write the pages directly; the dense fidelity path and the
clustering inputs gather the tokens they need.

Probe queries are captured inside the patched forward at the probe positions
only (the reference keeps every layer's full q_proj output).
"""

from __future__ import annotations

import contextlib
import math
import time
import types
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch

from .. import _lib
from .fingerprints import build_fingerprints, cluster_count, probe_positions
from .kmeans import SklearnLikeTorchMiniBatchKMeans
from .paged import PagedKVCache
from .prefill import santa_prefill
from .santapp import DecodeTrafficTracker, build_summary, santa_decode

__all__ = ["KMeansConfig", "SantaB200Config", "LayerCache", "SantaGeneration", "SantaB200Engine"]

_MISSING = object()


@dataclass
class KMeansConfig:
    """MiniBatchKMeansConfig of santapp_ruler/config.py."""
    batch_size: int = 4096
    n_init: int = 1
    max_iter: int = 100
    tol: float = 0.0
    max_no_improvement: int | None = 10
    init_size: int | None = None
    reassignment_ratio: float = 0.01
    random_state: int = 0


@dataclass
class SantaB200Config:
    """SantaPlusConfig (santapp_ruler/config.py:70-80) plus the hybrid
    estimator's exact-cluster count and an optional fixed cluster count."""
    mode: str = "guided"
    group_size: int = 16
    samples_per_head: int = 128
    probe_queries: int = 64
    recent_window: int = 64
    probe_region_start_fraction: float = 0.75
    probe_strategy: str = "end_quarter"
    sample_seed: int = 0
    kmeans: KMeansConfig = field(default_factory=KMeansConfig)
    topk_clusters: int = 16
    n_clusters: int | None = None
    kv_page_size: int | None = None   # paged KV cache (tokens per page, a power of two)


@dataclass
class LayerCache:
    """One layer's K/V (LayerCache, santapp.py:66-77, batched): contiguous
    ``[B, Hkv, capacity, D]`` tensors, or ``paged`` (key / value None)."""
    key: torch.Tensor | None     # [B, Hkv, capacity, D]
    value: torch.Tensor | None
    length: int
    paged: PagedKVCache | None = None

    @property
    def capacity(self) -> int:
        return self.paged.capacity if self.paged is not None else int(self.key.shape[2])

    def kv(self) -> tuple:
        """The (key_cache, value_cache) arguments of the santa_* entry points."""
        return (self.paged, None) if self.paged is not None else (self.key, self.value)

    def view(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Tokens [0, length) as [B, Hkv, length, D] tensors (a gather copy
        when paged)."""
        if self.paged is not None:
            return self.paged.to_contiguous(self.length)
        return self.key[:, :, : self.length], self.value[:, :, : self.length]


@dataclass(frozen=True)
class SantaGeneration:
    """Result of ``generate``: ``token_ids`` is ``list[int]`` for a batch of
    one sequence (the reference's SantaGeneration, santapp.py:145-148, which
    SantaPlusBackend.generate decodes directly) and one ``list[int]`` per
    sequence for larger batches."""
    token_ids: list[int] | list[list[int]]
    metrics: dict[str, Any]


# fields of SantaB200Config that the reference's SantaPlusConfig does not have
_EXTRA_DEFAULTS = {"topk_clusters": 16, "n_clusters": None, "kv_page_size": None}


def _patched_forward(attention, hidden_states, position_embeddings=None, attention_mask=None,
                     *args, **kwargs):
    del args, kwargs
    return attention._santa_engine._attention_forward(attention, hidden_states,
                                                      position_embeddings, attention_mask)


class SantaB200Engine:
    """Patch a loaded Qwen2 model only while running SANTA++ generation."""

    def __init__(self, model: Any, config: SantaB200Config):
        self.model = model
        self.config = config
        self.base_model = getattr(model, "model", None)
        if self.base_model is None or not hasattr(self.base_model, "layers"):
            raise TypeError("Expected a Hugging Face causal LM with model.layers.")
        cfg = model.config
        if getattr(cfg, "model_type", None) != "qwen2":
            raise TypeError(f"Qwen2/Qwen2.5 models only, not {cfg.model_type!r}.")
        if bool(getattr(cfg, "use_sliding_window", False)):
            raise NotImplementedError("use_sliding_window=True is unsupported.")
        self.num_layers = len(self.base_model.layers)
        self.num_query_heads = int(cfg.num_attention_heads)
        self.num_kv_heads = int(cfg.num_key_value_heads)
        if self.num_query_heads % self.num_kv_heads:
            raise ValueError("Query heads must be divisible by KV heads.")
        self.group = self.num_query_heads // self.num_kv_heads
        self.head_dim = int(getattr(cfg, "head_dim", None)
                            or cfg.hidden_size // cfg.num_attention_heads)
        self.mode = "dense"
        self.sample_end = 0
        self.cache_capacity = 0
        self.cache: dict[int, LayerCache] = {}
        self.summaries: dict[int, Any] = {}
        self.traffic = DecodeTrafficTracker()
        self._probe_idx: torch.Tensor | None = None
        self._probe_q: dict[int, torch.Tensor] = {}
        self._decode_step = 0
        self._n_groups_host: dict[int, np.ndarray] = {}
        self.track_traffic = True  # draw accounting, read back once per generate
        self._traffic_pending: list = []
        self._head_calls = 0
        self._capture_q: dict[int, torch.Tensor] | None = None
        self._plant_layer = None  # set during the planted-key dry run
        self._planted: dict | None = None
        self.log = None  # optional progress callback: log(message)
        self._prefill_flags: list[torch.Tensor] = []  # error words of the prefill launches
        self._lib = _lib.load()

    def _log(self, msg: str) -> None:
        if self.log is not None:
            self.log(msg)

    def _cfg(self, name: str):
        """A config field; SantaPlusConfig lacks the hybrid estimator's
        fields, which then take SantaB200Config's defaults."""
        return getattr(self.config, name, _EXTRA_DEFAULTS.get(name))

    # ---- patch ---------------------------------------------------------------
    @contextlib.contextmanager
    def patched(self):
        originals, attns = [], []
        try:
            for layer_id, layer in enumerate(self.base_model.layers):
                attn = layer.self_attn
                originals.append(attn.__dict__.get("forward", _MISSING))
                attns.append(attn)
                attn._santa_engine = self
                attn._santa_layer_id = layer_id
                attn.forward = types.MethodType(_patched_forward, attn)
            yield
        finally:
            for attn, orig in zip(attns, originals):
                if orig is _MISSING:
                    attn.__dict__.pop("forward", None)
                else:
                    attn.forward = orig
                attn.__dict__.pop("_santa_engine", None)
                attn.__dict__.pop("_santa_layer_id", None)

    def clear(self) -> None:
        self.cache.clear()
        self.summaries.clear()
        self._probe_q.clear()
        self._n_groups_host.clear()
        self._traffic_pending = []
        self._planted = None
        self.traffic = DecodeTrafficTracker()

    def _trim_cache(self, length: int) -> None:
        for layer_id, c in self.cache.items():
            if c.length < length:
                raise RuntimeError(f"Layer {layer_id} cache has only {c.length} tokens; "
                                   f"cannot trim to {length}.")
            c.length = length

    # ---- attention -----------------------------------------------------------
    def _attention_forward(self, attention, hidden_states, position_embeddings, attention_mask):
        if position_embeddings is None:
            raise RuntimeError("Qwen did not supply position_embeddings.")
        B, Tn, _ = hidden_states.shape
        Hq, Hkv, D = self.num_query_heads, self.num_kv_heads, self.head_dim
        q = attention.q_proj(hidden_states)
        k = attention.k_proj(hidden_states)
        v = attention.v_proj(hidden_states)
        if q.dtype != torch.bfloat16:
            raise ValueError("the engine runs bf16 models")
        cos, sin = position_embeddings
        cos = cos.to(torch.bfloat16).expand(B, Tn, D).contiguous()
        sin = sin.to(torch.bfloat16).expand(B, Tn, D).contiguous()
        layer_id = int(attention._santa_layer_id)
        cached = self.cache.get(layer_id)
        if cached is None:
            cap = max(self.cache_capacity, Tn)
            cap = (cap + 7) // 8 * 8
            page_size = self._cfg("kv_page_size")
            if page_size:
                cached = LayerCache(None, None, 0, PagedKVCache.allocate(
                    B, Hkv, D, max_tokens=cap, page_size=int(page_size), device=q.device))
            else:
                kb = torch.empty(B, Hkv, cap, D, dtype=torch.bfloat16, device=q.device)
                cached = LayerCache(kb, torch.empty_like(kb), 0)
            self.cache[layer_id] = cached
        start = cached.length
        if start + Tn > cached.capacity:
            raise RuntimeError(f"SANTA++ cache capacity exceeded in layer {layer_id}: need "
                               f"{start + Tn}, allocated {cached.capacity}.")
        sparse_decode = Tn == 1 and self.mode != "dense"
        q_bf = None if sparse_decode else torch.empty(B, Hq, Tn, D, dtype=torch.bfloat16,
                                                      device=q.device)
        q_f32 = torch.empty(B, Hq, Tn, D, dtype=torch.float32, device=q.device) \
            if sparse_decode else None
        if cached.paged is not None:   # maps the pages the new tokens need
            cached.paged.append(q.contiguous().view(B, Tn, Hq, D),
                                k.contiguous().view(B, Tn, Hkv, D),
                                v.contiguous().view(B, Tn, Hkv, D), cos, sin, start,
                                q_rot_bf16=q_bf, q_rot_f32=q_f32)
        else:
            _lib.check("santa_rope_append", self._lib.santa_rope_append(
                B, Tn, Hq, Hkv, D, q.contiguous().data_ptr(), k.contiguous().data_ptr(),
                v.contiguous().data_ptr(), cos.data_ptr(), sin.data_ptr(),
                cached.key.data_ptr(), cached.value.data_ptr(), cached.capacity, start,
                _lib.ptr(q_bf), _lib.ptr(q_f32), _lib.stream_handle()))
        cached.length = start + Tn
        if sparse_decode:
            res = santa_decode(q_f32[:, :, 0].contiguous(), *cached.kv(),
                               self.summaries[layer_id], mode=self.config.mode,
                               n_total=cached.length, sample_end=self.sample_end,
                               topk_clusters=self._cfg("topk_clusters"),
                               token_budget=self.config.samples_per_head,
                               samples=self.config.samples_per_head,
                               scale=float(attention.scaling), seed=self.config.sample_seed,
                               step=self._decode_step, with_stats=self.track_traffic)
            if self.track_traffic:
                # kept on the device; read back once when generate finishes
                if layer_id not in self._n_groups_host:
                    self._n_groups_host[layer_id] = self.summaries[layer_id].n_groups
                self._traffic_pending.append((cached.length, layer_id, res.n_exact.clone(),
                                              res.ess.clone()))
            if self._planted is not None and self._decode_step == 0:
                self._check_planted(layer_id, q_f32[:, :, 0].contiguous(), cached,
                                    float(attention.scaling))
            out = res.out.to(torch.bfloat16).view(B, 1, Hq * D)
        elif start == 0:
            # prompt: causal attention of every position over the prompt
            out = santa_prefill(q_bf, *cached.kv(), causal=True,
                                scale=float(attention.scaling))
            self._prefill_flags.append(out._santa_error_flag)
            if self.log is not None:  # progress (synchronises: diagnostics only)
                torch.cuda.synchronize()
                self._log(f"layer {layer_id} prefill attention done, error flag "
                          f"{int(out._santa_error_flag.item())}")
            if self._probe_idx is not None:
                self._probe_q[layer_id] = q_bf[:, :, self._probe_idx].float()
            out = out.transpose(1, 2).reshape(B, Tn, Hq * D)
        else:
            # dense decode / continued prompt over the cache (fidelity path)
            if self._capture_q is not None and Tn == 1:
                self._capture_q[layer_id] = q_bf[:, :, 0].float()
                if self._plant_layer is not None:
                    self._plant_layer(layer_id, q_bf[:, :, 0].float(), cached)
            kf, vf = cached.view()
            kf = kf.repeat_interleave(self.group, dim=1)
            vf = vf.repeat_interleave(self.group, dim=1)
            mask = None
            if Tn > 1:
                qa = torch.arange(start, start + Tn, device=q.device)[:, None]
                mask = (torch.arange(cached.length, device=q.device)[None, :] <= qa)[None, None]
            out = torch.nn.functional.scaled_dot_product_attention(
                q_bf, kf, vf, attn_mask=mask, scale=float(attention.scaling))
            out = out.transpose(1, 2).reshape(B, Tn, Hq * D)
        return attention.o_proj(out.contiguous()), None

    # ---- prefill and clustering ---------------------------------------------
    @torch.inference_mode()
    def _dense_prefill_and_cluster(self, input_ids: torch.Tensor, *, probe_seed: int):
        prefill_s, sample_end = self._prefill(input_ids, probe_seed=probe_seed)
        cluster_s, n_clusters = self._cluster()
        return prefill_s, cluster_s, sample_end, n_clusters

    @torch.inference_mode()
    def _prefill(self, input_ids: torch.Tensor, *, probe_seed: int):
        """Dense prefill of the prompt into the caches, keeping every layer's
        queries at the probe positions (santapp.py:542-597)."""
        B, T = input_ids.shape
        sample_end = T - 1 - self.config.recent_window
        if sample_end < 2:
            raise ValueError(f"Prompt has {T} tokens, too short for recent_window="
                             f"{self.config.recent_window}.")
        self.sample_end = sample_end
        self.mode = "dense"
        probes = probe_positions(self.config.probe_strategy, T, self.config.probe_queries,
                                 region_start_fraction=self.config.probe_region_start_fraction,
                                 probe_seed=probe_seed)
        self._probe_idx = torch.as_tensor(probes, dtype=torch.long, device=input_ids.device)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        self._prefill_flags = []
        try:
            self.model(input_ids, use_cache=False, logits_to_keep=1)
        finally:
            self._probe_idx = None
        torch.cuda.synchronize()
        if self._prefill_flags and int(torch.stack(self._prefill_flags).max()):
            raise RuntimeError("santa_prefill: a bounded wait of the prefill kernel gave up "
                               "(its output is invalid)")
        return time.perf_counter() - t0, sample_end

    @torch.inference_mode()
    def _cluster(self, workers: int | None = None):
        """Fingerprints, MiniBatchKMeans and the cluster summary of every
        (layer, KV head, sequence) over the old prefix (santapp.py:598-722).

        The fits are independent and each one is a chain of small launches
        with a host read-back per mini-batch (the reference's control flow),
        so they run concurrently: a pool of host threads, each fit on its own
        CUDA stream (the ctypes calls and torch's copies release the GIL)."""
        import concurrent.futures as cf
        sample_end = self.sample_end
        n_clusters = self._cfg("n_clusters") or cluster_count(sample_end, self.config.group_size)
        km = self.config.kmeans
        t1 = time.perf_counter()
        layers = list(range(self.num_layers))
        probes = {layer_id: self._probe_q.pop(layer_id) for layer_id in layers}
        B = probes[0].shape[0]
        dev = probes[0].device
        labels = {layer_id: torch.empty(B, self.num_kv_heads, sample_end, dtype=torch.int32,
                                        device=dev) for layer_id in layers}
        jobs = [(layer_id, b, kv) for layer_id in layers for b in range(B)
                for kv in range(self.num_kv_heads)]
        n_workers = workers or min(16, len(jobs))
        streams = [torch.cuda.Stream(device=dev) for _ in range(n_workers)]
        main = torch.cuda.current_stream(dev)
        ready = torch.cuda.Event()
        ready.record(main)  # the caches and probe queries are complete

        def fit(i, job):
            layer_id, b, kv = job
            st = streams[i % n_workers]
            # (inference mode is per thread: the worker enters it as well)
            with torch.inference_mode(), torch.cuda.device(dev), torch.cuda.stream(st):
                st.wait_event(ready)
                qp = probes[layer_id]
                P = qp.shape[2]
                c = self.cache[layer_id]
                keys = (c.paged.tokens(b, kv, sample_end) if c.paged is not None
                        else c.key[b, kv, :sample_end])
                fp = build_fingerprints(keys, qp[b].contiguous(), kv, self.group,
                                        np.arange(P))
                est = SklearnLikeTorchMiniBatchKMeans(
                    n_clusters, batch_size=km.batch_size, n_init=km.n_init,
                    max_iter=km.max_iter, tol=km.tol,
                    max_no_improvement=km.max_no_improvement, init_size=km.init_size,
                    reassignment_ratio=km.reassignment_ratio, random_state=km.random_state)
                labels[layer_id][b, kv].copy_(est.fit_predict(fp).to(torch.int32))
                if i % 64 == 63:
                    self._log(f"k-means fit {i + 1} of {len(jobs)}")
                done = torch.cuda.Event()
                done.record(st)
                return done

        if n_workers == 1:
            events = [fit(i, j) for i, j in enumerate(jobs)]
        else:
            # worker w runs jobs w, w + n, ... in order on stream w
            def run_lane(w):
                return [fit(i, jobs[i]) for i in range(w, len(jobs), n_workers)]
            with cf.ThreadPoolExecutor(n_workers) as pool:
                events = [e for lane in pool.map(run_lane, range(n_workers)) for e in lane]
        for e in events:
            main.wait_event(e)
        for layer_id in layers:
            cached = self.cache[layer_id]
            self.summaries[layer_id] = build_summary(*cached.kv(),
                                                     labels[layer_id], n_clusters,
                                                     sample_end=sample_end,
                                                     n_total=cached.length)
        torch.cuda.synchronize()
        return time.perf_counter() - t1, n_clusters

    # ---- planted-key retrieval check ------------------------------------------
    @torch.inference_mode()
    def _plant_keys(self, last_token: torch.Tensor, position: int, *, n_planted: int,
                    scale: float, seed: int) -> dict:
        """Synthetic retrieval check: for every (layer, sequence, KV head),
        ``n_planted`` old-prefix keys at seeded random positions are replaced
        by ``scale`` x the mean key norm along the direction of the first
        query head of the group at the first decode step.  The directions
        come from a dense dry run of that step in which each layer plants its
        keys just before its own attention, so a layer's query already
        reflects the planted keys of the layers below it (they change those
        layers' outputs, and so every later layer's queries).  Call after the
        prefill, before clustering."""
        B = last_token.shape[0]
        rs = np.random.RandomState(seed)
        planted = {}

        def plant(layer_id, q, c):
            pos = np.stack([[np.sort(rs.choice(self.sample_end, n_planted, replace=False))
                             for _ in range(self.num_kv_heads)] for _ in range(B)])
            for b in range(B):
                for kv in range(self.num_kv_heads):
                    qd = q[b, kv * self.group]
                    qhat = qd / qd.norm()
                    keys = (c.paged.tokens(b, kv, self.sample_end) if c.paged is not None
                            else c.key[b, kv, :self.sample_end])
                    norm = keys.float().norm(dim=-1).mean()
                    new = (scale * norm * qhat).to(keys.dtype)[None]
                    if c.paged is not None:
                        pages, slots = c.paged.slots(b, pos[b, kv])
                        c.paged.key_pool[pages, kv, slots] = new
                    else:
                        idx = torch.from_numpy(pos[b, kv]).to(keys.device)
                        c.key[b, kv, idx] = new
            planted[layer_id] = pos

        self._capture_q = {}
        self._plant_layer = plant
        try:
            self.model(last_token, position_ids=torch.full((B, 1), position, dtype=torch.long,
                                                           device=last_token.device),
                       use_cache=False, logits_to_keep=1)
        finally:
            self._capture_q = None
            self._plant_layer = None
        self._trim_cache(position)
        return planted

    def _check_planted(self, layer_id: int, q: torch.Tensor, cached, scale: float) -> None:
        """At the first sparse decode step: the selection of the first query
        head of every group, read out, must cover every planted position."""
        from .santapp import santa_decode_select
        summ = self.summaries[layer_id]
        sel, _, _ = santa_decode_select(q, *cached.kv(), summ,
                                        mode=self.config.mode, n_total=cached.length,
                                        sample_end=self.sample_end,
                                        topk_clusters=self._cfg("topk_clusters"),
                                        token_budget=self.config.samples_per_head,
                                        samples=self.config.samples_per_head, scale=scale,
                                        seed=self.config.sample_seed, step=0)
        pos = self._planted["positions"][layer_id]                  # [B, Hkv, n]
        B, Hkv, n = pos.shape
        positions = summ.positions.long()                           # [B, Hkv, N]
        p = torch.from_numpy(pos).to(positions.device)
        member_pos = torch.gather(positions, 2, p)                  # position in members
        # cluster row of a member position: the last start at or before it
        starts = summ.starts.long()
        G = starts.shape[2]
        valid = torch.arange(G, device=starts.device)[None, None] < summ.n_groups.long()[..., None]
        big = torch.where(valid, starts, torch.full_like(starts, 1 << 40))
        row = torch.searchsorted(big.contiguous(), member_pos.contiguous(), right=True) - 1
        heads = torch.arange(Hkv, device=sel.device) * self.group   # first head of each group
        sel_g = sel[:, heads]                                        # [B, Hkv, G]
        landed = torch.gather(sel_g.long(), 2, row)                  # [B, Hkv, n]
        self._planted["landed"] += int(landed.sum())
        self._planted["total"] += B * Hkv * n

    # ---- generation ------------------------------------------------------------
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, *, max_new_tokens: int,
                 eos_token_ids: set[int] | None = None, stop_on_eos: bool = False,
                 random_seed: int = 0, planted_keys: int = 0, plant_scale: float = 4.0,
                 plant_seed: int = 0) -> SantaGeneration:
        """santapp.py:794-908: prefill, clustering, then greedy decoding of
        ``max_new_tokens`` tokens.  ``planted_keys`` > 0 adds the synthetic
        retrieval check (``_plant_keys``): the metrics then report how many
        planted positions the first decode step's selections covered."""
        if input_ids.ndim != 2:
            raise ValueError("input_ids must be [batch, T]")
        B, T = input_ids.shape
        if T < 2:
            raise ValueError("SANTA++ requires at least two prompt tokens.")
        self.clear()
        self.cache_capacity = T + max_new_tokens
        t0 = time.perf_counter()
        with self.patched():
            self._log(f"prefill of {B} x {T} tokens")
            prefill_s, sample_end = self._prefill(input_ids, probe_seed=random_seed)
            self._log(f"prefill done in {prefill_s:.2f} s")
            self._trim_cache(T - 1)
            plant_s = 0.0
            if planted_keys > 0:
                tp = time.perf_counter()
                pos = self._plant_keys(input_ids[:, -1:], T - 1, n_planted=planted_keys,
                                       scale=plant_scale, seed=plant_seed)
                self._planted = {"positions": pos, "landed": 0, "total": 0}
                torch.cuda.synchronize()
                plant_s = time.perf_counter() - tp
            self._log("clustering")
            cluster_s, n_clusters = self._cluster()
            self._log(f"clustering done in {cluster_s:.2f} s")
            self.mode = self.config.mode
            self.traffic = DecodeTrafficTracker()
            generated = [[] for _ in range(B)]
            current = input_ids[:, -1:]
            position = T - 1
            done = torch.zeros(B, dtype=torch.bool, device=input_ids.device)
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            for step in range(max_new_tokens):
                if step % 64 == 0:
                    self._log(f"decode step {step}")
                self._decode_step = step
                out = self.model(current, position_ids=torch.full(
                    (B, 1), position, dtype=torch.long, device=input_ids.device),
                    use_cache=False, logits_to_keep=1)
                current = out.logits[:, -1].argmax(dim=-1, keepdim=True)
                ids = current[:, 0].tolist()
                for b in range(B):
                    generated[b].append(int(ids[b]))
                position += 1
                if stop_on_eos and eos_token_ids:
                    done |= torch.tensor([i in eos_token_ids for i in ids], device=done.device)
                    if bool(done.all()):
                        break
            torch.cuda.synchronize()
            decode_s = time.perf_counter() - t2
            self._flush_traffic()
        metrics = {
            "backend": "santapp_b200", "mode": self.config.mode, "batch": B,
            "prompt_tokens": T, "generated_tokens": len(generated[0]),
            "prefill_seconds": prefill_s, "clustering_seconds": cluster_s,
            "decode_seconds": decode_s, "total_seconds": time.perf_counter() - t0,
            "sampled_prefix_tokens": sample_end, "nominal_clusters_per_kv_head": n_clusters,
            "planted_check": (None if self._planted is None else {
                "planted_per_layer_sequence_kv_head": planted_keys,
                "landed": self._planted["landed"], "total": self._planted["total"],
                "all_landed": self._planted["landed"] == self._planted["total"],
                "scale": plant_scale, "dry_run_seconds": plant_s}),
            **self.traffic.as_dict(),
        }
        self.clear()
        return SantaGeneration(token_ids=generated[0] if B == 1 else generated, metrics=metrics)

    def _flush_traffic(self) -> None:
        """Feed the decode calls' draw counts to the traffic tracker (one
        device->host read for the whole generation)."""
        if not self._traffic_pending:
            return
        n_exact = torch.stack([t[2] for t in self._traffic_pending]).cpu().numpy()
        ess = torch.stack([t[3] for t in self._traffic_pending]).cpu().numpy()
        groups = {k: v.cpu().numpy() for k, v in self._n_groups_host.items()}
        for i, (n_total, layer_id, _, _) in enumerate(self._traffic_pending):
            self.traffic.record_step(
                mode=self.config.mode, n_total=n_total, sample_end=self.sample_end,
                n_exact=n_exact[i], samples=self.config.samples_per_head,
                n_groups=groups[layer_id], ess=ess[i])
        self._traffic_pending = []

    # ---- the reference's per-head call ----------------------------------------
    def _approximate_attention(self, query: torch.Tensor, full_key: torch.Tensor,
                               full_value: torch.Tensor, layer_id: int,
                               kv_head: int) -> torch.Tensor:
        """santapp.py:365-506 for one query head of sequence 0: query [D],
        full_key / full_value [n_total, D] (the layer's cache of that KV
        head), in ``self.mode``.  Returns the fp32 attention output [D] and
        records the call's draw counts.  Each call draws from its own Philox
        stream (seed, layer, KV head and a per-engine call counter), as the
        reference's per-head torch draws are independent."""
        n_total = int(full_key.shape[0])
        if not 0 < self.sample_end <= n_total:
            raise RuntimeError(
                f"Invalid sampled-prefix boundary {self.sample_end} for cache length {n_total}.")
        D = self.head_dim
        q = query.detach().float().reshape(1, 1, D).contiguous()
        kc = full_key.contiguous().view(1, 1, n_total, D)
        vc = full_value.contiguous().view(1, 1, n_total, D)
        summary = self.summaries[layer_id].segment(0, kv_head)
        mode = self.mode if self.mode != "dense" else self.config.mode
        seed = (int(self.config.sample_seed) + 0x9E3779B97F4A7C15 * (layer_id * 4096 + kv_head + 1)
                ) & 0xFFFFFFFFFFFFFFFF
        res = santa_decode(q, kc, vc, summary, mode=mode, n_total=n_total,
                           sample_end=self.sample_end, topk_clusters=self._cfg("topk_clusters"),
                           token_budget=self.config.samples_per_head,
                           samples=self.config.samples_per_head, scale=1.0 / math.sqrt(D),
                           seed=seed, step=self._head_calls, with_stats=True)
        self._head_calls += 1
        self.traffic.record_step(
            mode=mode, n_total=n_total, sample_end=self.sample_end,
            n_exact=res.n_exact.cpu().numpy(), samples=self.config.samples_per_head,
            n_groups=summary.n_groups.cpu().numpy(), ess=res.ess.cpu().numpy())
        return res.out.view(D)
