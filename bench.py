#!/usr/bin/env python
"""SANTA++ sparse decode attention throughput on B200.

One step = one decode step of SANTA++ attention for every (sequence, query
head) of the batch: cluster selection (q . centroid scoring, top-k) plus the
gather attention over the selected clusters, the uniformly sampled remainder
and the exact recent window.  Default workload: the Qwen3-8B attention shape
(32 query heads, 8 KV heads, head_dim 128), bf16 K/V, batch 16 at 128K
context, 1024 centroids per KV head, top-32 clusters + 512 samples per head.
On N GPUs (torchrun) the same job is split into N sequence shards (strong
scaling).  The single-GPU line also carries the Qwen2.5-7B batch-8 32K decode
and the Qwen2.5-7B 32K prefill (against torch SDPA in the same run).  Data:
seeded synthetic Gaussian-mixture keys.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the torch-CPU
restatement of the reference's per-head decode on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "opus-lab-notebooks_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from santapp_b200.synthetic import QWEN3_8B_128K, QWEN7B_32K, make_decode_workload  # noqa: E402

WORKLOADS = {"qwen7b-32k": QWEN7B_32K, "qwen3-8b-128k": QWEN3_8B_128K,
             "qwen7b-prefill-32k": None, "qwen7b-model-64k": None}
MODEL_METRIC = ("Qwen2.5-7B decode tokens/s with SANTA++ attention in all 28 layers "
                "(random init), 64K context; planted-key retrieval check")
PREFILL_METRIC = "causal prefill attention TFLOP/s (tcgen05) and MiniBatchKMeans seconds per fit"
METRIC = "SANTA++ decode attn tokens/s @32K-128K ctx; achieved HBM GB/s vs 8 TB/s peak"
L2_FLUSH_BYTES = 256 << 20
HEAD_START_S = 0.05  # device spin before the eager multi-GPU timed steps


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="qwen3-8b-128k",
                    help="qwen7b-prefill-32k: prompt prefill + clustering of the Qwen2.5-7B "
                         "shape (one GPU), not a decode step; qwen7b-model-64k: the whole "
                         "random-init Qwen2.5-7B model through the engine (one GPU)")
    ap.add_argument("--model-context", type=int, default=65536,
                    help="prompt length of the model workload (65536 reported; smaller for "
                         "quick checks)")
    ap.add_argument("--model-layers", type=int, default=28)
    ap.add_argument("--kv-page-size", type=int, default=None,
                    help="model workload: every layer's KV cache in pages of this many tokens "
                         "(SantaB200Config.kv_page_size)")
    ap.add_argument("--mode", default="hybrid")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="skip the host-side extras (byte accounting, e2e, CPU baseline)")
    ap.add_argument("--prefill-prompt", type=int, default=32768,
                    help="prompt length of the prefill workload (the reported one is 32768; "
                         "smaller values are for profiler captures)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU instead of the workload's own (small profiler "
                         "captures; the reported runs use the workload's batch)")
    ap.add_argument("--rank-share", type=int, default=1,
                    help="one GPU runs the share of the job one of N sequence-shard ranks holds "
                         "(1/N of the tokens, clusters, top-k clusters and samples), without the "
                         "exchange: the per-rank cost behind the N-GPU curve")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="bound on the CPU-baseline sample")
    ap.add_argument("--transport", choices=["nccl", "p2p"], default="p2p",
                    help="N > 1: the kernels' own peer-memory exchange, or NCCL all-gathers")
    ap.add_argument("--no-extras", action="store_true",
                    help="single GPU: skip the 32K decode and prefill blocks")
    return ap.parse_args()


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every millisecond
    while the timed region runs (nvidia-smi's 200 ms polling is too coarse
    for a sub-second region)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period_s: float = 0.001):
        import threading
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], 0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self.max_mhz = None
        self.ok = False

    def _run(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(visible.split(",")[self.index]) if visible else self.index
            h = nv.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.ok = True
            while not self._stop.is_set():
                self.samples.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(h))
                time.sleep(self.period)
            nv.nvmlShutdown()
        except Exception as e:  # NVML missing: report it rather than guess
            self.error = repr(e)

    def start(self):
        self._thread.start()
        t0 = time.time()
        while not self.ok and self._thread.is_alive() and time.time() - t0 < 5:
            time.sleep(0.001)

    def stop(self) -> dict:
        self._stop.set()
        self._thread.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz,
                    "reasons": [getattr(self, "error", "no samples")], "samples": 0}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for b, n in self.REASONS.items() if self.reasons & b),
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

class L2Flush:
    """Evicts L2 (126 MB) between timed steps: a write of one buffer larger
    than L2, then a read of a second one.  The read pushes the dirty lines
    of the write back to HBM before the step starts, so the step pays for
    no write-back of flush data."""

    def __init__(self, device):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.r = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)
        self.out = torch.empty((), dtype=torch.int32, device=device)

    def __call__(self):
        self.w.zero_()
        torch.amax(self.r, dim=0, out=self.out)


def algorithmic_bytes(runner, q, step, shape, summ, cid):
    """Bytes the two decode kernels must move for this step.

    attend: distinct K and V rows touched = the union of the GQA group's
    selected clusters + the exact recent window + distinct sampled rows outside
    that union, per (sequence, KV head).  select: centroids and cluster
    metadata of every (sequence, KV head)."""
    from santapp_b200.attention import santapp as S
    sel, rows, _ = S.santa_decode_select(
        q, *runner.kv_args, summ, mode=runner.mode,
        n_total=shape.context, topk_clusters=shape.topk_clusters, samples=shape.samples,
        seed=runner.p.seed, step=step)
    B, Hq, G = sel.shape
    g, N = shape.group, shape.sample_end
    BH = B * (Hq // g)
    union = sel.view(BH, g, G).amax(dim=1).bool()                      # [BH, G]
    covered = torch.gather(union, 1, cid)                               # [BH, N]
    srows = rows.reshape(BH, -1).long()
    sampled = torch.zeros(BH, N + 1, dtype=torch.bool, device=q.device)
    sampled.scatter_(1, torch.where(srows >= 0, srows, N), True)
    extra = int((sampled[:, :N] & ~covered).sum())
    rows_touched = int(covered.sum()) + extra + BH * (shape.context - shape.sample_end)
    esize = 2 if shape.kv_dtype == torch.bfloat16 else 4
    attend = rows_touched * 2 * shape.head_dim * esize
    select = BH * shape.n_clusters * (shape.head_dim * 4 + 12) + q.numel() * 4
    return attend, select, rows_touched


def cluster_of_row(summ, shape):
    """[BH, N] cluster row of every position of the cluster-sorted prefix."""
    BH = summ.n_groups.numel()
    N, G = shape.sample_end, summ.max_groups
    starts = summ.starts.view(BH, G).long()
    active = torch.arange(G, device=starts.device)[None, :] < summ.n_groups.view(BH, 1)
    marks = torch.zeros(BH, N + 1, dtype=torch.long, device=starts.device)
    marks.scatter_add_(1, torch.where(active, starts, N), active.long())
    return (torch.cumsum(marks[:, :N], dim=1) - 1).clamp_min_(0)


def measure_decode(args, shape, steps, warmup, dev, keep=False, page_size=None):
    """The K timed decode steps of one workload on one GPU: device time per
    step, the select / attend split, and the attend kernel's roofline from
    the algorithmic bytes of every timed step.  keep: also return the
    workload, summary and step object (for the e2e run).  page_size: the
    cache moved into page pools (pages in a seeded random order) first."""
    from santapp_b200.attention import santapp as S
    from santapp_b200.attention.paged import PagedKVCache
    from santapp_b200.synthetic import scaled_shape
    n_q = max(shape.steps, steps + warmup)
    w = make_decode_workload(scaled_shape(shape, steps=n_q), seed=args.seed, device=dev)
    kc, vc = w.keys, w.values
    if page_size:
        kc = PagedKVCache.from_contiguous(w.keys, w.values, length=shape.context,
                                          page_size=page_size, page_order_seed=args.seed)
        vc = None
        w.keys = w.values = None
        torch.cuda.empty_cache()
    labels = w.labels[:, :, :shape.sample_end].contiguous()
    summ = S.build_summary(kc, vc, labels, shape.n_clusters,
                           sample_end=shape.sample_end, n_total=shape.context)
    del labels
    w.labels = None
    runner = S.DecodeStep(kc, vc, summ, num_query_heads=shape.num_query_heads,
                          mode=args.mode, n_total=shape.context,
                          topk_clusters=shape.topk_clusters, samples=shape.samples,
                          seed=args.seed)
    queries = w.queries
    flush = L2Flush(dev)
    torch.cuda.synchronize()

    # algorithmic bytes of every timed step (selection read back, outside timing)
    attend_bytes, select_bytes, rows_touched = [], [], []
    if not args.profile:
        cid = cluster_of_row(summ, shape)
        for i in range(steps):
            step = warmup + i
            a_b, s_b, r_t = algorithmic_bytes(runner, queries[step], step, shape, summ, cid)
            attend_bytes.append(a_b)
            select_bytes.append(s_b)
            rows_touched.append(r_t)
        del cid
    torch.cuda.synchronize()

    for i in range(warmup):
        flush()
        runner(queries[i], step=i)
    torch.cuda.synchronize()

    # The K timed steps as one CUDA graph, the way a decode loop is captured
    # for serving: per step the L2 flush, then the selection and attention
    # kernels, timed on the device by event-record nodes around the two
    # kernels (the flush lies outside them).  Nothing sits between the two
    # kernels, as in a serving loop.  A second graph of the same steps
    # records one more event between the kernels: the phase split and the
    # attention kernel's roofline come from it.
    def capture(split):
        ev = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
              for _ in range(steps)]
        cap = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                for i in range(steps):
                    step = warmup + i
                    flush()
                    ev[i][0].record(cap)
                    runner.plan(queries[step], step=step)
                    if split:
                        ev[i][1].record(cap)
                    runner.execute()
                    ev[i][2].record(cap)
        torch.cuda.synchronize()
        return graph, ev

    graph, inner = capture(False)
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    graph.replay()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    del graph
    step_ms = np.array([e[0].elapsed_time(e[2]) for e in inner])
    graph, split = capture(True)
    graph.replay()
    torch.cuda.synchronize()
    del graph
    split_step_ms = np.array([e[0].elapsed_time(e[2]) for e in split])
    plan_ms = np.array([e[0].elapsed_time(e[1]) for e in split])
    att_ms = np.array([e[1].elapsed_time(e[2]) for e in split])
    peak, peak_kind = peaks()
    achieved = (float(np.sum(attend_bytes) / (att_ms.sum() / 1e3) / 1e9) if attend_bytes
                else float("nan"))
    step_bytes = (np.array(attend_bytes) + np.array(select_bytes)) if attend_bytes else None
    res = {
        "value": shape.batch * steps / (step_ms.sum() / 1e3),
        "ms_per_step": float(step_ms.mean()),
        "phase_ms": {"select": float(plan_ms.mean()), "attend": float(att_ms.mean()),
                     "step_with_split_event": float(split_step_ms.mean())},
        "roofline": {
            "kernel": "decode_attend_gather_kernel",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": load_traffic(shape),
            "algorithmic_bytes_per_launch": float(np.mean(attend_bytes)) if attend_bytes else None,
            "rows_touched_per_step": float(np.mean(rows_touched)) if rows_touched else None,
            "dense_kv_bytes_per_step": float(shape.batch * shape.num_kv_heads * shape.context
                                             * shape.head_dim * 2 * 2),
        },
        "select_roofline": {
            "achieved": (float(np.sum(select_bytes) / (plan_ms.sum() / 1e3) / 1e9)
                         if select_bytes else None),
            "unit": "GB/s",
        },
        "step_roofline": {
            "note": "both kernels: attend + select algorithmic bytes over the whole step time",
            "achieved": (float(step_bytes.sum() / (step_ms.sum() / 1e3) / 1e9)
                         if step_bytes is not None else None),
            "frac": (float(step_bytes.sum() / (step_ms.sum() / 1e3) / 1e9) / peak
                     if step_bytes is not None else None),
            "unit": "GB/s",
        },
        "wall_s": wall,
        "clocks": clk,
        "gpu_launches": runner.kernels_per_call * steps,
    }
    if keep:
        return res, (w, summ, runner)
    del runner, summ, w, kc, vc
    torch.cuda.empty_cache()
    return res


def decode_config(shape, mode, world, p=None, p2p=True):
    """The config block of a decode line (our arm and the reference arm
    print the same one for the same run)."""
    cfg = {
        "workload": shape.name,
        "query_heads": shape.num_query_heads, "kv_heads": shape.num_kv_heads,
        "head_dim": shape.head_dim, "batch": shape.batch, "context": shape.context,
        "clusters": shape.n_clusters, "topk_clusters": shape.topk_clusters,
        "samples": shape.samples, "recent_window": shape.recent_window, "mode": mode,
    }
    if world == 1:
        cfg["parallelism"] = "single GPU"
        cfg["l2"] = (f"flushed before every step, outside the events: {L2_FLUSH_BYTES >> 20} MiB "
                     f"write, then a {L2_FLUSH_BYTES >> 20} MiB read of another buffer so that "
                     "no dirty flush line is written back inside the step")
    else:
        cfg["parallelism"] = (f"sequence shards x{world}: the job's cache, clusters and sample "
                              "budget split over the ranks; "
                              + ("top-k keys and (m, l, o) partials stored by the kernels into "
                                 "every rank's buffer over NVLink (2 launches per step)"
                                 if p2p else "NCCL all-gathers of the top-k keys and of the "
                                             "(m, l, o) partials"))
        cfg["l2"] = ("flushed before every step outside the events (256 MiB write + 256 MiB "
                     "read of another buffer)")
    return cfg


def run_ours(args, rank, world):
    from santapp_b200.synthetic import scaled_shape
    shape = WORKLOADS[args.workload]
    if world > 1:
        raise SystemExit("multi-GPU decode runs in run_sharded (sequence shards)")
    if args.batch is not None:
        shape = scaled_shape(shape, batch=args.batch,
                             name=shape.name.rsplit("-b", 1)[0] + f"-b{args.batch}")
    if args.rank_share > 1:
        n = args.rank_share
        shape = scaled_shape(shape, name=f"{shape.name}-rank-share-1of{n}",
                             context=shape.context // n,
                             true_clusters=max(1, shape.true_clusters // n),
                             n_clusters=max(1, shape.n_clusters // n),
                             topk_clusters=max(1, shape.topk_clusters // n),
                             samples=max(1, shape.samples // n))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res, (w, summ, runner) = measure_decode(args, shape, args.steps, args.warmup, dev, keep=True)
    e2e = None if (args.no_e2e or args.profile) else run_e2e(args, shape, w, summ, runner)
    del runner, summ, w
    torch.cuda.empty_cache()
    line = {
        "metric": METRIC,
        "value": res["value"],
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16" if shape.kv_dtype == torch.bfloat16 else "f32",
        "data": "synthetic (seeded Gaussian-mixture keys, N(0,1) values and queries)",
        "config": decode_config(shape, args.mode, 1),
        "phase_ms": res["phase_ms"],
        "roofline": res["roofline"],
        "select_roofline": res["select_roofline"],
        "step_roofline": res["step_roofline"],
        "timing": ("one CUDA graph holding the K timed steps (per step: L2 flush, selection, "
                   "attention); each step timed by event-record nodes around its two kernels; "
                   "the phase split and roofline from a second graph of the same steps with "
                   "one more event between the kernels"),
        "wall_s": res["wall_s"],
        "clocks": res["clocks"],
        "gpu_launches": res["gpu_launches"],
        "e2e": e2e,
        "cpu_baseline": None,
    }
    if not args.no_extras and not args.profile and args.workload == "qwen3-8b-128k":
        # the other decode context of the metric (Qwen2.5-7B batch 8 at 32K),
        # and the prefill of that layer, next to torch SDPA in the same run
        steps32 = min(args.steps, 64)
        r32 = measure_decode(args, QWEN7B_32K, steps32, args.warmup, dev)
        line["ctx32768"] = {
            "workload": QWEN7B_32K.name, "steps": steps32, "value": r32["value"],
            "unit": "tokens/s", "ms_per_step": r32["ms_per_step"], "phase_ms": r32["phase_ms"],
            "roofline": r32["roofline"], "select_roofline": r32["select_roofline"],
            "step_roofline": r32["step_roofline"], "clocks": r32["clocks"],
            "gpu_launches": r32["gpu_launches"], "config": decode_config(QWEN7B_32K, args.mode, 1)}
        # the headline workload again with the cache in 256-token pages
        # scattered over the pool (block-table reads in every kernel)
        rp = measure_decode(args, shape, args.steps, args.warmup, dev, page_size=256)
        line["paged"] = {
            "workload": shape.name, "page_size": 256, "steps": args.steps,
            "value": rp["value"], "unit": "tokens/s", "ms_per_step": rp["ms_per_step"],
            "phase_ms": rp["phase_ms"], "roofline": rp["roofline"],
            "step_roofline": rp["step_roofline"], "clocks": rp["clocks"],
            "gpu_launches": rp["gpu_launches"]}
        line["prefill"] = prefill_block(args, dev, 32768, steps=min(args.steps, 10))
    if not (args.no_cpu_baseline or args.profile):
        line["cpu_baseline"] = cpu_baseline_sample(args, shape)
    return line


def load_traffic(shape):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of
    the attend kernel, from the committed ncu summary of this workload (its
    line ``dram_bytes_per_launch: N``)."""
    import re
    path = os.path.join(REPO, "profiles", f"decode_attend_gather_{shape.name}.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"^dram_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read(), re.M)
    return float(m.group(1)) if m else None


def run_e2e(args, shape, w, summ, runner):
    """Through the public decode API with host buffers, the way a serving
    loop calls it, synchronised every step: the step's queries copied
    host->device from pinned memory, DecodeStep (santa_decode_plan +
    santa_decode_execute, C ABI), the output copied into pinned host memory.
    The graph-captured form (GraphedDecodeStep: the step's queries copied on
    the host into the pinned staging buffer, then one graph launch holding
    the transfers, the selection and the attention) is timed beside it."""
    from santapp_b200.attention import santapp as S
    steps = args.steps
    q_all = w.queries[:steps].cpu()                     # the steps' queries on the host
    q_host = torch.empty(tuple(q_all.shape[1:]), dtype=torch.float32).pin_memory()
    out_host = torch.empty(shape.batch, shape.num_query_heads, shape.head_dim).pin_memory()
    step_api = S.DecodeStep(w.keys, w.values, summ, num_query_heads=shape.num_query_heads,
                            mode=args.mode, n_total=shape.context,
                            topk_clusters=shape.topk_clusters, samples=shape.samples,
                            seed=args.seed)
    graphed = step_api.graphed(q_host, out_host)
    stream = torch.cuda.current_stream()
    for i in range(2):
        q_host.copy_(q_all[i])
        graphed.run(i)
        stream.synchronize()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        q_host.copy_(q_all[i])
        graphed.run(i)
        stream.synchronize()
    dt = time.perf_counter() - t0
    # the per-call form: torch copies around two C ABI calls
    q_pin = q_all.pin_memory()
    q_dev = torch.empty_like(w.queries[0])
    for i in range(2):
        q_dev.copy_(q_pin[i], non_blocking=True)
        out_host.copy_(step_api(q_dev, step=i), non_blocking=True)
        stream.synchronize()
    t1 = time.perf_counter()
    for i in range(steps):
        q_dev.copy_(q_pin[i], non_blocking=True)
        out_host.copy_(step_api(q_dev, step=i), non_blocking=True)
        stream.synchronize()
    dt_calls = time.perf_counter() - t1
    del graphed
    return {"value": shape.batch * steps / dt_calls, "unit": "tokens/s",
            "h2d_bytes_per_step": int(q_host.numel() * 4),
            "d2h_bytes_per_step": int(out_host.numel() * 4),
            "api": "santapp_b200.attention.DecodeStep (torch copies from / to pinned memory "
                   "around santa_decode_plan + santa_decode_execute, C ABI)",
            "graphed_api": {"value": shape.batch * steps / dt, "unit": "tokens/s",
                            "h2d_bytes_per_step": int(q_host.numel() * 4) + 8,
                            "api": "santapp_b200.attention.GraphedDecodeStep.run (host copy "
                                   "into the pinned staging buffer, one graph launch with "
                                   "the transfers, the selection and the attention)"}}


def _port_sample(shape, seed, n_seq=1):
    """A bounded CPU sample of the workload for the torch-CPU restatement:
    the first n_seq sequences' caches (drawn on the host with the workload's
    generator and shape) and their cluster summaries."""
    from oracle import santa_torch_port as P
    from santapp_b200.synthetic import scaled_shape
    sh = scaled_shape(shape, batch=n_seq, steps=max(shape.steps, 64))
    w = make_decode_workload(sh, seed=seed, device="cpu")
    summ = {}
    for b in range(n_seq):
        for kv in range(shape.num_kv_heads):
            summ[(b, kv)] = P.build_summary(w.keys[b, kv, :shape.sample_end].float(),
                                            w.labels[b, kv, :shape.sample_end], shape.n_clusters)
    return w, summ


def _port_step(shape, w, summ, step, gen, n_seq=1):
    """One decode step of the sample's sequences, one call per (sequence,
    query head) as the reference's engine makes them."""
    from oracle import santa_torch_port as P
    for b in range(n_seq):
        for h in range(shape.num_query_heads):
            kv = h // shape.group
            P.approximate_attention_hybrid(w.queries[step, b, h], w.keys[b, kv], w.values[b, kv],
                                           summ[(b, kv)], shape.sample_end,
                                           shape.topk_clusters, shape.samples, generator=gen)


def cpu_baseline_sample(args, shape):
    """The torch-CPU restatement of the reference's per-head decode, timed on
    all host cores (torch intra-op threads, as the reference runs) over a
    bounded sample: decode steps of sequence 0 until ~args.cpu_seconds have
    passed; tokens/s = sequences decoded per second."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    w, summ = _port_sample(shape, args.seed)
    gen = torch.Generator().manual_seed(args.seed)
    _port_step(shape, w, summ, 0, gen)  # warm-up
    steps = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < args.cpu_seconds and steps < 63:
        _port_step(shape, w, summ, 1 + steps, gen)
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{steps} decode steps of sequence 0 ({steps * shape.num_query_heads} "
                      f"query-head calls over {shape.num_kv_heads} KV heads x {shape.context} "
                      "tokens), torch-CPU restatement of the reference's per-head "
                      "_approximate_attention (oracle/santa_torch_port.py), "
                      f"torch.set_num_threads({cores})"}


# ---------------------------------------------------------------------------
# prefill + clustering of one layer (Qwen2.5-7B shape, 32K prompt)
# ---------------------------------------------------------------------------

def prefill_block(args, dev, T, steps, kv_heads_fit=1):
    """Causal prefill attention of one Qwen2.5-7B layer, [1, 28, T, 128] bf16
    with 4 KV heads: santa_prefill (tcgen05) and torch SDPA (the library
    path the reference's prefill calls, santapp.py:320-346; flash / cuDNN
    as the wheel picks) timed the same way in the same run, the outputs
    compared; then MiniBatchKMeans of KV heads' 32K-token prefixes (k=256,
    minibatch 4096, 20 iterations, seed 0) through
    SklearnLikeTorchMiniBatchKMeans.  Seeded N(0,1) queries and values, the
    Gaussian-mixture keys of the decode workloads."""
    import torch.nn.functional as F
    from santapp_b200.attention.kmeans import SklearnLikeTorchMiniBatchKMeans
    from santapp_b200.attention.prefill import santa_prefill
    from santapp_b200.synthetic import scaled_shape
    B, Hq, Hkv, D = 1, 28, 4, 128
    shape = scaled_shape(QWEN7B_32K, batch=1, steps=1, context=T)
    w = make_decode_workload(shape, seed=args.seed, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    q = torch.randn(B, Hq, T, D, device=dev, generator=g).to(torch.bfloat16)
    k, v = w.keys, w.values
    flops = 4.0 * Hq * D * T * (T + 1) / 2
    out = santa_prefill(q, k, v)
    flush = L2Flush(dev)

    def timed(fn):
        ts = []
        for i in range(args.warmup + steps):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(e0.elapsed_time(e1))
        return float(np.mean(ts))

    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    ms = timed(lambda: santa_prefill(q, k, v, out=out))
    clk = clocks.stop()
    err = int(out._santa_error_flag.item())
    sdpa_out = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    ms_sdpa = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True,
                                                           enable_gqa=True))
    diff = (out.float() - sdpa_out.float()).abs()
    cmp = {"max_abs": float(diff.max()), "mean_abs": float(diff.mean())}
    del sdpa_out, diff
    peaks_d = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) \
        if os.path.exists(os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks_d.get("bf16_tflops", 1590.0))
    tflops = flops / (ms / 1e3) / 1e12
    # clustering: one fit per KV head, each timed with a host clock around the
    # call (the fit reads back one value per mini-batch, as the reference's
    # control flow needs)
    fits = []
    # one untimed fit first (first-call set-up: launch attributes, occupancy queries)
    SklearnLikeTorchMiniBatchKMeans(256, batch_size=4096, max_iter=20, random_state=0
                                    ).fit_predict(k[0, 0, :shape.sample_end].float())
    for kv in range(kv_heads_fit):
        x = k[0, kv, :shape.sample_end].float()
        est = SklearnLikeTorchMiniBatchKMeans(256, batch_size=4096, max_iter=20, random_state=0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        est.fit_predict(x)
        torch.cuda.synchronize()
        fits.append((time.perf_counter() - t0, est.n_steps_))
    return {
        "workload": f"qwen2.5-7b-prefill-ctx{T}", "query_heads": Hq, "kv_heads": Hkv,
        "head_dim": D, "batch": B, "prompt": T, "causal": True, "steps": steps,
        "ms": ms, "tflops": tflops,
        "roofline": {"kernel": "prefill_fwd_kernel", "bound": "tensor", "achieved": tflops,
                     "peak": peak, "peak_kind": "measured (burst)" if peaks_d else "fallback",
                     "unit": "TFLOP/s", "frac": tflops / peak, "algorithmic_flops": flops},
        "torch_sdpa_ms": ms_sdpa, "torch_sdpa_tflops": flops / (ms_sdpa / 1e3) / 1e12,
        "vs_torch_sdpa": ms_sdpa / ms,
        "vs_torch_sdpa_outputs": cmp,
        "error_flag": err,
        "clocks": clk,
        "kmeans": {"k": 256, "batch_size": 4096, "max_iter": 20, "rows": shape.sample_end,
                   "features": D, "seconds_per_fit": [round(f[0], 4) for f in fits],
                   "steps_per_fit": [int(f[1]) for f in fits]},
    }


def run_prefill(args):
    """--workload qwen7b-prefill-32k: the prefill block as its own line."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    blk = prefill_block(args, dev, args.prefill_prompt, args.steps, kv_heads_fit=4)
    return {
        "metric": PREFILL_METRIC, "value": blk["tflops"], "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": blk["ms"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) queries, Gaussian-mixture keys, N(0,1) values)",
        "config": {"workload": blk["workload"], "query_heads": blk["query_heads"],
                   "kv_heads": blk["kv_heads"], "head_dim": blk["head_dim"], "batch": 1,
                   "prompt": blk["prompt"], "causal": True, "kmeans": blk["kmeans"]},
        "roofline": blk["roofline"], "torch_sdpa_ms": blk["torch_sdpa_ms"],
        "vs_torch_sdpa": blk["vs_torch_sdpa"], "vs_torch_sdpa_outputs": blk["vs_torch_sdpa_outputs"],
        "error_flag": blk["error_flag"], "clocks": blk["clocks"],
        "gpu_launches": 2 * (args.steps + args.warmup),
    }


# ---------------------------------------------------------------------------
# the whole model: random-init Qwen2.5-7B through the engine
# ---------------------------------------------------------------------------

def qwen7b_model(layers, device, seed=0):
    """Random-init Qwen2.5-7B (hidden 3584, 28 query / 4 KV heads, head_dim
    128, SwiGLU FFN 18944, RMSNorm, RoPE theta 1e6, vocab 152064), bf16;
    initialised as the model's own initialiser does it (initializer_range
    0.02): weight matrices and embeddings ~ N(0, 0.02), biases 0, RMSNorm
    gains 1."""
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(hidden_size=3584, intermediate_size=18944, num_hidden_layers=layers,
                      num_attention_heads=28, num_key_value_heads=4, vocab_size=152064,
                      max_position_embeddings=131072, rope_theta=1e6, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, torch_dtype=torch.bfloat16)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        m = Qwen2ForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, (torch.nn.Linear, torch.nn.Embedding)):
                mod.weight.normal_(0.0, 0.02, generator=g)
                if getattr(mod, "bias", None) is not None:
                    mod.bias.zero_()
            elif hasattr(mod, "variance_epsilon"):  # Qwen2RMSNorm
                mod.weight.fill_(1.0)
    return m


def run_model(args):
    """The model-level workload: random-init Qwen2.5-7B, batch 4 at a 64K
    prompt of uniform random tokens (seed 0), SANTA++ hybrid attention
    (top-16 clusters + 256 samples, k=512 clusters per (layer, KV head,
    sequence)) in every layer through SantaB200Engine.generate: prefill
    (tcgen05 attention), fingerprints + MiniBatchKMeans + summaries, then
    greedy decoding of ``--steps`` tokens (256 reported).  16 keys per
    (layer, sequence, KV head) are planted along the first decode step's
    query direction and the check reports how many land in the selections.
    Decode tokens/s = batch x steps / decode seconds (host clock around the
    synchronised loop)."""
    import faulthandler
    from santapp_b200.attention.engine import KMeansConfig, SantaB200Config, SantaB200Engine
    # a stuck phase shows up as periodic stack dumps on stderr
    faulthandler.dump_traceback_later(300, repeat=True, file=sys.stderr)
    t_start = time.perf_counter()

    def log(msg):
        print(f"[model {time.perf_counter() - t_start:8.1f} s] {msg}", file=sys.stderr, flush=True)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, T = 4, args.model_context
    log("building the random-init model")
    model = qwen7b_model(args.model_layers, dev, seed=args.seed)
    log(f"model ready ({sum(p.numel() for p in model.parameters()) / 1e9:.2f} B parameters)")
    g = torch.Generator(device="cpu").manual_seed(args.seed)
    ids = torch.randint(0, 152064, (B, T), generator=g).to(dev)
    cfg = SantaB200Config(mode="hybrid", samples_per_head=256, topk_clusters=16, n_clusters=512,
                          recent_window=64, probe_queries=64, sample_seed=args.seed,
                          kmeans=KMeansConfig(), kv_page_size=args.kv_page_size)
    eng = SantaB200Engine(model, cfg)
    eng.log = log
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    gen = eng.generate(ids, max_new_tokens=args.steps, planted_keys=16, plant_scale=4.0,
                       plant_seed=args.seed)
    clk = clocks.stop()
    faulthandler.cancel_dump_traceback_later()
    log("done")
    m = gen.metrics
    value = B * m["generated_tokens"] / m["decode_seconds"]
    return {
        "metric": MODEL_METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": 0, "ms_per_step": m["decode_seconds"] / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights: matrices N(0, 0.02), norm gains 1, biases 0; "
                "uniform random prompt tokens)",
        "config": {"workload": f"qwen2.5-7b-model-ctx{T}-b{B}", "layers": args.model_layers,
                   "kv_cache": (f"paged, {args.kv_page_size}-token pages" if args.kv_page_size
                                else "contiguous"),
                   "hidden": 3584, "query_heads": 28, "kv_heads": 4, "head_dim": 128,
                   "ffn": 18944, "vocab": 152064, "batch": B, "context": T, "clusters": 512,
                   "topk_clusters": 16, "samples": 256, "mode": "hybrid"},
        "timing": "host clock around each synchronised phase of SantaB200Engine.generate",
        "phases_s": {"prefill": m["prefill_seconds"], "clustering": m["clustering_seconds"],
                     "decode": m["decode_seconds"], "total": m["total_seconds"]},
        "planted_check": m["planted_check"],
        "traffic": {k: v for k, v in m.items() if k.startswith("decode_") or k.startswith("mean_")},
        "clocks": clk,
        "generated_first_tokens": gen.token_ids[0][:8],
    }


# ---------------------------------------------------------------------------
# our arm on N GPUs: sequence shards
# ---------------------------------------------------------------------------

def run_sharded(args, rank, world):
    """Strong scaling over sequence shards: the workload's whole job (the
    Qwen3-8B batch-16 128K decode by default) is split over the N ranks,
    every sequence's clustered prefix into N contiguous shards, the
    mixture's clusters and the sample budget likewise.  Peer-memory exchange
    (default): one step = the selection launch (local candidates, key
    exchange, global top-k threshold, draws) and the attention launch
    (gather attention, partial exchange, merge), the K timed steps captured
    in one CUDA graph with event nodes.  NCCL exchange: candidates -> NCCL
    all-gather -> select -> attend -> NCCL all-gather -> merge, eager.  Time
    = max over ranks of the summed per-step device time."""
    import datetime
    import torch.distributed as dist
    from santapp_b200.attention import santapp as S
    from santapp_b200.attention.sharded import ShardedDecodeStep
    from santapp_b200.synthetic import make_shard_workload, scaled_shape
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    try:
        base = WORKLOADS[args.workload]
        shape = scaled_shape(base, steps=max(base.steps, args.steps + args.warmup))
        if args.batch is not None:
            shape = scaled_shape(shape, batch=args.batch)
        p = make_shard_workload(shape, rank, world, seed=args.seed, device=dev)
        summ = S.build_summary(p.keys, p.values, p.labels, p.n_clusters,
                               sample_end=p.sample_end, n_total=p.n_total)
        runner = ShardedDecodeStep(p.keys, p.values, summ, num_query_heads=shape.num_query_heads,
                                   n_total=p.n_total, topk_clusters=shape.topk_clusters,
                                   samples=p.samples, shard_index=rank, num_shards=world,
                                   cluster_base=p.cluster_base, seed=args.seed,
                                   transport=args.transport)
        p2p = runner.p2p is not None
        queries = p.queries
        flush = L2Flush(dev)
        torch.cuda.synchronize()
        dist.barrier()
        for i in range(args.warmup):
            flush()
            runner(queries[i], step=i)
        torch.cuda.synchronize()
        if p2p:
            runner.check_p2p()

        # peer memory: per step events around (select | attend); NCCL: around
        # (keys | exchange 1 | select | attend | exchange 2 | merge)
        names = (["select", "attend"] if p2p else
                 ["keys", "exchange_keys", "select", "attend", "exchange_partials", "merge"])
        ev = [[torch.cuda.Event(enable_timing=True, external=p2p) for _ in range(len(names) + 1)]
              for _ in range(args.steps)]

        def one_step(i, e, stream=None, split=True):
            st = args.warmup + i
            if p2p:
                runner.begin(queries[st], st)
                e[0].record(stream)
                runner.plan(stream=stream)
                if split:
                    e[1].record(stream)
                runner.execute(stream=stream)
                e[2].record(stream)
                return
            e[0].record(stream)
            runner.candidates(queries[st], st, stream=stream)
            e[1].record(stream)
            runner.exchange_keys()
            e[2].record(stream)
            runner.plan(stream=stream)
            e[3].record(stream)
            runner.execute(stream=stream)
            e[4].record(stream)
            runner.exchange_partials()
            e[5].record(stream)
            runner.merge(stream=stream)
            e[6].record(stream)

        graph = None

        def capture(events, split):
            # the K timed steps (each behind its L2 flush) as one CUDA graph,
            # as the single-GPU run; every captured launch carries its step's
            # epoch, and every rank captures the same sequence
            cap = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    for i in range(args.steps):
                        flush()
                        one_step(i, events[i], cap, split)
            torch.cuda.synchronize()
            return g

        if p2p:
            # timed without an event between the two launches (the attention
            # launch overlaps the selection's tail, as in a serving loop); the
            # phase split comes from a second graph of the same steps below
            graph = capture(ev, False)
        clocks = ClockSampler(local)
        clocks.start()
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        head_start = 0.0
        if graph is not None:
            graph.replay()
        else:
            # Eager steps are enqueued by Python (ctypes calls, NCCL calls,
            # event records).  A device-side spin ahead of the first step,
            # outside every event, lets the host fill the launch queue before
            # the GPU starts, so that the per-step events time the kernels
            # and collectives rather than a GPU waiting for its next launch.
            head_start = HEAD_START_S
            torch.cuda._sleep(int(head_start * 1.965e9))
            for i in range(args.steps):
                flush()
                one_step(i, ev[i])
        enqueued = time.perf_counter() - t0
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        clk = clocks.stop()
        del graph
        if p2p:
            runner.check_p2p()
            steps_ms = np.array([e[0].elapsed_time(e[2]) for e in ev])
            ev2 = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
                   for _ in range(args.steps)]
            dist.barrier()
            g2 = capture(ev2, True)
            dist.barrier()
            g2.replay()
            torch.cuda.synchronize()
            del g2
            runner.check_p2p()
            ph = np.array([[e[j].elapsed_time(e[j + 1]) for j in range(len(names))] for e in ev2])
        else:
            ph = np.array([[e[j].elapsed_time(e[j + 1]) for j in range(len(names))] for e in ev])
            steps_ms = ph.sum(axis=1)
        mine = torch.tensor([steps_ms.sum()], dtype=torch.float64, device=dev)
        dist.all_reduce(mine, op=dist.ReduceOp.MAX)
        total_ms = float(mine.item())
        value = shape.batch * args.steps / (total_ms / 1e3)
        phase = {k: float(v) for k, v in zip(names, ph.mean(axis=0))}
        # per-rank step times: the limiter is the slowest rank
        per_rank = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
        dist.all_gather(per_rank, torch.tensor([steps_ms.sum() / args.steps],
                                               dtype=torch.float64, device=dev))

        # end to end through the public call: pinned q in, merged out back
        e2e = None
        if not args.no_e2e:
            q_host = queries[:args.steps].cpu().pin_memory()
            out_host = torch.empty(shape.batch, shape.num_query_heads,
                                   shape.head_dim).pin_memory()
            q_dev = torch.empty_like(queries[0])
            dist.barrier()
            torch.cuda.synchronize()
            # as the single-GPU e2e: every step's output is read back into
            # pinned memory and waited for before the next step is issued
            t0 = time.perf_counter()
            for i in range(args.steps):
                q_dev.copy_(q_host[i], non_blocking=True)
                out = runner(q_dev, step=args.warmup + args.steps + i)
                out_host.copy_(out, non_blocking=True)
                torch.cuda.current_stream().synchronize()
            t = torch.tensor([(time.perf_counter() - t0) * 1e3], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e = {"value": shape.batch * args.steps / (float(t.item()) / 1e3),
                   "unit": "tokens/s", "h2d_bytes_per_step": int(q_host[0].numel() * 4),
                   "d2h_bytes_per_step": int(out_host.numel() * 4),
                   "api": "santapp_b200.attention.ShardedDecodeStep (ctypes -> "
                          + ("santa_shard_plan / santa_shard_attend C ABI, peer-memory exchange)"
                             if p2p else "santa_shard_* C ABI, NCCL all-gathers)")}
        peak, peak_kind = peaks()
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16" if shape.kv_dtype == torch.bfloat16 else "f32",
            "data": "synthetic (seeded Gaussian-mixture keys per shard, N(0,1) values and "
                    "queries)",
            "config": decode_config(shape, "hybrid", world, p2p=p2p),
            "shard": {"tokens": p.n_total, "clusters": p.n_clusters, "samples": p.samples},
            "phase_ms": phase,
            "rank_ms_per_step": [round(float(x.item()), 5) for x in per_rank],
            "timing": ("CUDA events around each step's launches on every rank, max over ranks "
                       "of the sum; "
                       + ("the K timed steps as one CUDA graph (flush, select, attend per step)"
                          if p2p else f"eager launches behind a {head_start * 1e3:.0f} ms "
                                      "device spin that lets the host queue steps ahead")),
            "wall_s": wall,
            "host_enqueue_s": enqueued,
            "clocks": clk,
            "gpu_launches": runner.kernels_per_call * args.steps,
            "e2e": e2e,
            "cpu_baseline": None,
            "roofline": {"kernel": "decode_attend_gather_kernel", "bound": "hbm",
                         "achieved": None, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": None, "traffic": None,
                         "note": "per-kernel roofline is reported by the single-GPU run"},
        }
        if p2p:
            bad = torch.tensor([int(runner.p2p_error.item())], device=dev)
            dist.all_reduce(bad, op=dist.ReduceOp.MAX)
            line["p2p_wait_timeouts"] = int(bad.item())
            # the same step through the NCCL exchanges: same kernels, same
            # merge arithmetic, so the outputs must agree bit for bit
            ref = ShardedDecodeStep(p.keys, p.values, summ,
                                    num_query_heads=shape.num_query_heads, n_total=p.n_total,
                                    topk_clusters=shape.topk_clusters, samples=p.samples,
                                    shard_index=rank, num_shards=world,
                                    cluster_base=p.cluster_base, seed=args.seed)
            st = args.warmup
            a = runner(queries[st], step=st).clone()
            b = ref(queries[st], step=st)
            torch.cuda.synchronize()
            diff = torch.tensor([float((a - b).abs().max())], dtype=torch.float64, device=dev)
            dist.all_reduce(diff, op=dist.ReduceOp.MAX)
            line["p2p_vs_nccl_max_abs_diff"] = float(diff.item())
        # (the CPU baseline is timed by the single-GPU run: under torchrun the
        # host cores are shared with the other ranks' processes)
        dist.barrier()
        return line if rank == 0 else None
    finally:
        dist.barrier()
        if "runner" in locals():
            torch.cuda.synchronize()
            runner.close()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# reference arm: the CPU restatement on all host cores
# ---------------------------------------------------------------------------

def run_reference(args, rank, world):
    """The reference's decode path on the host cores: the torch-CPU
    restatement of SantaPlusEngine._approximate_attention for the hybrid
    estimator (one call per (sequence, query head), torch intra-op threads
    on every core), on the same workload and config as our arm.  Each step
    decodes a bounded sample of that workload (one sequence's query heads
    over its full cache), reported as tokens/s.  Under torchrun only rank 0
    runs."""
    if rank != 0:
        return None
    shape = WORKLOADS[args.workload]
    if shape is None:
        raise SystemExit("the reference arm times the decode workloads")
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    w, summ = _port_sample(shape, args.seed)
    gen = torch.Generator().manual_seed(args.seed)
    n_q = w.queries.shape[0]
    for i in range(args.warmup):
        _port_step(shape, w, summ, i % n_q, gen)
    t0 = time.perf_counter()
    for i in range(args.steps):
        _port_step(shape, w, summ, (args.warmup + i) % n_q, gen)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    sample = (f"{args.steps} decode steps of sequence 0 of the batch ({shape.num_query_heads} "
              f"query-head calls per step over {shape.num_kv_heads} KV heads x {shape.context} "
              "tokens), torch-CPU restatement of the reference's per-head "
              "_approximate_attention (oracle/santa_torch_port.py)")
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian-mixture keys, N(0,1) values and queries)",
        "config": decode_config(shape, args.mode, world, p2p=args.transport == "p2p"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference is Python over torch and is not present at run time; its "
                "per-head CPU path is timed through a torch restatement with the same ops",
    }


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        line = run_sharded(args, rank, world)
    elif args.gpus > 1:
        raise SystemExit("--gpus N > 1 runs under torchrun (one process per GPU)")
    elif args.workload == "qwen7b-prefill-32k":
        line = run_prefill(args)
    elif args.workload == "qwen7b-model-64k":
        line = run_model(args)
    else:
        line = run_ours(args, rank, world)
    if line is not None and rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
