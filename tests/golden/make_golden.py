"""Generate the golden vectors under tests/golden/ by running the reference.

Run in a container where the reference source tree is mounted (read-only is
fine), naming its ``src`` directory:

    python tests/golden/make_golden.py --reference-src PATH
    SANTA_REFERENCE_SRC=PATH python tests/golden/make_golden.py

It imports santapp_ruler from the reference's ``src`` directory and drives
its hot-path functions headlessly on seeded synthetic inputs:

* ``SklearnLikeTorchMiniBatchKMeans.fit_predict``  (minibatch_kmeans.py:128-334)
* ``SantaPlusEngine._build_summary``                (santapp.py:508-540)
* ``SantaPlusEngine._approximate_attention``        (santapp.py:365-506)
  in the topk, guided, uniform and santa modes, with the engine's
  ``DecodeTrafficTracker`` (santapp.py:80-142) accumulating over every head
  call of a mode: its ``as_dict()`` and each call's exact-token count and ESS
  ratio are kept.

Shims (documented in the fixture's ``notes`` field):

1. The engine is built with ``object.__new__`` and the attributes the hot
   path reads are set directly (no model is loaded).
2. ``torch.argsort`` is made stable for the duration of each call, so the
   member order inside a cluster and equal-guess cluster order are
   deterministic (lowest index first).  santapp.py:401 and :517 call the
   unstable default.
3. ``torch.multinomial``, ``torch.rand`` and ``torch.randint`` are wrapped to
   record the draws of guided / uniform / santa mode, so the CUDA path can be
   fed the same samples.

Inputs are not stored: they are regenerated from the seed by
``santapp_b200.synthetic`` and guarded by a sha256 digest kept in the fixture.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "opus-lab-notebooks_b200"))

from santapp_b200.synthetic import (  # noqa: E402
    QWEN05B_4K, QWEN7B_32K, make_decode_workload, scaled_shape, tensor_digest)

# Small bf16 case with the Qwen2.5-7B head geometry (28 q-heads, 4 KV heads,
# head_dim 128) at a context the CPU reference handles in seconds.
QWEN7B_SMALL = scaled_shape(QWEN7B_32K, name="qwen2.5-7b-attn-ctx2048-b2", batch=2,
                            context=2048, true_clusters=32, n_clusters=32,
                            topk_clusters=4, samples=64, steps=1)


class _Recorder:
    def __init__(self):
        self.draws = []
        self._orig = {}

    def __enter__(self):
        for name in ("multinomial", "rand", "randint"):
            orig = getattr(torch, name)
            self._orig[name] = orig

            def wrapped(*a, __orig=orig, __name=name, **kw):
                out = __orig(*a, **kw)
                self.draws.append((__name, out.detach().clone()))
                return out
            setattr(torch, name, wrapped)
        orig_argsort = torch.argsort
        self._orig["argsort"] = orig_argsort

        def stable_argsort(x, dim=-1, descending=False, stable=False):
            return orig_argsort(x, dim=dim, descending=descending, stable=True)
        torch.argsort = stable_argsort
        return self

    def __exit__(self, *exc):
        for name, orig in self._orig.items():
            setattr(torch, name, orig)


def _engine(santapp_mod, config_mod, head_dim, mode, samples, sample_end, summaries):
    eng = object.__new__(santapp_mod.SantaPlusEngine)
    eng.head_dim = head_dim
    eng.summaries = summaries
    eng.traffic = santapp_mod.DecodeTrafficTracker()
    cfg = config_mod.SantaPlusConfig()
    cfg.mode = mode
    cfg.samples_per_head = samples
    eng.config = cfg
    eng.mode = mode
    eng.sample_end = sample_end
    return eng


def _summary_arrays(s):
    return dict(members=s.members.numpy().astype(np.int64),
                starts=s.starts.numpy().astype(np.int64),
                lengths=s.lengths_long.numpy().astype(np.int64),
                centroids=s.key_centroids.numpy().astype(np.float32))


def run_decode_case(shape, labels_by_bkv, santapp_mod, config_mod, prefix, out,
                    modes_budget):
    """Summaries + per-head reference decode for every (b, q-head)."""
    w = make_decode_workload(shape)
    out[prefix + "digest"] = np.array(tensor_digest(w.keys, w.values, w.queries))
    B, Hq, Hkv, D = shape.batch, shape.num_query_heads, shape.num_kv_heads, shape.head_dim
    g = shape.group
    se = shape.sample_end
    summaries = {}
    with _Recorder():
        helper = _engine(santapp_mod, config_mod, D, "topk", 1, se, {})
        for b in range(B):
            for kv in range(Hkv):
                keys = w.keys[b, kv, :se].float()
                lab = torch.as_tensor(labels_by_bkv[(b, kv)], dtype=torch.long)
                s = helper._build_summary(keys, lab, shape.n_clusters)
                summaries[(b, kv)] = s
                for k, v in _summary_arrays(s).items():
                    out[f"{prefix}summary_{b}_{kv}_{k}"] = v
    for mode, samples in modes_budget:
        res = np.zeros((B, Hq, D), np.float32)
        draws_g, draws_w, draws_i = [], [], []
        tracker = santapp_mod.DecodeTrafficTracker()
        n_draw = np.zeros((B, Hq), np.int64)
        ess = np.full((B, Hq), np.nan, np.float64)
        for b in range(B):
            for h in range(Hq):
                kv = h // g
                eng = _engine(santapp_mod, config_mod, D, mode, samples, se,
                              {(0, kv): summaries[(b, kv)]})
                eng.traffic = tracker
                drawn0, n_ess0 = tracker.sampled_token_draws, len(tracker.ess_ratios)
                q = w.queries[0, b, h].float()
                torch.manual_seed(1000 * b + h)
                with _Recorder() as rec:
                    o = eng._approximate_attention(q, w.keys[b, kv], w.values[b, kv], 0, kv)
                res[b, h] = o.numpy()
                n_draw[b, h] = tracker.sampled_token_draws - drawn0
                if len(tracker.ess_ratios) > n_ess0:
                    ess[b, h] = tracker.ess_ratios[-1]
                d = dict((n, t) for n, t in rec.draws)
                if mode == "guided":
                    lengths = summaries[(b, kv)].lengths_long
                    grp = d["multinomial"].numpy().astype(np.int64)
                    u = d["rand"]
                    within = torch.floor(u * lengths[d["multinomial"]].float()).long()
                    draws_g.append(grp)
                    draws_w.append(within.numpy().astype(np.int64))
                elif mode == "uniform":
                    draws_i.append(d["randint"].numpy().astype(np.int64))
                elif mode == "santa":
                    draws_i.append(d["multinomial"].numpy().astype(np.int64))
        out[f"{prefix}{mode}_out"] = res
        out[f"{prefix}{mode}_samples"] = np.array(samples)
        out[f"{prefix}{mode}_traffic"] = np.array(json.dumps(tracker.as_dict()))
        out[f"{prefix}{mode}_draws_per_call"] = n_draw
        out[f"{prefix}{mode}_ess"] = ess
        if draws_g:
            out[f"{prefix}{mode}_groups"] = np.stack(draws_g).reshape(B, Hq, -1)
            out[f"{prefix}{mode}_within"] = np.stack(draws_w).reshape(B, Hq, -1)
        if draws_i:
            out[f"{prefix}{mode}_idx"] = np.stack(draws_i).reshape(B, Hq, -1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("SANTA_REFERENCE_SRC"),
                    help="the reference's santapp-ruler-bench/src directory "
                         "(or the SANTA_REFERENCE_SRC environment variable)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("name the reference source tree: --reference-src PATH or SANTA_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from santapp_ruler import config as config_mod
    from santapp_ruler.attention import santapp as santapp_mod
    from santapp_ruler.attention.minibatch_kmeans import SklearnLikeTorchMiniBatchKMeans

    notes = ("reference driven headlessly; torch.argsort forced stable; "
             "random draws recorded from torch.multinomial/rand/randint")

    # ---- k-means fixtures ------------------------------------------------
    km = {"notes": np.array(notes)}
    w1 = make_decode_workload(QWEN05B_4K)
    km["qwen05b_digest"] = np.array(tensor_digest(w1.keys, w1.values, w1.queries))
    cases = []
    for kv in range(QWEN05B_4K.num_kv_heads):
        for seed in (0, 1, 2):
            cases.append(("qwen05b", kv, 64, 1024, 10, seed))
    w2 = make_decode_workload(scaled_shape(QWEN7B_32K, batch=1, steps=1))
    km["qwen7b_digest"] = np.array(tensor_digest(w2.keys, w2.values, w2.queries))
    cases.append(("qwen7b", 0, 256, 4096, 20, 0))
    for src, kv, k, bs, it, seed in cases:
        w = w1 if src == "qwen05b" else w2
        se = w.keys.shape[2] - 64
        x = w.keys[0, kv, :se].float()
        est = SklearnLikeTorchMiniBatchKMeans(k, batch_size=bs, max_iter=it, random_state=seed)
        lab = est.fit_predict(x)
        tag = f"{src}_kv{kv}_k{k}_bs{bs}_it{it}_s{seed}"
        km[tag + "_labels"] = lab.numpy().astype(np.int32)
        km[tag + "_centers"] = est.cluster_centers_.numpy().astype(np.float32)
        km[tag + "_counts"] = est.counts_.numpy().astype(np.float32)
        km[tag + "_n_steps"] = np.array(est.n_steps_)
        km[tag + "_inertia"] = np.array(est.inertia_)
    km["cases"] = np.array([f"{s}_kv{kv}_k{k}_bs{bs}_it{it}_s{sd}" for s, kv, k, bs, it, sd in cases])
    # the unit test of the reference (tests/test_kmeans_optional.py:12-25)
    tiny = torch.tensor([[0.0, 0.0], [0.1, 0.0], [10.0, 10.0], [10.1, 10.0]])
    km["tiny_labels"] = SklearnLikeTorchMiniBatchKMeans(
        n_clusters=2, batch_size=4, max_iter=5, random_state=0).fit_predict(tiny).numpy()
    np.savez_compressed(os.path.join(HERE, "kmeans_golden.npz"), **km)

    # ---- decode fixtures ------------------------------------------------
    dec = {"notes": np.array(notes)}
    # (a) Qwen2.5-0.5B shape, fp32, clustered by the reference k-means
    labels = {}
    for kv in range(QWEN05B_4K.num_kv_heads):
        labels[(0, kv)] = km[f"qwen05b_kv{kv}_k64_bs1024_it10_s0_labels"]
    S = QWEN05B_4K.samples
    budget = QWEN05B_4K.topk_clusters * (QWEN05B_4K.sample_end // QWEN05B_4K.n_clusters)
    run_decode_case(QWEN05B_4K, labels, santapp_mod, config_mod, "qwen05b_", dec,
                    [("topk", budget), ("guided", S), ("uniform", S), ("santa", S)])
    # (b) Qwen2.5-7B head geometry, bf16 K/V, ground-truth mixture labels
    sh = QWEN7B_SMALL
    w = make_decode_workload(sh)
    labels = {(b, kv): w.labels[b, kv, :sh.sample_end].numpy()
              for b in range(sh.batch) for kv in range(sh.num_kv_heads)}
    budget = sh.topk_clusters * (sh.sample_end // sh.n_clusters)
    run_decode_case(sh, labels, santapp_mod, config_mod, "qwen7b_", dec,
                    [("topk", budget), ("guided", sh.samples), ("uniform", sh.samples),
                     ("santa", sh.samples)])
    dec["scale_qwen05b"] = np.array(1.0 / math.sqrt(QWEN05B_4K.head_dim))
    np.savez_compressed(os.path.join(HERE, "decode_golden.npz"), **dec)
    for f in ("kmeans_golden.npz", "decode_golden.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
