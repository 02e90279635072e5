"""Worker of tests/test_sharded_multi_gpu.py: one rank of a real multi-GPU
sequence-sharded decode (launched by torchrun, one process per GPU).

Every rank decodes its shard of the same workload for three steps through
both exchange paths (NCCL all-gathers, and the kernels' own peer-memory
exchange); the outputs of the two must agree bit for bit and be identical on
every rank.  Rank 0 then rebuilds every shard (with the ranks' own device
generator) and checks the selections of its own shard and the merged output
against the oracle's sharded estimator (max-abs 2e-2 / mean-abs 2e-3).
Every rank takes the same collective steps on failure too; prints "RANK r OK"
or one "RANK r FAIL ..." line per failure.
"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "opus-lab-notebooks_b200"))
sys.path.insert(0, os.path.dirname(HERE))

from oracle import santa_oracle as O  # noqa: E402
from santapp_b200.attention import santapp as S  # noqa: E402
from santapp_b200.attention.sharded import ShardedDecodeStep, shard_seed  # noqa: E402
from santapp_b200.synthetic import QWEN3_8B_128K, make_shard_workload, scaled_shape  # noqa: E402

SH = scaled_shape(QWEN3_8B_128K, name="mgpu", batch=2, context=8192, true_clusters=64,
                  n_clusters=64, topk_clusters=8, samples=64, steps=3)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    seed = 3
    p = make_shard_workload(SH, rank, world, seed=seed, device=dev)
    summ = S.build_summary(p.keys, p.values, p.labels, p.n_clusters, sample_end=p.sample_end,
                           n_total=p.n_total)
    kw = dict(num_query_heads=SH.num_query_heads, n_total=p.n_total,
              topk_clusters=SH.topk_clusters, samples=p.samples, shard_index=rank,
              num_shards=world, cluster_base=p.cluster_base, seed=seed)
    nccl = ShardedDecodeStep(p.keys, p.values, summ, transport="nccl", **kw)
    peer = ShardedDecodeStep(p.keys, p.values, summ, transport="p2p", **kw)
    # Every rank takes the same collective steps whatever fails: a failure is
    # recorded, the steps go on, and the ranks agree on the outcome at the end.
    failures = []
    try:
        for step in range(3):  # both parities of the exchange buffers
            q = p.queries[step].contiguous()
            a = nccl(q, step=step).clone()
            sel = nccl.select()
            b = peer(q, step=step).clone()
            torch.cuda.synchronize()
            try:
                peer.check_p2p()
            except RuntimeError as e:
                failures.append(f"step {step}: {e}")
            if not torch.equal(a, b):
                failures.append(f"step {step}: exchange paths differ")
            if not (torch.equal(nccl.lse, peer.lse) and torch.equal(nccl.ess, peer.ess)):
                failures.append(f"step {step}: lse / ess differ between exchange paths")
            every = [torch.empty_like(a) for _ in range(world)]
            dist.all_gather(every, a)
            if not all(torch.equal(x, a) for x in every):
                failures.append(f"step {step}: ranks hold different merged outputs")
        if rank == 0:
            try:
                oracle_check(world, seed, dev, q, sel, a)
            except AssertionError as e:
                failures.append(f"oracle check: {e}")
    finally:
        # every rank's kernels are done (its synchronize precedes its part of
        # the reduction) before any rank unmaps the exchange buffers
        torch.cuda.synchronize()
        flag = torch.tensor([len(failures)], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        any_failed = int(flag.item())
        peer.close()
        dist.destroy_process_group()
    for f in failures:
        print(f"RANK {rank} FAIL {f}", flush=True)
    if failures or any_failed:
        sys.exit(1)
    print(f"RANK {rank} OK", flush=True)


def oracle_check(world, seed, dev, q, sel, a):
    """Rank 0: rebuild every shard (on the device, so that the generator is
    the one the ranks used, then on the host) and check this shard's
    selections and the merged output of the last step against the oracle's
    sharded estimator."""
    parts = [make_shard_workload(SH, r, world, seed=seed, device=dev) for r in range(world)]
    bases = [pp.cluster_base for pp in parts]
    errs = []
    qh = q.cpu().numpy()
    sel0 = sel[0].cpu().numpy()
    host = [(pp.keys.float().cpu().numpy(), pp.values.float().cpu().numpy(),
             pp.labels.cpu().numpy()) for pp in parts]
    for bb in range(SH.batch):
        for kv in range(SH.num_kv_heads):
            shards = []
            for pp, (K, V, L) in zip(parts, host):
                osum = O.build_summary(K[bb, kv, :pp.sample_end], L[bb, kv], pp.n_clusters)
                shards.append((K[bb, kv], V[bb, kv], osum, pp.sample_end, pp.n_total))
            for h in range(kv * SH.group, (kv + 1) * SH.group):
                osel = O.shard_topk([s_[2] for s_ in shards], qh[bb, h], SH.scale,
                                    SH.topk_clusters, bases)
                got = np.nonzero(sel0[bb, h])[0]
                assert np.array_equal(got, osel[0]), f"selection of (b {bb}, head {h})"
                ranks = []
                for r, (pp, s_) in enumerate(zip(parts, shards)):
                    n_rest = pp.sample_end - int(sum(s_[2].lengths[c] for c in osel[r]))
                    ranks.append(O.philox_ranks(shard_seed(seed, r), 2, bb, h, pp.samples,
                                                n_rest) if n_rest > 0
                                 else np.zeros(0, np.int64))
                ref = O.decode_hybrid_sharded(qh[bb, h], shards, SH.topk_clusters, ranks,
                                              SH.scale, bases)
                errs.append(np.abs(a[bb, h].cpu().numpy() - ref.out))
    e = np.stack(errs)
    assert e.max() < 2e-2 and e.mean() < 2e-3, f"max-abs {e.max():.3g} mean-abs {e.mean():.3g}"
    print(f"oracle max-abs {e.max():.3g} mean-abs {e.mean():.3g}", flush=True)


if __name__ == "__main__":
    main()
