"""Worker of tests/test_sharded_multi_gpu.py: one rank of a real multi-GPU
sequence-sharded decode (launched by torchrun, one process per GPU).

Every rank decodes its shard of the same workload for three steps through
both exchange paths (NCCL all-gathers, and the kernels' own peer-memory
exchange); the outputs of the two must agree bit for bit and be identical on
every rank.  Rank 0 then rebuilds every shard on the host and checks the
selections of its own shard and the merged output against the oracle's
sharded estimator (max-abs 2e-2 / mean-abs 2e-3).  Prints "RANK r OK".
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
    try:
        for step in range(3):  # both parities of the exchange buffers
            q = p.queries[step].contiguous()
            a = nccl(q, step=step).clone()
            sel = nccl.select()
            b = peer(q, step=step).clone()
            torch.cuda.synchronize()
            peer.check_p2p()
            assert torch.equal(a, b), f"rank {rank} step {step}: exchange paths differ"
            assert torch.equal(nccl.lse, peer.lse) and torch.equal(nccl.ess, peer.ess)
            every = [torch.empty_like(a) for _ in range(world)]
            dist.all_gather(every, a)
            for x in every:
                assert torch.equal(x, a), "ranks hold different merged outputs"
        # oracle check of the last step on rank 0 (every shard rebuilt on the host)
        if rank == 0:
            parts = [make_shard_workload(SH, r, world, seed=seed) for r in range(world)]
            bases = [pp.cluster_base for pp in parts]
            errs = []
            qh = q.cpu().numpy()
            for bb in range(SH.batch):
                for h in range(SH.num_query_heads):
                    kv = h // SH.group
                    shards = []
                    for pp in parts:
                        K = pp.keys[bb, kv].float().numpy()
                        osum = O.build_summary(K[:pp.sample_end], pp.labels[bb, kv].numpy(),
                                               pp.n_clusters)
                        shards.append((K, pp.values[bb, kv].float().numpy(), osum,
                                       pp.sample_end, pp.n_total))
                    osel = O.shard_topk([s_[2] for s_ in shards], qh[bb, h], SH.scale,
                                        SH.topk_clusters, bases)
                    got = np.nonzero(sel[0][bb, h].cpu().numpy())[0]
                    assert np.array_equal(got, osel[0]), (bb, h)
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
            assert e.max() < 2e-2 and e.mean() < 2e-3, (e.max(), e.mean())
            print(f"oracle max-abs {e.max():.3g} mean-abs {e.mean():.3g}", flush=True)
        dist.barrier()
        print(f"RANK {rank} OK", flush=True)
    finally:
        torch.cuda.synchronize()
        peer.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
