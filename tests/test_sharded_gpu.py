"""Sequence-sharded decode on one GPU: the shards of a workload are decoded
one after another on the same device, the exchanges are tensor copies, and
the result is compared with the oracle's sharded estimator.

Bit-exact: each shard's selected clusters (the global top-k) and sample rows.
Attention output: max-abs 2e-2 / mean-abs 2e-3 against the fp64 oracle (the
stated bf16 tolerance); observed errors are ~1e-6.
"""
import numpy as np
import pytest
import torch

from oracle import santa_oracle as O
from santapp_b200.attention import santapp as S
from santapp_b200.attention.sharded import ShardedDecodeStep
from santapp_b200.synthetic import QWEN7B_32K, make_shard_workload, scaled_shape

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

SH = scaled_shape(QWEN7B_32K, name="shard-gpu", batch=2, context=3000, true_clusters=24,
                  n_clusters=24, topk_clusters=5, samples=48, steps=2)


class Shards:
    def __init__(self, shape, n, injected, seed=0):
        self.shape, self.n, self.seed = shape, n, seed
        self.parts = [make_shard_workload(shape, r, n, seed=seed) for r in range(n)]
        self.steps = []
        for r, p in enumerate(self.parts):
            kc, vc = p.keys.cuda(), p.values.cuda()
            summ = S.build_summary(kc, vc, p.labels.cuda(), p.n_clusters,
                                   sample_end=p.sample_end, n_total=p.n_total)
            self.steps.append(ShardedDecodeStep(
                kc, vc, summ, num_query_heads=shape.num_query_heads, n_total=p.n_total,
                topk_clusters=shape.topk_clusters, samples=p.samples, shard_index=r,
                num_shards=n, cluster_base=p.cluster_base, seed=seed, injected=injected))
        self.osum = {}
        for r, p in enumerate(self.parts):
            for b in range(shape.batch):
                for kv in range(shape.num_kv_heads):
                    K = p.keys[b, kv].float().numpy()
                    self.osum[(r, b, kv)] = O.build_summary(K[:p.sample_end],
                                                            p.labels[b, kv].numpy(), p.n_clusters)

    def exchange_keys(self):
        for st in self.steps:
            for r, src in enumerate(self.steps):
                st.all_keys[r].copy_(src.keys)

    def exchange_partials(self):
        for st in self.steps:
            for r, src in enumerate(self.steps):
                st.all_partials[r].copy_(src.partial)

    def run(self, step, ranks=None):
        q = self.parts[0].queries[step].cuda().contiguous()
        for st in self.steps:
            st.candidates(q, step)
        self.exchange_keys()
        sels = []
        for r, st in enumerate(self.steps):
            sa = ranks[r] if ranks is not None else None
            sels.append(st.select(sa))
            st.plan(sa)
            st.execute()
        self.exchange_partials()
        outs = [st.merge() for st in self.steps]
        torch.cuda.synchronize()
        return q, sels, outs

    def oracle_shards(self, b, kv):
        res = []
        for r, p in enumerate(self.parts):
            res.append((p.keys[b, kv].float().numpy(), p.values[b, kv].float().numpy(),
                        self.osum[(r, b, kv)], p.sample_end, p.n_total))
        return res


def _oracle_ranks(sh, parts, osums, sels, b, h, seed=None, step=0, injected=None):
    out = []
    for r, (p, summ, sel) in enumerate(zip(parts, osums, sels)):
        n_rest = p.sample_end - int(sum(summ.lengths[c] for c in sel))
        if n_rest <= 0:
            out.append(np.zeros(0, np.int64))
        elif injected is not None:
            out.append(injected[r][b, h].cpu().numpy().astype(np.int64))
        else:
            from santapp_b200.attention.sharded import shard_seed
            out.append(O.philox_ranks(shard_seed(seed, r), step, b, h, p.samples, n_rest))
    return out


def _check(sh_obj, q, sels, outs, ranks_of, tol=(2e-2, 2e-3)):
    sh = sh_obj.shape
    g = sh.group
    bases = [p.cluster_base for p in sh_obj.parts]
    errs = []
    for b in range(sh.batch):
        for h in range(sh.num_query_heads):
            kv = h // g
            shards = sh_obj.oracle_shards(b, kv)
            qv = q[b, h].cpu().numpy()
            osel = O.shard_topk([s[2] for s in shards], qv, sh.scale, sh.topk_clusters, bases)
            for r in range(sh_obj.n):
                got = np.nonzero(sels[r][0][b, h].cpu().numpy())[0]
                assert np.array_equal(got, osel[r]), (b, h, r)
            ranks = ranks_of(b, h, osel, [s[2] for s in shards])
            for r in range(sh_obj.n):
                rows = sels[r][1][b, h].cpu().numpy()
                summ = shards[r][2]
                exp = (O.hybrid_positions(summ, osel[r], ranks[r]) if len(ranks[r])
                       else np.zeros(0, np.int64))
                assert np.array_equal(rows[: len(exp)], exp), (b, h, r)
                assert (rows[len(exp):] == -1).all()
            ref = O.decode_hybrid_sharded(qv, shards, sh.topk_clusters, ranks, sh.scale, bases)
            for out in outs:  # every rank holds the same merged output
                assert torch.equal(out[b, h], outs[0][b, h])
            e = np.abs(outs[0][b, h].cpu().numpy() - ref.out)
            errs.append(e)
            lse = float(sh_obj.steps[0].lse[b, h])
            assert abs(lse - ref.lse) < 1e-3
            ess = float(sh_obj.steps[0].ess[b, h])
            assert abs(ess - ref.ess) < 1e-4
    e = np.stack(errs)
    assert e.max() < tol[0] and e.mean() < tol[1], (e.max(), e.mean())
    return e.max()


@pytest.mark.parametrize("n", [1, 2, 3])
def test_sharded_injected_draws_match_oracle(n):
    sh = SH
    obj = Shards(sh, n, injected=True)
    rs = np.random.RandomState(7 + n)
    # injected ranks must lie in [0, n_rest): draw after the selection is known
    q = obj.parts[0].queries[0].cuda()
    for st in obj.steps:
        st.candidates(q, 0)
    obj.exchange_keys()
    ranks_t = []
    for r, st in enumerate(obj.steps):
        sel, _, n_exact = st.select(torch.zeros(sh.batch, sh.num_query_heads, st.p.samples,
                                                dtype=torch.int32, device="cuda"))
        n_rest = obj.parts[r].sample_end - n_exact.cpu().numpy()
        ra = np.zeros((sh.batch, sh.num_query_heads, st.p.samples), np.int32)
        for b in range(sh.batch):
            for h in range(sh.num_query_heads):
                if n_rest[b, h] > 0:
                    ra[b, h] = rs.randint(0, n_rest[b, h], st.p.samples)
        ranks_t.append(torch.from_numpy(ra).cuda())
    q, sels, outs = obj.run(0, ranks_t)

    def ranks_of(b, h, osel, osums):
        return _oracle_ranks(sh, obj.parts, osums, osel, b, h, injected=ranks_t)

    _check(obj, q, sels, outs, ranks_of)


@pytest.mark.parametrize("n", [2, 4])
def test_sharded_device_sampler_matches_philox_oracle(n):
    sh = SH
    obj = Shards(sh, n, injected=False, seed=11)
    q, sels, outs = obj.run(1)

    def ranks_of(b, h, osel, osums):
        return _oracle_ranks(sh, obj.parts, osums, osel, b, h, seed=11, step=1)

    _check(obj, q, sels, outs, ranks_of)


def test_one_shard_equals_santa_decode():
    sh = SH
    obj = Shards(sh, 1, injected=False, seed=3)
    q, _, outs = obj.run(0)
    p, st = obj.parts[0], obj.steps[0]
    res = S.santa_decode(q, st.key_cache, st.value_cache, st.summary, mode="hybrid",
                         n_total=p.n_total, topk_clusters=sh.topk_clusters, samples=sh.samples,
                         seed=3, with_stats=True)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], res.out)
    assert torch.equal(st.lse, res.lse)
    assert torch.allclose(st.ess, res.ess, rtol=1e-6, atol=0)


def test_shard_api_rejects_unsupported():
    sh = SH
    p = make_shard_workload(sh, 0, 2)
    kc, vc = p.keys.cuda(), p.values.cuda()
    summ = S.build_summary(kc, vc, p.labels.cuda(), p.n_clusters, sample_end=p.sample_end,
                           n_total=p.n_total)
    with pytest.raises(ValueError):  # 32 shards x top-20 > 512 candidate keys
        ShardedDecodeStep(kc, vc, summ, num_query_heads=sh.num_query_heads, n_total=p.n_total,
                          topk_clusters=20, samples=8, shard_index=0, num_shards=32,
                          cluster_base=0)
    with pytest.raises(ValueError):
        ShardedDecodeStep(kc.float(), vc.float(), summ, num_query_heads=sh.num_query_heads,
                          n_total=p.n_total, topk_clusters=4, samples=8, shard_index=0,
                          num_shards=2, cluster_base=0)


class PeerShards:
    """The peer-memory form of the same shards on one GPU.  Emulated ranks
    share one device, so no kernel may wait for another one's stores: before
    rank r's launches, the other ranks' words of the step (their keys and
    partials, from the NCCL-form run of the same step, tagged with the
    epoch) are written into rank r's buffer, so its waits find them at once.
    The exchange buffers are torch allocations (zeroed) on this device."""

    def __init__(self, base: Shards, wait_limit_us=0):
        from santapp_b200.attention.sharded import exchange_layout
        sh = base.shape
        self.base, self.n = base, base.n
        self.steps = []
        for r, p in enumerate(base.parts):
            st0 = base.steps[r]
            self.steps.append(ShardedDecodeStep(
                st0.key_cache, st0.value_cache, st0.summary,
                num_query_heads=sh.num_query_heads, n_total=p.n_total,
                topk_clusters=sh.topk_clusters, samples=p.samples, shard_index=r,
                num_shards=self.n, cluster_base=p.cluster_base, seed=base.seed,
                wait_limit_us=wait_limit_us))
        st = self.steps[0]
        self.lay = exchange_layout(self.n, st.rows, st.topk, st.head_dim)
        self.bufs = [torch.zeros(self.lay["bytes"], dtype=torch.uint8, device="cuda")
                     for _ in range(self.n)]
        for s_ in self.steps:
            s_.bind_p2p([b.data_ptr() for b in self.bufs])

    def _words(self, r, region, epoch, rank):
        """The int64 words of `rank`'s slot of `region` in buffer r."""
        st = self.steps[0]
        per = st.rows * (st.topk if region == "keys" else st.partial.shape[1])
        off = self.lay[region] // 8 + ((epoch & 1) * self.n + rank) * per
        return self.bufs[r].view(torch.int64)[off: off + per]

    def run(self, step, ref_keys, ref_partials):
        """Step `step` on every emulated rank; ref_keys / ref_partials: every
        rank's candidate keys and partials of this step (NCCL form)."""
        from santapp_b200.attention.sharded import key_words, partial_words
        q = self.base.parts[0].queries[step].cuda().contiguous()
        outs, sels = [], []
        for r, st in enumerate(self.steps):
            st.begin(q, step)
            for o in range(self.n):
                if o != r:
                    self._words(r, "keys", st.epoch, o).copy_(key_words(ref_keys[o],
                                                                              st.epoch))
            st.plan()
            sels.append(st.select())
            for o in range(self.n):
                if o != r:
                    self._words(r, "parts", st.epoch, o).copy_(
                        partial_words(ref_partials[o].reshape(-1), st.epoch))
            outs.append(st.execute().clone())
        torch.cuda.synchronize()
        return q, sels, outs


@pytest.mark.parametrize("n", [1, 2, 3])
def test_sharded_peer_memory_exchange_matches_nccl_form(n):
    """The kernels' own exchange (selection launch: candidates + key exchange
    + threshold selection; attention launch: partial exchange + merge) gives
    the same bits as the NCCL form with its four launches and host-side
    exchanges, over both parities of the exchange buffers, and the result
    matches the oracle's sharded estimator."""
    sh = scaled_shape(SH, steps=3)
    ref = Shards(sh, n, injected=False, seed=5)
    obj = PeerShards(ref)
    for step in range(3):
        q, sels_ref, outs_ref = ref.run(step)
        keys = [st.keys.clone() for st in ref.steps]
        parts = [st.partial.clone() for st in ref.steps]
        _, sels, outs = obj.run(step, keys, parts)
        for r in range(n):
            assert torch.equal(sels[r][0], sels_ref[r][0]), (step, r)
            assert torch.equal(sels[r][1], sels_ref[r][1]), (step, r)
            assert torch.equal(outs[r], outs_ref[0]), (step, r)
            assert torch.equal(obj.steps[r].lse, ref.steps[0].lse)
            assert torch.equal(obj.steps[r].ess, ref.steps[0].ess)
        assert all(int(st.p2p_error.item()) == 0 for st in obj.steps)

    def ranks_of(b, h, osel, osums):
        return _oracle_ranks(sh, ref.parts, osums, osel, b, h, seed=5, step=2)

    _check(ref, q, sels_ref, outs_ref, ranks_of)


def test_peer_memory_wait_runs_out():
    """A peer that never sends: rank 0 of two emulated shards runs alone with
    a 2 ms wait limit.  Its selection launch gives up waiting for rank 1's
    keys and sets the error flag; the attention launch sees the flag, does
    not wait at all and writes NaN outputs; both launches return; the Python
    step raises on its next call and in check_p2p()."""
    sh = scaled_shape(SH, steps=2)
    ref = Shards(sh, 2, injected=False, seed=9)
    obj = PeerShards(ref, wait_limit_us=2000)
    st = obj.steps[0]
    q = ref.parts[0].queries[0].cuda().contiguous()
    out = st(q, 0)
    torch.cuda.synchronize()
    assert int(st.p2p_error.item()) == 1
    assert torch.isnan(out).all()
    assert torch.isnan(st.lse).all()
    with pytest.raises(RuntimeError, match="ran out of time"):
        st.check_p2p()
    with pytest.raises(RuntimeError, match="ran out of time"):
        st(q, 1)
