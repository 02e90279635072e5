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
    def __init__(self, shape, n, injected, seed=0, p2p=False):
        self.shape, self.n = shape, n
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
        self.p2p = p2p
        self.buffers = []
        if p2p:  # one exchange buffer per shard, all on this device
            import ctypes
            from santapp_b200 import _lib
            lib = _lib.load()
            nbytes = self.steps[0].p2p_buffer_bytes()
            for _ in range(n):
                ptr = ctypes.c_void_p()
                _lib.check("alloc", lib.santa_p2p_alloc(nbytes, ctypes.byref(ptr)))
                self.buffers.append(ptr.value)
            for st in self.steps:
                st.bind_p2p(self.buffers)
        self.osum = {}
        for r, p in enumerate(self.parts):
            for b in range(shape.batch):
                for kv in range(shape.num_kv_heads):
                    K = p.keys[b, kv].float().numpy()
                    self.osum[(r, b, kv)] = O.build_summary(K[:p.sample_end],
                                                            p.labels[b, kv].numpy(), p.n_clusters)

    def _raise_flags(self, ex):
        """Emulated ranks share one stream, so no kernel may wait for another:
        after the producing kernels finished, the host raises every shard's
        flag in every buffer; the consuming kernels then find them up."""
        import ctypes
        from santapp_b200 import _lib
        torch.cuda.synchronize()
        lib = _lib.load()
        epoch = self.steps[0].epoch
        for buf in self.buffers:
            for r in range(self.n):
                _lib.check("poke", lib.santa_p2p_poke(ctypes.c_void_p(buf + (ex * 32 + r) * 8),
                                                      epoch))

    def exchange_keys(self):
        if self.p2p:  # the kernels wrote every shard's keys into every buffer
            self._raise_flags(0)
            return
        for st in self.steps:
            for r, src in enumerate(self.steps):
                st.all_keys[r].copy_(src.keys)

    def exchange_partials(self):
        if self.p2p:
            self._raise_flags(1)
            return
        for st in self.steps:
            for r, src in enumerate(self.steps):
                st.all_partials[r].copy_(src.partial)

    def close(self):
        import ctypes
        from santapp_b200 import _lib
        for ptr in self.buffers:
            _lib.load().santa_p2p_free(ctypes.c_void_p(ptr))
        self.buffers = []

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


@pytest.mark.parametrize("n", [2, 3])
def test_sharded_peer_memory_exchange_matches_oracle(n):
    """The kernels' own exchange (keys and partials stored into every
    shard's buffer, flags awaited) gives the same result as the host-side
    exchange.  The emulated shards run on one stream, so the host raises the
    flags between the producing and the consuming kernels and no wait is
    ever outstanding."""
    sh = scaled_shape(SH, steps=3)
    obj = Shards(sh, n, injected=False, seed=5, p2p=True)
    ref = Shards(sh, n, injected=False, seed=5)
    for step in range(3):  # both parities of the exchange buffers
        q, sels, outs = obj.run(step)
        _, _, outs_ref = ref.run(step)
        for out in outs:
            assert torch.equal(out, outs_ref[0])
        assert all(int(st.p2p_error.item()) == 0 for st in obj.steps)

    def ranks_of(b, h, osel, osums):
        return _oracle_ranks(sh, obj.parts, osums, osel, b, h, seed=5, step=2)

    _check(obj, q, sels, outs, ranks_of)
    obj.close()
