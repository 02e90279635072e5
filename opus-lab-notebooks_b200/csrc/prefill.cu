// Dense prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the prefill branch of SantaPlusEngine._attention_forward
// (santapp_ruler/attention/santapp.py:320-346), which calls
// transformers' sdpa_attention_forward -> torch scaled_dot_product_attention
// with is_causal=True on [B, H, T, D] bf16 tensors with GQA (query head h reads
// KV head h / (Hq / Hkv)).
//
//   out[b, h, t] = sum_{s <= t} softmax_s(q_t . k_s * scale) v_s
//
// Two launches:
//   prefill_image_kernel  writes every 128-key tile of K and of V^T as the
//       exact 32 KB shared-memory image the MMAs read (K-major, 128-byte
//       swizzle, two 64-element halves), zero-filled past T, so one bulk copy
//       moves a tile;
//   prefill_fwd_kernel    one CTA per (pair of 128-query tiles, query head),
//       heaviest causal pairs first, warp-specialised:
//         warps 0-7 / 8-15 softmax of query tile 0 / 1, two warpgroups per
//                          tile: a thread owns one query row (= TMEM lane)
//                          and one half (64) of its scores; the halves
//                          exchange row maxima at a named barrier and row
//                          sums once at the end; P (bf16) goes back into
//                          each half's own score columns of TMEM;
//         warp 16          one thread issues every tcgen05.mma:
//                            S_t = Q_t K_j^T   (smem x smem -> TMEM cols S_t)
//                            O_t += P_t V_j    (TMEM x smem -> TMEM cols O_t)
//                          in the order S0(j) S1(j) PV0(j) S0(j+1) PV1(j)
//                          S1(j+1) ..., so the tensor core runs one tile's
//                          products while the other tile's softmax runs;
//         warp 17          one thread streams K_j and V^T_j (two stages,
//                          one 32 KB bulk copy each).
//       The softmax is bound by its instruction issue, not by the MUFU:
//       exp2 is the MUFU ex2.approx instruction, the scaling FMAs and the
//       row-sum adds use the paired fp32 instructions (two lanes each), row
//       maxima the three-input max, all over independent partial
//       accumulators (no serial chains).  The two tiles' softmax passes run
//       whenever their scores are ready (making them take turns for the
//       MUFU, or moving part of the exponentials to an FMA-pipe polynomial,
//       both measured slower).
//       TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
//       The running maximum is updated lazily: O and l are rescaled only
//       when the maximum grows by more than 8 (log2 units), so p <= 2^8.
//       tcgen05.commit orders everything: the commit after S_t(j+1) fires
//       only when PV_t(j) (issued before it) has finished, so the softmax of
//       tile t may rescale O_t as soon as it sees its next scores.
//       Every mbarrier wait is bounded; a wait that gives up sets the error
//       flag, every role stops, and the MMAs in flight drain before TMEM is
//       released.
#include "decode_common.cuh"
#include "tcgen05.cuh"

#include <math.h>

namespace santa {

constexpr int kPfD = 128;             // head dim
constexpr int kPfRows = 128;          // query rows per tile = keys per KV tile
constexpr int kPfSoftmaxWarps = 16;   // 2 warpgroups per query tile (one per score half)
constexpr int kPfThreads = 32 * (kPfSoftmaxWarps + 2);  // + MMA warp + load warp
constexpr int kPfMmaWarp = kPfSoftmaxWarps;  // the next warp loads K / V^T
constexpr int kPfTile = 32768;        // bytes of one 128 x 128 bf16 tile image
constexpr int kPfHalf = 16384;        // one 64-element half of a tile
constexpr uint32_t kIdesc = umma_idesc_bf16(128, 128);

// byte offset of 16-byte chunk ch (of 16 along the 128-element row) of row r
// in a tile image (K-major, 128-byte swizzle, 8-row atoms 1024 bytes apart)
__host__ __device__ __forceinline__ uint32_t pf_img_off(int r, int ch) {
    return (uint32_t)((ch >> 3) * kPfHalf + (r >> 3) * 1024 + (r & 7) * 128 +
                      (((ch & 7) ^ (r & 7)) << 4));
}

struct PrefillArgs {
    const __nv_bfloat16 *q;     // [B, Hq, T, D]
    const unsigned char *kimg;  // [B, Hkv, n_tiles] 32 KB tile images of K
    const unsigned char *vimg;  // [B, Hkv, n_tiles] 32 KB tile images of V^T
    __nv_bfloat16 *out;         // [B, Hq, T, D]
    float *lse;                 // [B, Hq, T] natural log, or null
    int32_t *err;               // error flag (a bounded wait gave up)
    int B, Hq, Hkv, T, n_tiles, n_pairs;
    float scale_log2;           // scale * log2(e)
    int causal;
};

// 2^x with the MUFU instruction (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, subnormal results flushed to zero); p is rounded to bf16
// right after, so the approximation is far below the output precision
__device__ __forceinline__ float pf_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// Paired fp32 arithmetic (the sm_100 two-lane FP32 instructions: each lane
// rounds as the scalar instruction does) and the three-input maximum.
__device__ __forceinline__ uint64_t pf_pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void pf_unpack2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;\n" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t pf_fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t pf_add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float pf_max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// named barrier over n threads (whole warps) that also ORs a predicate
__device__ __forceinline__ bool bar_red_or(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void bulk_g2s_u32(uint32_t dst, const void *src, uint32_t bytes,
                                             uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(kPfThreads, 1) prefill_fwd_kernel(PrefillArgs a) {
    extern __shared__ __align__(16) unsigned char pf_raw[];
    unsigned char *base = (unsigned char *)(((uintptr_t)pf_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sQ = smem_u32(base);              // Q tile t at sQ + t * kPfTile
    const uint32_t sK = sQ + 2 * kPfTile;            // K stage s at sK + s * kPfTile
    const uint32_t sV = sK + 2 * kPfTile;            // V^T stage s at sV + s * kPfTile
    __shared__ __align__(8) uint64_t bar_k[2], bar_v[2], bar_free[2], bar_s[2], bar_p[2];
    __shared__ __align__(8) uint64_t bar_q, bar_o, bar_drain;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x % (a.B * a.Hq);
    const int pair = a.n_pairs - 1 - blockIdx.x / (a.B * a.Hq);
    const int b = bh / a.Hq, h = bh - b * a.Hq;
    const int kvh = h / (a.Hq / a.Hkv);
    const int qt0 = 2 * pair;
    // KV tiles per query tile (tile 1 may lie past T: its rows are computed
    // on zero queries and never stored)
    const int nj0 = a.causal ? min(qt0 + 1, a.n_tiles) : a.n_tiles;
    const int nj = a.causal ? min(qt0 + 2, a.n_tiles) : a.n_tiles;  // tile 1, >= nj0

    if (warp == kPfMmaWarp) tmem_alloc(smem_u32(&s_tmem), 512);
    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bar_k[s], 1);
            mbar_init(&bar_v[s], 1);
            mbar_init(&bar_free[s], 1);
            mbar_init(&bar_s[s], 1);
            mbar_init(&bar_p[s], 256);
        }
        mbar_init(&bar_q, 512);
        mbar_init(&bar_o, 1);
        mbar_init(&bar_drain, 1);
        s_abort = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPfMmaWarp) tmem_relinquish();
    const uint32_t tmem = s_tmem;

    if (warp < kPfSoftmaxWarps) {
        // ---------------- softmax: tile t, score half hf ----------------
        // warpgroup (t, hf) owns score columns [64 hf, 64 hf + 64) of every
        // row of tile t; the two halves of a tile exchange row maxima through
        // shared memory at a named barrier (id 1 + t) and their row sums once
        // at the end.  The named barriers carry every thread's wait outcome
        // (bar.red.or), so a timed-out wait ends both halves together.
        // row maxima, double-buffered by iteration parity (a half writes
        // buffer j & 1 only after the barrier of iteration j - 1, which the
        // other half passes only after reading it), and the row sums
        __shared__ float s_red[2][2][2][kPfRows], s_l[2][2][kPfRows];
        const int t = warp >> 3, hf = (warp >> 2) & 1;
        const int row = 32 * (warp & 3) + lane;  // TMEM lane = query row in the tile
        const int qtile = qt0 + t;
        const int qpos = qtile * kPfRows + row;
        const int bar_id = 1 + t;
        // this thread's half of its query row into the swizzled Q tile
        {
            const bool ok = qpos < a.T;
            const __nv_bfloat16 *qg =
                a.q + (((int64_t)b * a.Hq + h) * a.T + (ok ? qpos : 0)) * kPfD;
            const uint32_t dst = sQ + t * kPfTile;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int ch = 8 * hf + c;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(
                                 dst + pf_img_off(row, ch)),
                             "l"(qg + ch * 8), "r"(ok ? 16 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            fence_proxy_async_smem();
            mbar_arrive(&bar_q);
        }
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const uint32_t tS = tmem + lane_off + (uint32_t)(t * 128 + 64 * hf);  // my score half
        const uint32_t tO = tmem + lane_off + (uint32_t)(256 + t * 128 + 64 * hf);  // my O half
        const int njt = t ? nj : nj0;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < njt; ++j) {
            bool wok = !s_abort && mbar_wait(&bar_s[t], (uint32_t)(j & 1));
            // the TMEM loads below are warp-collective: the warp goes on only
            // if every lane's wait succeeded
            wok = __all_sync(0xffffffffu, wok);
            tc_fence_after();
            // keys [0, lim) of this tile are visible to this row; only the
            // diagonal tile (causal) and the ragged last tile mask anything
            const int kv0 = j * kPfRows;
            const bool masked = (a.causal && j == qtile) || kv0 + kPfRows > a.T;
            const int lim = (a.causal ? min(a.T, qpos + 1) : a.T) - kv0 - 64 * hf;
            // pass 1: maximum over my 64 scores (eight partial maxima)
            float mp[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mp[e] = -INFINITY;
            if (wok) {
                uint32_t r0[32], r1[32];
                tmem_ld_x32(tS, r0);
                tmem_ld_x32(tS + 32, r1);
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float v0 = i < lim ? __uint_as_float(r0[i]) : -INFINITY;
                        const float v1 = 32 + i < lim ? __uint_as_float(r1[i]) : -INFINITY;
                        mp[i & 7] = pf_max3(mp[i & 7], v0, v1);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        mp[i & 7] = pf_max3(mp[i & 7], __uint_as_float(r0[i]),
                                            __uint_as_float(r1[i]));
                }
            }
            s_red[j & 1][t][hf][row] = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
            // a failed wait joins the barrier's OR so both halves leave together
            if (bar_red_or(bar_id, 256, !wok)) {
                ok = false;
                break;
            }
            const float mx =
                fmaxf(s_red[j & 1][t][0][row], s_red[j & 1][t][1][row]) * a.scale_log2;
            const float m_new = fmaxf(m_used, mx);
            // Lazy rescale: a row's O and l are rescaled only when its maximum
            // grew by more than 8 (log2 units).  The decision is per row, but
            // tcgen05.ld / st are warp-collective (.sync.aligned): a warp in
            // which any row needs it rescales all 32 rows together, the others
            // by 1 (exact).  PV(j-1) of this tile has finished (it was issued
            // before S(j), whose commit this thread waited for).
            const bool grow = m_used != -INFINITY && m_new > m_used + 8.0f;
            float alpha = 1.f;
            if (m_used == -INFINITY) {
                m_used = m_new;
            } else if (grow) {
                alpha = pf_exp2(m_used - m_new);
                m_used = m_new;
                l *= alpha;
            }
            if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t r[32];
                    tmem_ld_x32(tO + 32 * c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    tmem_st_x32(tO + 32 * c, r);
                }
            }
            // pass 2: p = 2^(s * scale - m) as bf16 pairs (two keys per
            // column) over my own first 32 score columns: the P columns of
            // chunk c, [16 c, 16 c + 16), lie below every column still to be read
            const float neg = m_used == -INFINITY ? 0.f : -m_used;
            const uint64_t sc2 = pf_pack2(a.scale_log2, a.scale_log2), ng2 = pf_pack2(neg, neg);
            uint64_t lp[2] = {0ull, 0ull};  // partial sums, two lanes each
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t r[32], pk[16];
                tmem_ld_x32(tS + 32 * c, r);
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (32 * c + i >= lim) r[i] = __float_as_uint(-INFINITY);
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    float x0, x1;
                    pf_unpack2(pf_fma2(pf_pack2(__uint_as_float(r[2 * i]),
                                                __uint_as_float(r[2 * i + 1])), sc2, ng2),
                               x0, x1);
                    const float p0 = pf_exp2(x0), p1 = pf_exp2(x1);
                    lp[i & 1] = pf_add2(lp[i & 1], pf_pack2(p0, p1));
                    pk[i] = pack_bf16(p0, p1);
                }
                tmem_st_x16(tS + 16 * c, pk);
            }
            {
                float s0, s1;
                pf_unpack2(pf_add2(lp[0], lp[1]), s0, s1);
                l += s0 + s1;
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar_p[t]);
        }
        if (!ok) {
            s_abort = 1;
            atomicExch(a.err, 1);
        }
        // ---- epilogue: O / (l of both halves) ----
        const bool eok = ok && !s_abort && mbar_wait(&bar_o, 0);
        s_l[t][hf][row] = l;
        if (!bar_red_or(bar_id, 256, !eok)) {
            tc_fence_after();
            const float lt = s_l[t][0][row] + s_l[t][1][row];
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
            __nv_bfloat16 *og = a.out + (((int64_t)b * a.Hq + h) * a.T + qpos) * kPfD + 64 * hf;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t r[32];
                tmem_ld_x32(tO + 32 * c, r);
                tmem_wait_ld();
                if (qpos < a.T) {
                    uint32_t o[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        o[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv,
                                         __uint_as_float(r[2 * i + 1]) * inv);
                    uint4 *dst = (uint4 *)(og + 32 * c);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                }
            }
            if (a.lse && hf == 0 && qpos < a.T)
                a.lse[((int64_t)b * a.Hq + h) * a.T + qpos] =
                    lt > 0.f ? (m_used + log2f(lt)) * kLn2 : -INFINITY;
        } else {
            s_abort = 1;
            atomicExch(a.err, 1);
        }
    } else if (warp == kPfMmaWarp) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            bool ok = mbar_wait(&bar_q, 0);
            tc_fence_after();
            auto s_mma = [&](int t, int j) -> bool {
                const int st = j & 1;
                if (s_abort || !mbar_wait(&bar_k[st], (uint32_t)((j >> 1) & 1))) return false;
                tc_fence_after();
                const uint32_t q0 = sQ + t * kPfTile, k0 = sK + st * kPfTile;
#pragma unroll
                for (int kk = 0; kk < kPfD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kPfHalf + (kk & 3) * 32;
                    umma_bf16_ss(tmem + t * 128, umma_desc_sw128(q0 + off),
                                 umma_desc_sw128(k0 + off), kIdesc, kk > 0);
                }
                umma_commit(smem_u32(&bar_s[t]));
                return true;
            };
            auto pv_mma = [&](int t, int j) -> bool {
                const int st = j & 1;
                if (s_abort || !mbar_wait(&bar_v[st], (uint32_t)((j >> 1) & 1)) ||
                    !mbar_wait(&bar_p[t], (uint32_t)(j & 1)))
                    return false;
                tc_fence_after();
                const uint32_t v0 = sV + st * kPfTile;
#pragma unroll
                for (int kk = 0; kk < kPfRows / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kPfHalf + (kk & 3) * 32;
                    // P of keys 0-63 in columns [0, 32), of keys 64-127 in
                    // [64, 96): each score half wrote P over its own columns
                    umma_bf16_ts(tmem + 256 + t * 128,
                                 tmem + t * 128 + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8),
                                 umma_desc_sw128(v0 + off), kIdesc, (j > 0 || kk > 0) ? 1u : 0u);
                }
                return true;
            };
            if (ok && nj0 > 0) ok = s_mma(0, 0);
            if (ok) ok = s_mma(1, 0);
            for (int j = 0; ok && j < nj; ++j) {
                if (j < nj0) {
                    ok = pv_mma(0, j);
                    if (ok && j + 1 < nj0) ok = s_mma(0, j + 1);
                }
                if (ok) ok = pv_mma(1, j);
                if (ok) umma_commit(smem_u32(&bar_free[j & 1]));  // stage j & 1 read
                if (ok && j + 1 < nj) ok = s_mma(1, j + 1);
            }
            if (ok) {
                umma_commit(smem_u32(&bar_o));
            } else {
                s_abort = 1;
                atomicExch(a.err, 1);
            }
            // every MMA issued so far has finished before TMEM is released
            umma_commit(smem_u32(&bar_drain));
            if (!mbar_wait(&bar_drain, 0)) atomicExch(a.err, 1);
        }
    } else {
        // ---------------- K / V^T loads ----------------
        if (lane == 0) {
            const size_t tile0 = ((size_t)b * a.Hkv + kvh) * a.n_tiles;
            int issued = 0;
            for (int j = 0; j < nj; ++j) {
                const int st = j & 1;
                if (j >= 2 && (s_abort || !mbar_wait(&bar_free[st], (uint32_t)(((j >> 1) - 1) & 1)))) {
                    s_abort = 1;
                    atomicExch(a.err, 1);
                    break;
                }
                mbar_arrive_expect_tx(&bar_k[st], kPfTile);
                bulk_g2s_u32(sK + st * kPfTile, a.kimg + (tile0 + j) * kPfTile, kPfTile, &bar_k[st]);
                mbar_arrive_expect_tx(&bar_v[st], kPfTile);
                bulk_g2s_u32(sV + st * kPfTile, a.vimg + (tile0 + j) * kPfTile, kPfTile, &bar_v[st]);
                issued = j + 1;
            }
            // the last copies into each stage have landed before the CTA ends
            for (int j = max(0, issued - 2); j < issued; ++j) {
                mbar_wait(&bar_k[j & 1], (uint32_t)((j >> 1) & 1));
                mbar_wait(&bar_v[j & 1], (uint32_t)((j >> 1) & 1));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPfMmaWarp) tmem_dealloc(tmem, 512);
}

// K and V (tokens [0, T) of a contiguous [B, Hkv, cap, D] cache or of paged
// pools, rows through cache_row) -> the tile images of K and V^T
// (pf_img_off layout, zeros past T).  One CTA per (128-key tile, b * kv head).
__global__ void __launch_bounds__(256) prefill_image_kernel(const __nv_bfloat16 *k,
                                                            const __nv_bfloat16 *v,
                                                            unsigned char *kimg,
                                                            unsigned char *vimg, int T,
                                                            int n_tiles, SantaGeometry geo) {
    __shared__ __align__(16) __nv_bfloat16 vs[kPfRows][kPfD + 8];
    const int j = blockIdx.x, bh = blockIdx.y, tid = threadIdx.x;
    unsigned char *ki = kimg + ((size_t)bh * n_tiles + j) * kPfTile;
    unsigned char *vi = vimg + ((size_t)bh * n_tiles + j) * kPfTile;
    for (int idx = tid; idx < kPfRows * 16; idx += 256) {
        const int r = idx >> 4, ch = idx & 15;
        const int t = j * kPfRows + r;
        const bool ok = t < T;
        const int64_t src = ok ? cache_row(geo, bh, t) * kPfD + ch * 8 : 0;
        const uint4 kv = ok ? *(const uint4 *)(k + src) : make_uint4(0, 0, 0, 0);
        *(uint4 *)(ki + pf_img_off(r, ch)) = kv;
        const uint4 vv = ok ? *(const uint4 *)(v + src) : make_uint4(0, 0, 0, 0);
        *(uint4 *)(&vs[r][ch * 8]) = vv;
    }
    __syncthreads();
    // V^T: row = dim d, 16-byte chunk ch = keys 8 ch .. 8 ch + 7
    for (int idx = tid; idx < kPfD * 16; idx += 256) {
        const int d = idx & (kPfD - 1), ch = idx >> 7;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __nv_bfloat16 lo = vs[8 * ch + 2 * e][d], hi = vs[8 * ch + 2 * e + 1][d];
            w[e] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
        }
        *(uint4 *)(vi + pf_img_off(d, ch)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace santa

using namespace santa;

static int check_prefill(const SantaPrefillShape *s) {
    if (!s) return SANTA_ERR_INVALID_ARGUMENT;
    if (s->batch <= 0 || s->num_query_heads <= 0 || s->num_kv_heads <= 0 || s->seq_len <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (s->num_query_heads % s->num_kv_heads) return SANTA_ERR_INVALID_ARGUMENT;
    if (s->head_dim != kPfD) return SANTA_ERR_UNSUPPORTED;
    if (!(s->scale > 0.f)) return SANTA_ERR_INVALID_ARGUMENT;
    if (s->kv_capacity && s->kv_capacity < s->seq_len) return SANTA_ERR_INVALID_ARGUMENT;
    return SANTA_OK;
}

extern "C" int santa_prefill_workspace_bytes(const SantaPrefillShape *shape, size_t *bytes) {
    int st = check_prefill(shape);
    if (st) return st;
    if (!bytes) return SANTA_ERR_INVALID_ARGUMENT;
    const size_t n_tiles = ((size_t)shape->seq_len + kPfRows - 1) / kPfRows;
    *bytes = 2 * (size_t)shape->batch * shape->num_kv_heads * n_tiles * kPfTile + 256;
    return SANTA_OK;
}

// Both entry points: geo describes where token t of (b, kv head) lives.
static int prefill(const SantaPrefillShape *shape, const SantaGeometry &geo, const void *q,
                   const void *k, const void *v, void *out, float *lse, int32_t *error_flag,
                   void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!q || !k || !v || !out || !error_flag) return SANTA_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    santa_prefill_workspace_bytes(shape, &need);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out | (uintptr_t)workspace) & 15)
        return SANTA_ERR_UNSUPPORTED;
    const int T = shape->seq_len;
    const int n_tiles = (T + kPfRows - 1) / kPfRows;
    const int BHkv = shape->batch * shape->num_kv_heads;
    unsigned char *kimg = (unsigned char *)workspace;
    unsigned char *vimg = kimg + (size_t)BHkv * n_tiles * kPfTile;
    prefill_image_kernel<<<dim3(n_tiles, BHkv), 256, 0, stream>>>(
        (const __nv_bfloat16 *)k, (const __nv_bfloat16 *)v, kimg, vimg, T, n_tiles, geo);
    SANTA_LAUNCH_CHECK();
    PrefillArgs a;
    a.q = (const __nv_bfloat16 *)q;
    a.kimg = kimg;
    a.vimg = vimg;
    a.out = (__nv_bfloat16 *)out;
    a.lse = lse;
    a.err = error_flag;
    a.B = shape->batch;
    a.Hq = shape->num_query_heads;
    a.Hkv = shape->num_kv_heads;
    a.T = T;
    a.n_tiles = n_tiles;
    a.n_pairs = (n_tiles + 1) / 2;
    a.scale_log2 = shape->scale * 1.4426950408889634f;
    a.causal = shape->causal ? 1 : 0;
    const size_t smem = 6 * (size_t)kPfTile + 1024;
    if (int st = ensure_dyn_smem((const void *)prefill_fwd_kernel, smem)) return st;
    const unsigned grid = (unsigned)a.n_pairs * a.B * a.Hq;
    prefill_fwd_kernel<<<grid, kPfThreads, smem, stream>>>(a);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_prefill(const SantaPrefillShape *shape, const void *q, const void *k,
                             const void *v, void *out, float *lse, int32_t *error_flag,
                             void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    int st = check_prefill(shape);
    if (st) return st;
    SantaGeometry geo = {};
    geo.batch = shape->batch;
    geo.num_kv_heads = shape->num_kv_heads;
    geo.capacity = shape->kv_capacity ? shape->kv_capacity : shape->seq_len;
    return prefill(shape, geo, q, k, v, out, lse, error_flag, workspace, workspace_bytes, stream);
}

extern "C" int santa_prefill_paged(const SantaPrefillShape *shape, const void *q,
                                   const void *key_pool, const void *value_pool,
                                   const int32_t *block_table, int32_t page_size,
                                   int32_t max_pages, int32_t num_pages, void *out, float *lse,
                                   int32_t *error_flag, void *workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    int st = check_prefill(shape);
    if (st) return st;
    if (!block_table || page_size <= 0 || (page_size & (page_size - 1)) || max_pages <= 0 ||
        num_pages <= 0 || (int64_t)max_pages * page_size < shape->seq_len ||
        (int64_t)max_pages * page_size > INT32_MAX)
        return SANTA_ERR_INVALID_ARGUMENT;
    SantaGeometry geo = {};
    geo.batch = shape->batch;
    geo.num_kv_heads = shape->num_kv_heads;
    geo.capacity = max_pages * page_size;
    geo.block_table = block_table;
    geo.page_size = page_size;
    geo.max_pages = max_pages;
    geo.num_pages = num_pages;
    return prefill(shape, geo, q, key_pool, value_pool, out, lse, error_flag, workspace,
                   workspace_bytes, stream);
}
