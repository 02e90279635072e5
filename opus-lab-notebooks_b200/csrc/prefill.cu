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
// Kernel (one CTA of 8 warps per (128-query tile, query head); the heaviest
// causal tiles are scheduled first):
//   * Q, K and V^T tiles live in shared memory in the canonical K-major
//     128-byte-swizzle layout (two 64-element halves of the 128 dims; rows in
//     1024-byte atoms of 8), so every MMA operand uses one descriptor form.
//     V is transposed once into the workspace so that the P.V product's B
//     operand (K = keys, N = dims) is K-major too.
//   * S = Q K^T: 8 tcgen05.mma (M=128, N=128, K=16) into TMEM columns
//     [0, 128); O += P V^T: 8 more into columns [128, 256).  One thread issues
//     them and commits to an mbarrier; every wait is bounded.
//   * Softmax: warp w reads TMEM lanes 32*(w%4).. (its 32 query rows) and
//     columns 64*(w/4).. (half of the keys) with tcgen05.ld, so a query row
//     is owned by two threads that exchange their row maxima through shared
//     memory.  The running maximum is updated lazily: O (in TMEM) and l are
//     rescaled only when the maximum grows by more than 8 (log2 units), so
//     p <= 2^8 and most tiles skip the TMEM round trip.  P is written to
//     shared memory as bf16 in the same swizzled layout (A operand of P.V).
//   * K and V^T tiles are double-buffered with 16-byte cp.async; the next K
//     tile streams in during the S MMA and softmax, the next V^T tile during
//     the P.V MMA.
#include "decode_common.cuh"
#include "tcgen05.cuh"

#include <math.h>

namespace santa {

constexpr int kPfD = 128;            // head dim
constexpr int kPfRows = 128;         // query rows per CTA = keys per tile
constexpr int kPfThreads = 256;
constexpr int kPfTile = 32768;       // bytes of one 128 x 128 bf16 tile
constexpr int kPfHalf = 16384;       // one 64-element half of a tile
constexpr uint32_t kIdesc = umma_idesc_bf16(128, 128);

struct PrefillArgs {
    const __nv_bfloat16 *q;   // [B, Hq, T, D]
    const __nv_bfloat16 *k;   // [B, Hkv, T, D]
    const __nv_bfloat16 *vt;  // [B, Hkv, D, T] (transposed V)
    __nv_bfloat16 *out;       // [B, Hq, T, D]
    float *lse;               // [B, Hq, T] natural log, or null
    int32_t *err;             // error flag (a bounded wait gave up)
    int B, Hq, Hkv, T, n_tiles;
    int64_t cap;              // tokens between consecutive (b, kv head) blocks of k
    int Tp;                   // row stride of V^T: T rounded up to a multiple of 8
    float scale_log2;         // scale * log2(e)
    int causal;
};

// one 128-row x 128-column bf16 tile from a row-major matrix into the
// swizzled K-major layout; rows >= rows_ok and columns >= cols_ok read as 0
__device__ __forceinline__ void pf_load_tile(uint32_t dst, const __nv_bfloat16 *src, int64_t ld,
                                             int rows_ok, int cols_ok, int tid) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
        const int ci = tid + it * kPfThreads;  // 16-byte chunk: 16 per row
        const int row = ci >> 4, ch = ci & 15;
        const int half = ch >> 3, c = ch & 7;
        const uint32_t d = dst + half * kPfHalf + (row >> 3) * 1024 + (row & 7) * 128 +
                           ((c ^ (row & 7)) << 4);
        const bool ok = row < rows_ok && ch * 8 < cols_ok;
        const __nv_bfloat16 *s = src + (ok ? (int64_t)row * ld + ch * 8 : 0);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(s),
                     "r"(ok ? 16 : 0)
                     : "memory");
    }
}

__device__ __forceinline__ void pf_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pf_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kPfThreads, 1) prefill_fwd_kernel(PrefillArgs a) {
    extern __shared__ __align__(16) unsigned char pf_raw[];
    unsigned char *base = (unsigned char *)(((uintptr_t)pf_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sQ = smem_u32(base);
    const uint32_t sK0 = sQ + kPfTile, sV0 = sQ + 3 * kPfTile, sP = sQ + 5 * kPfTile;
    __shared__ __align__(8) uint64_t mbar[2];  // 0: S done, 1: P.V done
    __shared__ uint32_t s_tmem;
    __shared__ float red_m[kPfRows][2], red_l[kPfRows][2];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = 32 * (warp & 3) + lane;   // query row of this thread (TMEM lane)
    const int hv = warp >> 2;                  // key / dim half of this thread
    const int bh = blockIdx.x % (a.B * a.Hq);
    const int tile = a.n_tiles - 1 - blockIdx.x / (a.B * a.Hq);
    const int b = bh / a.Hq, h = bh - b * a.Hq;
    const int kvh = h / (a.Hq / a.Hkv);
    const int q0 = tile * kPfRows;
    const int nj = a.causal ? tile + 1 : a.n_tiles;

    if (warp == 0) tmem_alloc(smem_u32(&s_tmem), 256);
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_relinquish();
    const uint32_t tS = s_tmem, tO = s_tmem + 128;
    const uint32_t tlane = (uint32_t)(32 * (warp & 3)) << 16;

    const __nv_bfloat16 *qg = a.q + (((int64_t)b * a.Hq + h) * a.T + q0) * kPfD;
    const __nv_bfloat16 *kg = a.k + ((int64_t)b * a.Hkv + kvh) * a.cap * kPfD;
    const __nv_bfloat16 *vg = a.vt + ((int64_t)b * a.Hkv + kvh) * kPfD * a.Tp;

    // prologue: Q, K_0 | V_0
    pf_load_tile(sQ, qg, kPfD, min(kPfRows, a.T - q0), kPfD, tid);
    pf_load_tile(sK0, kg, kPfD, min(kPfRows, a.T), kPfD, tid);
    pf_commit();
    pf_load_tile(sV0, vg, a.Tp, kPfD, min(kPfRows, a.T), tid);
    pf_commit();

    const int qpos = q0 + row;
    float m_used = -INFINITY, l_part = 0.f;
    bool failed = false;  // block-uniform: decided at block barriers only
    int j_fail = 0, n_pv = 0;
    for (int j = 0; j < nj; ++j) {
        const int buf = j & 1;
        const int kv0 = j * kPfRows;
        // K_j (and Q) landed; groups after it: V_j
        pf_wait<1>();
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sK = sK0 + buf * kPfTile;
#pragma unroll
            for (int kk = 0; kk < kPfD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kPfHalf + (kk & 3) * 32;
                umma_bf16_ss(tS, umma_desc_sw128(sQ + off), umma_desc_sw128(sK + off), kIdesc,
                             kk > 0);
            }
            umma_commit(smem_u32(&mbar[0]));
        }
        // prefetch K_{j+1} into the other buffer (its S MMA finished last iteration)
        if (j + 1 < nj)
            pf_load_tile(sK0 + (buf ^ 1) * kPfTile, kg + (int64_t)(kv0 + kPfRows) * kPfD, kPfD,
                         min(kPfRows, a.T - kv0 - kPfRows), kPfD, tid);
        pf_commit();

        const bool ok_s = mbar_wait(&mbar[0], j & 1);
        tc_fence_after();
        // ---- S row: 64 keys of this thread's half ----
        float s[64];
        {
            uint32_t r[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                tmem_ld_x16(tS + tlane + 64 * hv + 16 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) s[16 * c + i] = __uint_as_float(r[i]);
            }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            const int kpos = kv0 + 64 * hv + i;
            const bool on = kpos < a.T && (!a.causal || kpos <= qpos);
            s[i] = on ? s[i] * a.scale_log2 : -INFINITY;
            mx = fmaxf(mx, s[i]);
        }
        red_m[row][hv] = mx;
        tc_fence_before();
        if (__syncthreads_or(!ok_s)) {
            failed = true;
            j_fail = j;
            break;
        }
        const float m_tile = fmaxf(red_m[row][0], red_m[row][1]);
        const float m_new = fmaxf(m_used, m_tile);
        float alpha = 1.f;
        bool rescale = false;
        if (m_used == -INFINITY) {
            m_used = m_new;
        } else if (m_new > m_used + 8.0f) {
            alpha = exp2f(m_used - m_new);
            m_used = m_new;
            rescale = true;
        }
        uint32_t pk[32];
        float lsum = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const float p0 = m_used == -INFINITY ? 0.f : exp2f(s[2 * i] - m_used);
            const float p1 = m_used == -INFINITY ? 0.f : exp2f(s[2 * i + 1] - m_used);
            lsum += p0 + p1;
            pk[i] = pack_bf16(p0, p1);
        }
        l_part = l_part * alpha + lsum;

        // the previous P.V MMA has read P and V_{j-1}, and O is settled
        const bool ok_o = j == 0 || mbar_wait(&mbar[1], (j - 1) & 1);
        tc_fence_after();
        // prefetch V_{j+1} into the buffer V_{j-1} used
        if (j + 1 < nj && ok_o)
            pf_load_tile(sV0 + (buf ^ 1) * kPfTile, vg + kv0 + kPfRows, a.Tp, kPfD,
                         min(kPfRows, a.T - kv0 - kPfRows), tid);
        pf_commit();
        if (rescale && j > 0 && ok_o) {
            uint32_t r[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t ta = tO + tlane + 64 * hv + 16 * c;
                tmem_ld_x16(ta, r);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                tmem_st_x16(ta, r);
            }
            tmem_wait_st();
        }
        // P (bf16) -> swizzled A operand, keys 64*hv .. 64*hv+63 = half hv
        if (ok_o) {
            const uint32_t prow = sP + hv * kPfHalf + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t d = prow + ((c ^ (row & 7)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(d),
                             "r"(pk[4 * c]), "r"(pk[4 * c + 1]), "r"(pk[4 * c + 2]),
                             "r"(pk[4 * c + 3])
                             : "memory");
            }
        }
        // V_j landed; groups after it: K_{j+1}, V_{j+1}
        pf_wait<2>();
        fence_proxy_async_smem();
        tc_fence_before();
        if (__syncthreads_or(!ok_o)) {
            failed = true;
            j_fail = j;
            break;
        }
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sV = sV0 + buf * kPfTile;
#pragma unroll
            for (int kk = 0; kk < kPfRows / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kPfHalf + (kk & 3) * 32;
                umma_bf16_ss(tO, umma_desc_sw128(sP + off), umma_desc_sw128(sV + off), kIdesc,
                             (j > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(smem_u32(&mbar[1]));
        }
        n_pv = j + 1;
    }
    pf_wait<0>();
    if (!failed && nj > 0) {
        const bool ok = mbar_wait(&mbar[1], (nj - 1) & 1);
        tc_fence_after();
        if (__syncthreads_or(!ok)) {
            failed = true;
            j_fail = nj;
        }
    }
    if (failed) {
        // record it, and let the MMAs already issued finish (bounded) before
        // TMEM is released
        if (tid == 0) atomicExch(a.err, 1);
        if (j_fail < nj) mbar_wait(&mbar[0], j_fail & 1);
        if (n_pv > 0) mbar_wait(&mbar[1], (n_pv - 1) & 1);
    }
    // ---- epilogue: O / l ----
    red_l[row][hv] = l_part;
    tc_fence_after();
    __syncthreads();
    if (!failed) {
        const float l = red_l[row][0] + red_l[row][1];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint32_t r[16];
        __nv_bfloat16 *og = a.out + (((int64_t)b * a.Hq + h) * a.T + qpos) * kPfD + 64 * hv;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            tmem_ld_x16(tO + tlane + 64 * hv + 16 * c, r);
            tmem_wait_ld();
            if (qpos < a.T) {
                uint32_t o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    o[i] = pack_bf16(__uint_as_float(r[2 * i]) * inv,
                                     __uint_as_float(r[2 * i + 1]) * inv);
                uint4 *dst = (uint4 *)(og + 16 * c);
                dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
        }
        if (a.lse && hv == 0 && qpos < a.T)
            a.lse[((int64_t)b * a.Hq + h) * a.T + qpos] =
                l > 0.f ? (m_used + log2f(l)) * kLn2 : -INFINITY;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tS, 256);
}

// V [B, Hkv, cap, D] (tokens [0, T)) -> V^T [B, Hkv, D, Tp], 32 x 32 tiles;
// columns [T, Tp) are zero (a partial key tile's masked columns multiply them)
__global__ void prefill_transpose_v_kernel(const __nv_bfloat16 *v, __nv_bfloat16 *vt, int T,
                                           int Tp, int D, int64_t cap) {
    __shared__ __nv_bfloat16 tile[32][33];
    const int64_t mat = blockIdx.z;
    const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
    const __nv_bfloat16 *src = v + mat * cap * D;
    __nv_bfloat16 *dst = vt + mat * (int64_t)Tp * D;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int t = t0 + i, d = d0 + threadIdx.x;
        tile[i][threadIdx.x] = (t < T && d < D) ? src[(int64_t)t * D + d] : __float2bfloat16(0.f);
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int d = d0 + i, t = t0 + threadIdx.x;
        if (t < Tp && d < D) dst[(int64_t)d * Tp + t] = tile[threadIdx.x][i];
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
    const int64_t Tp = ((int64_t)shape->seq_len + 7) / 8 * 8;  // 16-byte rows of V^T
    *bytes = (size_t)shape->batch * shape->num_kv_heads * Tp * shape->head_dim * 2 + 256;
    return SANTA_OK;
}

extern "C" int santa_prefill(const SantaPrefillShape *shape, const void *q, const void *k,
                             const void *v, void *out, float *lse, int32_t *error_flag,
                             void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    int st = check_prefill(shape);
    if (st) return st;
    if (!q || !k || !v || !out || !error_flag) return SANTA_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    santa_prefill_workspace_bytes(shape, &need);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out | (uintptr_t)workspace) & 15)
        return SANTA_ERR_UNSUPPORTED;
    const int T = shape->seq_len, D = shape->head_dim;
    __nv_bfloat16 *vt = (__nv_bfloat16 *)workspace;
    const int Tp = (T + 7) / 8 * 8;
    dim3 tg((Tp + 31) / 32, (D + 31) / 32, shape->batch * shape->num_kv_heads);
    const int64_t cap = shape->kv_capacity ? shape->kv_capacity : T;
    prefill_transpose_v_kernel<<<tg, dim3(32, 8), 0, stream>>>((const __nv_bfloat16 *)v, vt, T,
                                                                Tp, D, cap);
    SANTA_LAUNCH_CHECK();
    PrefillArgs a;
    a.q = (const __nv_bfloat16 *)q;
    a.k = (const __nv_bfloat16 *)k;
    a.vt = vt;
    a.out = (__nv_bfloat16 *)out;
    a.lse = lse;
    a.err = error_flag;
    a.B = shape->batch;
    a.Hq = shape->num_query_heads;
    a.Hkv = shape->num_kv_heads;
    a.T = T;
    a.cap = cap;
    a.Tp = Tp;
    a.n_tiles = (T + kPfRows - 1) / kPfRows;
    a.scale_log2 = shape->scale * 1.4426950408889634f;
    a.causal = shape->causal ? 1 : 0;
    const size_t smem = 6 * (size_t)kPfTile + 1024;
    static bool attr = false;
    if (!attr) {
        SANTA_CUDA_CHECK(cudaFuncSetAttribute(prefill_fwd_kernel,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem));
        attr = true;
    }
    const unsigned grid = (unsigned)a.n_tiles * a.B * a.Hq;
    prefill_fwd_kernel<<<grid, kPfThreads, smem, stream>>>(a);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}
