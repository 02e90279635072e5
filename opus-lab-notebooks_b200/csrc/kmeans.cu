// MiniBatchKMeans kernels (santapp_ruler/attention/minibatch_kmeans.py).
//
// The host keeps the reference's control flow and its numpy RandomState
// stream (batch draws, reassignment draws, early stopping); every
// data-dependent computation runs here, under the defined arithmetic the
// oracle restates (oracle/santa_oracle.c), so labels and centres match it
// bit for bit:
//
//   dot(a, b)    sequential fmaf chain over the features, ascending
//   dist2        max(0, fl32(fl32(|x|^2 + |c|^2) - 2 dot))     (:58-66)
//   argmin       lowest centre index on ties                      (:68-71)
//   inertia, potentials, prefix sums
//                sums of non-negative fp32 values in exact Q64.64 fixed
//                point (order independent, so parallel reductions agree
//                with the sequential oracle), returned as fl32(fl64(sum))
//   batch sums   sequential fp32 adds in ascending batch order per
//                (cluster, feature) (index_add_, :226-233)
//   new centre   fl32(fl32(fl32(c * n) + sum) / fl32(n + bc))     (:234-239)
//
// Kernels:
//   kmeans_sqnorm_kernel        |x|^2 per row
//   kmeans_assign_kernel        32 rows x all centres per CTA: centres staged
//                               through shared memory in 64-row chunks, each
//                               thread runs 2 x 4 independent fmaf chains
//                               (float4 loads, padded pitch: conflict-free)
//   kmeans_partition_kernel     stable counting sort of the batch labels
//   kmeans_update_kernel        one CTA per cluster, one thread per feature
//   kmeans_reassign_kernel      centre <- batch row, count <- given value
//   kpp_*                       greedy k-means++ (:73-126): one fixed-point
//                               scan + search launch (one CTA of 1024
//                               threads) and one candidate launch per new
//                               centre, no host round trip.  (One cooperative
//                               launch with grid barriers between the phases
//                               measured slower: its one-CTA scan phase ran
//                               on the persistent grid's 256-thread CTA.)
#include "common.cuh"

#include <math.h>

namespace santa {

typedef unsigned __int128 u128;

constexpr int kKmMaxDim = 512;
constexpr int kKmMaxClusters = 4096;
constexpr int kKmMaxTrials = 16;

__device__ __forceinline__ u128 fx_of(float v) {
    const uint32_t bits = __float_as_uint(v);
    if (bits & 0x80000000u) return 0;  // negative or -0: treated as 0
    const uint32_t ex = (bits >> 23) & 0xffu;
    uint32_t mant = bits & 0x7fffffu;
    int e2;
    if (ex == 0) {
        e2 = -149;
    } else {
        mant |= 0x800000u;
        e2 = (int)ex - 150;
    }
    if (mant == 0) return 0;
    int sh = e2 + 64;
    if (sh >= 0) {
        if (sh > 103) sh = 103;
        return ((u128)mant) << sh;
    }
    if (sh <= -32) return 0;
    return (u128)(mant >> (-sh));
}

__device__ __forceinline__ float fx_to_float(u128 s) {
    const unsigned long long hi = (unsigned long long)(s >> 64);
    const unsigned long long lo = (unsigned long long)s;
    const double d = __dadd_rn(__ull2double_rn(hi), __dmul_rn(__ull2double_rn(lo), 0x1p-64));
    return __double2float_rn(d);
}

__device__ __forceinline__ float dist2_def(float xx, float cc, float dt) {
    const float s = __fadd_rn(xx, cc);
    const float r = __fsub_rn(s, __fmul_rn(2.0f, dt));
    return r > 0.0f ? r : 0.0f;
}

__device__ __forceinline__ u128 shfl_xor_u128(u128 v, int o) {
    const unsigned long long lo = __shfl_xor_sync(0xffffffffu, (unsigned long long)v, o);
    const unsigned long long hi = __shfl_xor_sync(0xffffffffu, (unsigned long long)(v >> 64), o);
    return ((u128)hi << 64) | lo;
}

__device__ __forceinline__ u128 warp_sum_u128(u128 v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += shfl_xor_u128(v, o);
    return v;
}

// exact 128-bit add into two 64-bit words (lo, hi)
__device__ __forceinline__ void atomic_add_u128(unsigned long long *p, u128 v) {
    const unsigned long long lo = (unsigned long long)v;
    unsigned long long hi = (unsigned long long)(v >> 64);
    if (lo) {
        const unsigned long long old = atomicAdd(p, lo);
        if (old + lo < old) hi += 1ull;
    }
    if (hi) atomicAdd(p + 1, hi);
}

// sum over the block (every thread passes its value); thread 0 adds it to p
template <int NT>
__device__ void block_add_u128(u128 v, unsigned long long *p, u128 *sw) {
    v = warp_sum_u128(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sw[warp] = v;
    __syncthreads();
    if (warp == 0) {
        u128 s = lane < NT / 32 ? sw[lane] : (u128)0;
        s = warp_sum_u128(s);
        if (lane == 0 && s) atomic_add_u128(p, s);
    }
    __syncthreads();
}

__device__ __forceinline__ int64_t row_of(const int64_t *rows, int64_t i) {
    return rows ? rows[i] : i;
}

// ---------------------------------------------------------------------------
// |x_i|^2
// ---------------------------------------------------------------------------
__global__ void kmeans_sqnorm_kernel(const float *x, int64_t n, int d, float *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float *xi = x + i * d;
    float acc = 0.0f;
    if ((d & 3) == 0 && ((uintptr_t)x & 15) == 0) {
        const float4 *x4 = (const float4 *)xi;
        for (int t = 0; t < d / 4; ++t) {
            const float4 v = x4[t];
            acc = fmaf(v.x, v.x, acc);
            acc = fmaf(v.y, v.y, acc);
            acc = fmaf(v.z, v.z, acc);
            acc = fmaf(v.w, v.w, acc);
        }
    } else {
        for (int t = 0; t < d; ++t) acc = fmaf(xi[t], xi[t], acc);
    }
    out[i] = acc;
}

// ---------------------------------------------------------------------------
// nearest centre (minibatch_kmeans.py:58-71)
// ---------------------------------------------------------------------------
constexpr int kAsRows = 32;     // rows per CTA
constexpr int kAsCent = 64;     // centres per shared-memory chunk
constexpr int kAsThreads = 256; // 16 row groups x 16 centre groups

__global__ void __launch_bounds__(kAsThreads) kmeans_assign_kernel(
    const float *x, const int64_t *rows, const float *xx, int64_t n, int d, const float *centers,
    const float *cc, int k, int32_t *labels, float *min_dist, unsigned long long *inertia_fx) {
    extern __shared__ __align__(16) float km_smem[];
    const int P = d + 4;  // padded pitch (floats)
    float *xs = km_smem;                   // [kAsRows][P]
    float *cs = xs + kAsRows * P;          // [kAsCent][P]
    float *ccs = cs + kAsCent * P;         // [kAsCent]
    __shared__ u128 sw[kAsThreads / 32];
    const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
    const int64_t r0 = (int64_t)blockIdx.x * kAsRows;
    const int d4 = d / 4;

    for (int i = tid; i < kAsRows * d4; i += kAsThreads) {
        const int r = i / d4, t = i - r * d4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 + r < n) v = ((const float4 *)(x + row_of(rows, r0 + r) * d))[t];
        *(float4 *)(xs + r * P + 4 * t) = v;
    }
    float xxr[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t r = r0 + rg + 16 * i;
        xxr[i] = r < n ? xx[row_of(rows, r)] : 0.f;
    }
    float best[2] = {INFINITY, INFINITY};
    int bestj[2] = {0, 0};
    for (int c0 = 0; c0 < k; c0 += kAsCent) {
        __syncthreads();  // previous chunk consumed (and the row tile written)
        for (int i = tid; i < kAsCent * d4; i += kAsThreads) {
            const int j = i / d4, t = i - j * d4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + j < k) v = ((const float4 *)(centers + (int64_t)(c0 + j) * d))[t];
            *(float4 *)(cs + j * P + 4 * t) = v;
        }
        for (int j = tid; j < kAsCent; j += kAsThreads) ccs[j] = c0 + j < k ? cc[c0 + j] : 0.f;
        __syncthreads();
        float acc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.f;
        const float *xa = xs + rg * P, *xb = xs + (rg + 16) * P;
        for (int t = 0; t < d; t += 4) {
            const float4 a = *(const float4 *)(xa + t), b = *(const float4 *)(xb + t);
            float4 c[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) c[jj] = *(const float4 *)(cs + (cg + 16 * jj) * P + t);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                acc[0][jj] = fmaf(a.x, c[jj].x, acc[0][jj]);
                acc[0][jj] = fmaf(a.y, c[jj].y, acc[0][jj]);
                acc[0][jj] = fmaf(a.z, c[jj].z, acc[0][jj]);
                acc[0][jj] = fmaf(a.w, c[jj].w, acc[0][jj]);
                acc[1][jj] = fmaf(b.x, c[jj].x, acc[1][jj]);
                acc[1][jj] = fmaf(b.y, c[jj].y, acc[1][jj]);
                acc[1][jj] = fmaf(b.z, c[jj].z, acc[1][jj]);
                acc[1][jj] = fmaf(b.w, c[jj].w, acc[1][jj]);
            }
        }
        // centres visited in ascending index inside a thread: strict < keeps the lowest
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = c0 + cg + 16 * jj;
            if (j < k) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float v = dist2_def(xxr[i], ccs[cg + 16 * jj], acc[i][jj]);
                    if (v < best[i]) {
                        best[i] = v;
                        bestj[i] = j;
                    }
                }
            }
        }
    }
    // across the 16 centre groups of a row (lanes of one half-warp)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best[i], o);
            const int oj = __shfl_xor_sync(0xffffffffu, bestj[i], o);
            if (ov < best[i] || (ov == best[i] && oj < bestj[i])) {
                best[i] = ov;
                bestj[i] = oj;
            }
        }
    }
    u128 fx = 0;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t r = r0 + rg + 16 * i;
        if (cg == 0 && r < n) {
            if (labels) labels[r] = bestj[i];
            if (min_dist) min_dist[r] = best[i];
            fx += fx_of(best[i]);
        }
    }
    if (inertia_fx) block_add_u128<kAsThreads>(fx, inertia_fx, sw);
}

// ---------------------------------------------------------------------------
// mini-batch centre update (minibatch_kmeans.py:226-239)
// ---------------------------------------------------------------------------
constexpr int kPartThreads = 1024;

// counts, starts and the members of every cluster in ascending batch order
__global__ void __launch_bounds__(kPartThreads) kmeans_partition_kernel(
    const int32_t *labels, int64_t nb, int k, int32_t *bcount, int32_t *bstart,
    int32_t *members) {
    extern __shared__ int part_smem[];
    int *cnt = part_smem;        // [k]
    int *fill = cnt + k;         // [k]
    __shared__ int sw[33];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int g = tid; g < k; g += kPartThreads) {
        cnt[g] = 0;
        fill[g] = 0;
    }
    __syncthreads();
    for (int64_t i = tid; i < nb; i += kPartThreads) {
        const int l = labels[i];
        if (l >= 0 && l < k) atomicAdd(&cnt[l], 1);  // labels outside [0, k) are ignored
    }
    __syncthreads();
    // exclusive scan of cnt -> bstart (k <= 4096: 4 per thread at most)
    const int per = (k + kPartThreads - 1) / kPartThreads;
    int local = 0;
    for (int j = 0; j < per; ++j) {
        const int g = tid * per + j;
        if (g < k) local += cnt[g];
    }
    int x = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sw[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = sw[lane];
        int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sw[lane] = s - w;
    }
    __syncthreads();
    int run = sw[warp] + x - local;
    for (int j = 0; j < per; ++j) {
        const int g = tid * per + j;
        if (g < k) {
            bstart[g] = run;
            bcount[g] = cnt[g];
            run += cnt[g];
        }
    }
    __syncthreads();
    // stable scatter: one warp walks the batch in order, 32 rows at a time
    if (warp == 0) {
        for (int64_t base = 0; base < nb; base += 32) {
            const int64_t i = base + lane;
            const int l0 = i < nb ? labels[i] : -1;
            const bool on = l0 >= 0 && l0 < k;
            const unsigned act = __ballot_sync(0xffffffffu, on);
            const int l = on ? l0 : -1;
            const unsigned peers = __match_any_sync(0xffffffffu, l);
            const int rank = __popc(peers & act & ((1u << lane) - 1u));
            int f = 0;
            if (on) f = fill[l];
            __syncwarp();
            if (on) {
                members[bstart[l] + f + rank] = (int32_t)i;
                if ((peers & act & ((1u << lane) - 1u)) == 0u) fill[l] = f + __popc(peers & act);
            }
            __syncwarp();
        }
    }
}

__global__ void kmeans_update_kernel(const float *x, const int64_t *rows, int d,
                                     const int32_t *bcount, const int32_t *bstart,
                                     const int32_t *members, const float *centers, float *counts,
                                     float *centers_new, float *batch_counts) {
    const int g = blockIdx.x;
    const int bc = bcount[g];
    const float n_old = counts[g];
    __syncthreads();  // every thread read counts[g] before thread 0 rewrites it
    const float bcf = (float)bc;
    const float nc = __fadd_rn(n_old, bcf);
    const int s0 = bstart[g];
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float cgj = centers[(int64_t)g * d + j];
        float out = cgj;
        if (bc > 0) {
            float sum = 0.0f;
            for (int m = 0; m < bc; ++m)
                sum = __fadd_rn(sum, x[row_of(rows, members[s0 + m]) * d + j]);
            const float a = __fmul_rn(cgj, n_old);
            const float b = __fadd_rn(a, sum);
            out = __fdiv_rn(b, nc);
        }
        centers_new[(int64_t)g * d + j] = out;
    }
    if (threadIdx.x == 0) {
        counts[g] = nc;
        if (batch_counts) batch_counts[g] = bcf;
    }
}

__global__ void kmeans_reassign_kernel(const float *x, const int64_t *rows, const int32_t *brow,
                                       const int32_t *clusters, int d, float *centers,
                                       float *counts, float new_count) {
    const int i = blockIdx.x;
    const int g = clusters[i];
    const float *src = x + row_of(rows, brow[i]) * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) centers[(int64_t)g * d + j] = src[j];
    if (threadIdx.x == 0) counts[g] = new_count;
}

// ---------------------------------------------------------------------------
// greedy k-means++ (minibatch_kmeans.py:73-126)
// ---------------------------------------------------------------------------
struct KppWs {
    float *closest;               // [n]
    float *cum;                   // [n]
    float *cand;                  // [trials][n]
    unsigned long long *pot_fx;   // [trials + 1][2]; slot trials = first potential
    int64_t *cid;                 // [trials]
};

static size_t kpp_layout(int64_t n, int trials, char *base, KppWs *ws) {
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off = (off + b + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_cl = take((size_t)n * 4), o_cu = take((size_t)n * 4);
    const size_t o_ca = take((size_t)trials * n * 4);
    const size_t o_pf = take((size_t)(trials + 1) * 16), o_ci = take((size_t)trials * 8);
    if (base && ws) {
        ws->closest = (float *)(base + o_cl);
        ws->cum = (float *)(base + o_cu);
        ws->cand = (float *)(base + o_ca);
        ws->pot_fx = (unsigned long long *)(base + o_pf);
        ws->cid = (int64_t *)(base + o_ci);
    }
    return off;
}

constexpr int kKppThreads = 256;

// centre 0 = init row first_id; closest distance of every init row to it.
// Rows i = blk * NT + tid, blk + nblk, ... (a grid-stride loop); c0s is the
// first centre staged in shared memory by the caller.
template <int NT>
__device__ __forceinline__ void kpp_first_rows(const float *x, const int64_t *rows,
                                               const float *xx, int64_t n, int d, int trials,
                                               int64_t first_id, const float *c0s, int blk,
                                               int nblk, KppWs &ws, u128 *sw) {
    const float c0 = xx[row_of(rows, first_id)];
    for (int64_t i0 = (int64_t)blk * NT; i0 < n; i0 += (int64_t)nblk * NT) {
        const int64_t i = i0 + threadIdx.x;
        u128 fx = 0;
        if (i < n) {
            const float *xi = x + row_of(rows, i) * d;
            float acc = 0.0f;
            for (int t = 0; t < d; ++t) acc = fmaf(xi[t], c0s[t], acc);
            const float v = dist2_def(xx[row_of(rows, i)], c0, acc);
            ws.closest[i] = v;
            fx = fx_of(v);
        }
        block_add_u128<NT>(fx, ws.pot_fx + 2 * trials, sw);
    }
}

__global__ void __launch_bounds__(kKppThreads) kpp_first_kernel(
    const float *x, const int64_t *rows, const float *xx, int64_t n, int d, int trials,
    int64_t first_id, float *centers, int64_t *chosen, KppWs ws) {
    __shared__ u128 sw[kKppThreads / 32];
    extern __shared__ __align__(16) float kpp_smem[];  // [d] first centre
    const int64_t fr = row_of(rows, first_id);
    for (int j = threadIdx.x; j < d; j += kKppThreads) {
        kpp_smem[j] = x[fr * d + j];
        if (blockIdx.x == 0) centers[j] = kpp_smem[j];
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && chosen) chosen[0] = first_id;
    __syncthreads();
    kpp_first_rows<kKppThreads>(x, rows, xx, n, d, trials, first_id, kpp_smem, blockIdx.x,
                                gridDim.x, ws, sw);
}

constexpr int kScanThreads = 1024;

// One CTA of NT threads.  ci >= 2: pick the best candidate of centre ci-1
// (lowest potential, first on ties), make it centre ci-1 and its distances
// the new closest distances.  ci <= k-1: fixed-point prefix sums of closest,
// then the searchsorted of the trials' uniform draws for centre ci.  The
// prefix sums are exact integers, so any split of the rows over threads
// gives the same values.
template <int NT>
__device__ __forceinline__ void kpp_scan_cta(const float *x, const int64_t *rows, int64_t n,
                                             int d, int k, int trials, int ci,
                                             const double *uniforms, float *centers,
                                             int64_t *chosen, KppWs &ws, u128 *sw, float &s_pot,
                                             int &s_best) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        if (ci >= 2) {
            int best = 0;
            float bp = INFINITY;
            for (int t = 0; t < trials; ++t) {
                const u128 s = ((u128)ws.pot_fx[2 * t + 1] << 64) | ws.pot_fx[2 * t];
                const float p = fx_to_float(s);
                if (t == 0 || p < bp) {
                    bp = p;
                    best = t;
                }
            }
            s_best = best;
            s_pot = bp;
            if (chosen) chosen[ci - 1] = ws.cid[best];
        } else {
            const u128 s = ((u128)ws.pot_fx[2 * trials + 1] << 64) | ws.pot_fx[2 * trials];
            s_best = -1;
            s_pot = fx_to_float(s);
        }
    }
    __syncthreads();
    const int best = s_best;
    if (best >= 0) {
        const int64_t src = row_of(rows, ws.cid[best]);
        for (int j = tid; j < d; j += NT) centers[(int64_t)(ci - 1) * d + j] = x[src * d + j];
        const float *cb = ws.cand + (int64_t)best * n;
        for (int64_t i = tid; i < n; i += NT) ws.closest[i] = cb[i];
    }
    __syncthreads();
    if (ci >= k) return;  // the last centre is placed: no further draw
    if (tid < 2 * trials) ws.pot_fx[tid] = 0ull;  // candidate sums of centre ci
    // inclusive prefix sums: thread chunks, block scan of the chunk totals
    const int64_t per = (n + NT - 1) / NT;
    const int64_t i0 = (int64_t)tid * per, i1 = min(n, i0 + per);
    u128 local = 0;
    for (int64_t i = i0; i < i1; ++i) local += fx_of(ws.closest[i]);
    u128 v = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long lo = __shfl_up_sync(0xffffffffu, (unsigned long long)v, o);
        const unsigned long long hi = __shfl_up_sync(0xffffffffu, (unsigned long long)(v >> 64), o);
        if (lane >= o) v += ((u128)hi << 64) | lo;
    }
    if (lane == 31) sw[warp] = v;
    __syncthreads();
    if (warp == 0) {
        const u128 w = lane < NT / 32 ? sw[lane] : (u128)0;
        u128 s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long lo = __shfl_up_sync(0xffffffffu, (unsigned long long)s, o);
            const unsigned long long hi =
                __shfl_up_sync(0xffffffffu, (unsigned long long)(s >> 64), o);
            if (lane >= o) s += ((u128)hi << 64) | lo;
        }
        if (lane < NT / 32) sw[lane] = s - w;
    }
    __syncthreads();
    u128 run = sw[warp] + v - local;
    for (int64_t i = i0; i < i1; ++i) {
        run += fx_of(ws.closest[i]);
        ws.cum[i] = fx_to_float(run);
    }
    __syncthreads();
    // searchsorted(side="left") in fp64, clipped to n - 1
    if (tid < trials) {
        const double val = __dmul_rn(uniforms[(int64_t)(ci - 1) * trials + tid], (double)s_pot);
        int64_t lo = 0, hi = n;
        while (lo < hi) {
            const int64_t mid = lo + (hi - lo) / 2;
            if ((double)ws.cum[mid] < val) lo = mid + 1;
            else hi = mid;
        }
        ws.cid[tid] = lo > n - 1 ? n - 1 : lo;
    }
}

__global__ void __launch_bounds__(kScanThreads) kpp_scan_kernel(
    const float *x, const int64_t *rows, int64_t n, int d, int k, int trials, int ci,
    const double *uniforms, float *centers, int64_t *chosen, KppWs ws) {
    __shared__ u128 sw[kScanThreads / 32 + 1];
    __shared__ float s_pot;
    __shared__ int s_best;
    kpp_scan_cta<kScanThreads>(x, rows, n, d, k, trials, ci, uniforms, centers, chosen, ws, sw,
                               s_pot, s_best);
}

// The trials' candidate rows staged into shared memory ([trials][d]) and
// their squared norms.
__device__ __forceinline__ void kpp_stage_candidates(const float *x, const int64_t *rows,
                                                     const float *xx, int d, int trials,
                                                     const KppWs &ws, float *cs, float *s_cc,
                                                     int nt) {
    for (int i = threadIdx.x; i < trials * d; i += nt) {
        const int t = i / d, j = i - t * d;
        cs[i] = x[row_of(rows, ws.cid[t]) * d + j];
    }
    if (threadIdx.x < trials) s_cc[threadIdx.x] = xx[row_of(rows, ws.cid[threadIdx.x])];
}

// distance of every init row to each candidate (capped by the closest
// distance so far) and the candidates' potentials; rows as kpp_first_rows
template <int NT>
__device__ __forceinline__ void kpp_candidate_rows(const float *x, const int64_t *rows,
                                                   const float *xx, int64_t n, int d, int trials,
                                                   const float *cs, const float *s_cc, int blk,
                                                   int nblk, KppWs &ws, u128 *sw) {
    for (int64_t r0 = (int64_t)blk * NT; r0 < n; r0 += (int64_t)nblk * NT) {
        const int64_t i = r0 + threadIdx.x;
        float acc[kKmMaxTrials];
#pragma unroll
        for (int t = 0; t < kKmMaxTrials; ++t) acc[t] = 0.f;
        float xxi = 0.f, cl = 0.f;
        if (i < n) {
            const float *xi = x + row_of(rows, i) * d;
            for (int tt = 0; tt < d; ++tt) {
                const float a = xi[tt];
#pragma unroll
                for (int t = 0; t < kKmMaxTrials; ++t)
                    if (t < trials) acc[t] = fmaf(cs[t * d + tt], a, acc[t]);
            }
            xxi = xx[row_of(rows, i)];
            cl = ws.closest[i];
        }
#pragma unroll
        for (int t = 0; t < kKmMaxTrials; ++t) {
            if (t < trials) {  // block-uniform
                u128 fx = 0;
                if (i < n) {
                    float v = dist2_def(s_cc[t], xxi, acc[t]);
                    if (cl < v) v = cl;
                    ws.cand[(int64_t)t * n + i] = v;
                    fx = fx_of(v);
                }
                block_add_u128<NT>(fx, ws.pot_fx + 2 * t, sw);
            }
        }
    }
}

__global__ void __launch_bounds__(kKppThreads) kpp_candidates_kernel(
    const float *x, const int64_t *rows, const float *xx, int64_t n, int d, int trials,
    KppWs ws) {
    extern __shared__ __align__(16) float kpp_smem[];  // [trials][d]
    __shared__ u128 sw[kKppThreads / 32];
    __shared__ float s_cc[kKmMaxTrials];
    kpp_stage_candidates(x, rows, xx, d, trials, ws, kpp_smem, s_cc, kKppThreads);
    __syncthreads();
    kpp_candidate_rows<kKppThreads>(x, rows, xx, n, d, trials, kpp_smem, s_cc, blockIdx.x,
                                    gridDim.x, ws, sw);
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
static int km_set_smem(const void *fn, size_t bytes) {
    return bytes > 48 * 1024 ? ensure_dyn_smem(fn, bytes) : SANTA_OK;
}

}  // namespace santa

using namespace santa;

extern "C" int santa_kmeans_sqnorm(const float *x, int64_t n, int32_t d, float *out,
                                   cudaStream_t stream) {
    if (!x || !out || n <= 0 || d <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    kmeans_sqnorm_kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, stream>>>(x, n, d, out);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_kmeans_assign(const float *x, const int64_t *rows, const float *xx,
                                   int64_t n, int32_t d, const float *centers, const float *cc,
                                   int32_t k, int32_t *labels, float *min_dist,
                                   unsigned long long *inertia_fx, cudaStream_t stream) {
    if (!x || !xx || !centers || !cc || n <= 0 || k <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    if (d <= 0 || (d & 3) || d > kKmMaxDim) return SANTA_ERR_UNSUPPORTED;
    if (((uintptr_t)x | (uintptr_t)centers) & 15) return SANTA_ERR_UNSUPPORTED;
    const size_t smem = ((size_t)(kAsRows + kAsCent) * (d + 4) + kAsCent) * 4;
    int st = km_set_smem((const void *)kmeans_assign_kernel, smem);
    if (st) return st;
    kmeans_assign_kernel<<<(unsigned)ceil_div64(n, kAsRows), kAsThreads, smem, stream>>>(
        x, rows, xx, n, d, centers, cc, k, labels, min_dist, inertia_fx);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_kmeans_update_workspace_bytes(int64_t nb, int32_t k, size_t *bytes) {
    if (!bytes || nb <= 0 || k <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    *bytes = (((size_t)2 * k * 4 + 255) & ~(size_t)255) + (size_t)nb * 4;
    return SANTA_OK;
}

extern "C" int santa_kmeans_update(const float *x, const int64_t *rows, int64_t nb, int32_t d,
                                   const int32_t *labels, int32_t k, const float *centers,
                                   float *counts, float *centers_new, float *batch_counts,
                                   void *workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (!x || !labels || !centers || !counts || !centers_new || nb <= 0 || d <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (k <= 0 || k > kKmMaxClusters || d > kKmMaxDim) return SANTA_ERR_UNSUPPORTED;
    size_t need = 0;
    santa_kmeans_update_workspace_bytes(nb, k, &need);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    char *w = (char *)workspace;
    int32_t *bcount = (int32_t *)w, *bstart = bcount + k;
    int32_t *members = (int32_t *)(w + (((size_t)2 * k * 4 + 255) & ~(size_t)255));
    const size_t psm = (size_t)2 * k * 4;
    int st = km_set_smem((const void *)kmeans_partition_kernel, psm);
    if (st) return st;
    kmeans_partition_kernel<<<1, kPartThreads, psm, stream>>>(labels, nb, k, bcount, bstart,
                                                              members);
    SANTA_LAUNCH_CHECK();
    const int bt = d >= 128 ? 128 : ((d + 31) / 32) * 32;
    kmeans_update_kernel<<<k, bt, 0, stream>>>(x, rows, d, bcount, bstart, members, centers,
                                               counts, centers_new, batch_counts);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_kmeans_reassign(const float *x, const int64_t *rows,
                                     const int32_t *batch_rows, const int32_t *clusters,
                                     int32_t n_reassign, int32_t d, float *centers,
                                     float *counts, float new_count, cudaStream_t stream) {
    if (n_reassign == 0) return SANTA_OK;
    if (!x || !batch_rows || !clusters || !centers || !counts || n_reassign < 0 || d <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    kmeans_reassign_kernel<<<n_reassign, 128, 0, stream>>>(x, rows, batch_rows, clusters, d,
                                                          centers, counts, new_count);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_kmeans_plusplus_workspace_bytes(int64_t n, int32_t trials, size_t *bytes) {
    if (!bytes || n <= 0 || trials <= 0 || trials > kKmMaxTrials)
        return SANTA_ERR_INVALID_ARGUMENT;
    *bytes = kpp_layout(n, trials, nullptr, nullptr);
    return SANTA_OK;
}

extern "C" int santa_kmeans_plusplus(const float *x, const int64_t *rows, const float *xx,
                                     int64_t n, int32_t d, int32_t k, int32_t trials,
                                     int64_t first_id, const double *uniforms, float *centers,
                                     int64_t *chosen_ids, void *workspace,
                                     size_t workspace_bytes, cudaStream_t stream) {
    if (!x || !xx || !uniforms || !centers || n <= 0 || d <= 0 || k <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (trials <= 0 || trials > kKmMaxTrials || d > kKmMaxDim || k > kKmMaxClusters)
        return SANTA_ERR_UNSUPPORTED;
    if (k > n || first_id < 0 || first_id >= n) return SANTA_ERR_INVALID_ARGUMENT;
    const size_t need = kpp_layout(n, trials, nullptr, nullptr);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    KppWs ws;
    kpp_layout(n, trials, (char *)workspace, &ws);
    SANTA_CUDA_CHECK(cudaMemsetAsync(ws.pot_fx, 0, (size_t)(trials + 1) * 16, stream));
    const unsigned grid = (unsigned)ceil_div64(n, kKppThreads);
    kpp_first_kernel<<<grid, kKppThreads, (size_t)d * 4, stream>>>(x, rows, xx, n, d, trials,
                                                                   first_id, centers, chosen_ids,
                                                                   ws);
    SANTA_LAUNCH_CHECK();
    const size_t csm = (size_t)trials * d * 4;
    int st = km_set_smem((const void *)kpp_candidates_kernel, csm);
    if (st) return st;
    for (int ci = 1; ci < k; ++ci) {
        kpp_scan_kernel<<<1, kScanThreads, 0, stream>>>(x, rows, n, d, k, trials, ci, uniforms,
                                                        centers, chosen_ids, ws);
        SANTA_LAUNCH_CHECK();
        kpp_candidates_kernel<<<grid, kKppThreads, csm, stream>>>(x, rows, xx, n, d, trials,
                                                                  ws);
        SANTA_LAUNCH_CHECK();
    }
    if (k >= 2) {
        kpp_scan_kernel<<<1, kScanThreads, 0, stream>>>(x, rows, n, d, k, trials, k, uniforms,
                                                        centers, chosen_ids, ws);
        SANTA_LAUNCH_CHECK();
    }
    return SANTA_OK;
}
