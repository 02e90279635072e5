// SANTA++ decode, selection phase: one CTA per (batch, KV head).
//
// Replaces the ranking and sampling half of SantaPlusEngine._approximate_attention
// (santapp_ruler/attention/santapp.py:395-468):
//   guess_g = log(n_g) + c_g . q * scale           (:397-400, :431-434)
//   ranking = argsort(guess, descending)           (:401, lowest index first on ties)
//   topk    = shortest ranked prefix holding >= token_budget tokens (:402-411)
//   guided  = multinomial over softmax(guess), uniform inside the cluster (:436-448)
//   uniform = randint(old_end), santa = multinomial over the exact softmax (:450-467)
//   hybrid  = the k best-ranked clusters exactly + uniform draws of the rest.
// The guess follows the oracle's defined arithmetic bit for bit: the dot
// product is a sequential fmaf chain over head_dim, then fl32(dot * scale),
// then fl32(log_n + that).
//
// Structure (512 threads = 16 warps):
//   1. q, cluster starts/lengths and the first 128-centroid tile are loaded
//      together; each later tile is prefetched into registers while the
//      current one is scored.  A thread scores two centroids for one query
//      head with two interleaved fmaf chains.
//   2. Top-k: one warp per query head; every lane keeps its clusters' keys
//      (orderable guess << 32 | ~index) sorted in registers.  Hybrid with
//      k <= 16 takes the 16 largest with a butterfly of bitonic merges; the
//      budget walk and larger k extract the next best cluster with two
//      redux.sync steps and a register shift per cluster.
//   3. Union of the group's selections and its expanded row list.
//   4. Draws: two warps per query head.
#include "decode_common.cuh"

#include <math.h>

namespace santa {

constexpr int kTileC = 128;  // centroids per scoring tile

__device__ int sel_block_exclusive_scan(int v, int *sw, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = kSelThreads / 32;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sw[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < NW ? sw[lane] : 0;
        int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < NW) sw[lane] = s - w;
        if (lane == 31) sw[32] = s;
    }
    __syncthreads();
    int r = sw[warp] + x - v;
    if (total) *total = sw[32];
    __syncthreads();
    return r;
}

// KPL == 8 (at most 256 clusters): the whole centroid block is loaded at
// once; otherwise 128-centroid tiles.
template <int D, int KPL>
struct SelSmem {
    static constexpr int ROWS = KPL == 8 ? 256 : kTileC;
    // whole-block variant: 16-byte rows (pitch D + 4) read as float4, which
    // keeps 8 consecutive rows of a quarter warp on distinct bank groups
    static constexpr int PITCH = KPL == 8 ? D + 4 : D + 1;
    static constexpr int CT_FLOATS = ROWS * PITCH;
    static constexpr int MAXG = KPL * 32;
    static_assert(CT_FLOATS >= SANTA_MAX_GROUP * MAXG,
                  "the centroid area also holds the guided CDF");
    static_assert(CT_FLOATS >= 3 * MAXG, "the centroid area also holds the union entries");
    static_assert(CT_FLOATS * 4 >= SANTA_MAX_GROUP * SANTA_SHARD_MAX_KEYS * 8,
                  "the centroid area also holds the gathered shard keys");
};

__device__ __forceinline__ void cp_async4(void *dst_smem, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst_smem)), "l"(src)
                 : "memory");
}

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int o) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, o);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), o);
    return ((uint64_t)hi << 32) | lo;
}

// The 16 largest of the warp's 32 x 8 keys (every lane's 8 sorted
// descending, 0 = none), sorted descending, in every lane.  Each butterfly
// level merges the lane's list with its partner's: the elementwise maximum of
// one list and the other reversed holds the 16 largest of both as a bitonic
// sequence, which four half-cleaner stages sort.  Keys are unique (the low
// word is the cluster id), so the result does not depend on the order of
// the levels.
__device__ __forceinline__ void warp_top16(const uint64_t (&k8)[8], uint64_t (&t)[16]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        t[i] = k8[i];
        t[i + 8] = 0ull;
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        // entries i and 15 - i exchange with the partner together (two live
        // temporaries instead of a copy of the partner's list)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint64_t a = shfl_xor_u64(t[15 - i], o), b = shfl_xor_u64(t[i], o);
            t[i] = t[i] > a ? t[i] : a;
            t[15 - i] = t[15 - i] > b ? t[15 - i] : b;
        }
#pragma unroll
        for (int j = 8; j > 0; j >>= 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if ((i & j) == 0) {
                    const uint64_t x = t[i], y = t[i + j];
                    t[i] = x > y ? x : y;
                    t[i + j] = x > y ? y : x;
                }
            }
        }
    }
}

// a candidate key (the peer-memory exchange runs on the cluster kernel only)
__device__ __forceinline__ void store_key(const DecodeArgs &a, int64_t idx, uint64_t key) {
    a.cand_out[idx] = key;
}

// KPL: keys per lane in the top-k extraction (clusters lane, lane+32, ...).
template <int D, int KPL>
__global__ void __launch_bounds__(kSelThreads) decode_select_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int bh = blockIdx.x;
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const int g = a.geo.group;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Gmax = a.sum.max_groups;
    const int mode = a.p.mode;
    const int S = a.p.samples;
    const int sample_end = a.geo.sample_end;
    const bool uses_clusters = (mode == SANTA_MODE_TOPK || mode == SANTA_MODE_GUIDED ||
                                mode == SANTA_MODE_HYBRID);
    const int kcap = (mode == SANTA_MODE_HYBRID) ? max(a.p.topk_clusters, 1) : 1;

    // shared memory carve-up
    float *qs = (float *)smem_raw;                              // [8][D]
    float *ct = qs + SANTA_MAX_GROUP * D;                       // [ROWS][D+1]
    int *starts_s = (int *)(ct + SelSmem<D, KPL>::CT_FLOATS);   // [Gmax]
    int *len_s = starts_s + Gmax;                               // [Gmax]
    int *mask_s = len_s + Gmax;                                 // [Gmax]
    float *guess_s = (float *)(mask_s + Gmax);                  // [8][Gmax]
    int *gapcum = (int *)(guess_s + SANTA_MAX_GROUP * Gmax);    // [8][2*kcap+1]
    int *sw = gapcum + SANTA_MAX_GROUP * (2 * kcap + 1);        // [40]
    int *head_sel = sw + 40;                                    // [8]
    int *head_exact = head_sel + 8;                             // [8]
    int *head_ns = head_exact + 8;                              // [8]
    int *head_sbase = head_ns + 8;                              // [8]
    int *head_cnt = head_sbase + 8;                             // [8]
    float *head_f = (float *)(head_cnt + 8);                    // [8][4]

    // ---- 1. loads: q, cluster metadata and centroids requested together ----
    const float *cent = a.sum.centroids + (int64_t)bh * Gmax * D;
    constexpr int V4 = kTileC * D / 4 / kSelThreads;  // float4 per thread per tile
    float4 pre[KPL == 8 ? 1 : V4];
    auto load_tile = [&](int c0, int nrow) {
#pragma unroll
        for (int j = 0; j < V4; ++j) {
            const int i = tid + j * kSelThreads;  // float4 index in the tile
            const int r = (i * 4) / D;
            pre[j] = r < nrow ? *(const float4 *)(cent + (int64_t)(c0 + r) * D + (i * 4 - r * D))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    if (uses_clusters) {
        if constexpr (KPL == 8) {
            // the whole block (<= 256 rows) straight into shared memory with
            // 16-byte copies, rows D + 4 floats apart
            constexpr int P = SelSmem<D, KPL>::PITCH;
            for (int i = tid; i < Gmax * D / 4; i += kSelThreads) {
                const int r = (4 * i) / D;
                cp_async16(ct + r * P + (4 * i - r * D), cent + 4 * i);
            }
            for (int i = tid; i < Gmax; i += kSelThreads) {
                cp_async4(starts_s + i, a.sum.starts + (int64_t)bh * Gmax + i);
                cp_async4(len_s + i, a.sum.lengths + (int64_t)bh * Gmax + i);
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        } else {
            load_tile(0, min(kTileC, Gmax));
        }
    }
    const int n_groups = uses_clusters ? a.sum.n_groups[bh] : 0;
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    for (int i = tid; i < g * D; i += kSelThreads) qs[i] = qb[i];
    if constexpr (KPL != 8) {
        for (int i = tid; i < n_groups; i += kSelThreads) {
            starts_s[i] = a.sum.starts[(int64_t)bh * Gmax + i];
            len_s[i] = a.sum.lengths[(int64_t)bh * Gmax + i];
        }
    }
    for (int i = tid; i < Gmax; i += kSelThreads) mask_s[i] = 0;
    if (tid == 0) {
        a.ws.counters[bh] = 0;  // arrival counter of the attention merge
        a.ws.flag[bh] = 0;      // set by the draws below (after block barriers)
    }
    if (tid < 8) {
        head_sel[tid] = 0;
        head_exact[tid] = 0;
        head_ns[tid] = 0;
        head_cnt[tid] = 0;
    }

    // ---- 2. centroid guesses: fl32(log_n + fl32(dot * scale)), dot = fmaf chain ----
    if constexpr (KPL == 8) {
      if (uses_clusters) {
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();
        const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
        const int c = tid & 63, h = tid >> 6;  // 64 slots x 8 heads, 4 centroids a thread
        if (h < g) {
            constexpr int P = SelSmem<D, KPL>::PITCH;
            const float *qh = qs + h * D;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int d = 0; d < D; d += 4) {
                const float4 q4 = *(const float4 *)(qh + d);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    // fmaf chain in ascending d, four dimensions per load
                    const float4 c4 = *(const float4 *)(ct + (c + 64 * k) * P + d);
                    acc[k] = fmaf(c4.x, q4.x, acc[k]);
                    acc[k] = fmaf(c4.y, q4.y, acc[k]);
                    acc[k] = fmaf(c4.z, q4.z, acc[k]);
                    acc[k] = fmaf(c4.w, q4.w, acc[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int cc = c + 64 * k;
                if (cc < n_groups)
                    guess_s[h * Gmax + cc] = __fadd_rn(logn[cc], __fmul_rn(acc[k], a.p.scale));
            }
        }
      }
    } else {
      if (uses_clusters) {
        const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
        for (int c0 = 0; c0 < n_groups; c0 += kTileC) {
#pragma unroll
            for (int j = 0; j < V4; ++j) {
                const int i = tid + j * kSelThreads;
                const int r = (i * 4) / D, d = i * 4 - r * D;
                float *dst = ct + r * (D + 1) + d;
                dst[0] = pre[j].x;
                dst[1] = pre[j].y;
                dst[2] = pre[j].z;
                dst[3] = pre[j].w;
            }
            __syncthreads();
            if (c0 + kTileC < n_groups) load_tile(c0 + kTileC, min(kTileC, n_groups - c0 - kTileC));
            const int nc = min(kTileC, n_groups - c0);
            const int c = tid & 63, h = tid >> 6;  // 64 centroid slots x 8 heads; 2 centroids each
            if (h < g && c < nc) {
                const float *r0p = ct + c * (D + 1);
                const float *r1p = ct + (c + 64) * (D + 1);
                const float *qh = qs + h * D;
                float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 8
                for (int d = 0; d < D; ++d) {
                    const float qd = qh[d];
                    acc0 = fmaf(r0p[d], qd, acc0);
                    acc1 = fmaf(r1p[d], qd, acc1);
                }
                guess_s[h * Gmax + c0 + c] = __fadd_rn(logn[c0 + c], __fmul_rn(acc0, a.p.scale));
                if (c + 64 < nc)
                    guess_s[h * Gmax + c0 + c + 64] =
                        __fadd_rn(logn[c0 + c + 64], __fmul_rn(acc1, a.p.scale));
            }
            __syncthreads();
        }
      }
    }
    __syncthreads();

    // ---- 3. ranking (TOPK / HYBRID): warp per query head, per-lane sorted keys ----
    // key = order bits of the guess << 32 | ~(global cluster id): descending
    // keys rank by guess, lowest id first on ties
    const int cbase = a.cluster_base;
    const int kk = a.p.topk_clusters;  // HYBRID: candidate keys per (b, query head)
    uint64_t *cand_s = (uint64_t *)ct;  // sharded plan: [g][num_shards][kk], in the free tile area
    if (a.shard_cands) {
        const int NS = a.num_shards, per = NS * kk;
        const int64_t rows = (int64_t)a.geo.batch * a.geo.num_kv_heads * g;
        for (int i = tid; i < g * per; i += kSelThreads) {
            const int h = i / per, r = (i - h * per) / kk, j = i - h * per - r * kk;
            cand_s[i] = a.shard_cands[((int64_t)r * rows + (int64_t)bh * g + h) * kk + j];
        }
        __syncthreads();
    }
    if ((mode == SANTA_MODE_TOPK || mode == SANTA_MODE_HYBRID) && warp < g) {
        const int h = warp;
        uint64_t key[KPL];
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            const int c = lane + 32 * j;
            key[j] = c < n_groups ? (((uint64_t)float_order_key(guess_s[h * Gmax + c]) << 32) |
                                     (uint64_t)(0xFFFFFFFFu - (uint32_t)(c + cbase)))
                                  : 0ull;
        }
        // bitonic sort, descending, entirely in registers
#pragma unroll
        for (int k = 2; k <= KPL; k <<= 1) {
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
                for (int i = 0; i < KPL; ++i) {
                    const int l = i ^ j;
                    if (l > i) {
                        const bool desc = (i & k) == 0;
                        const uint64_t x = key[i], y = key[l];
                        if (desc ? (x < y) : (x > y)) {
                            key[i] = y;
                            key[l] = x;
                        }
                    }
                }
            }
        }
        const int kmax = (mode == SANTA_MODE_HYBRID) ? min(a.p.topk_clusters, n_groups) : n_groups;
        int nsel = 0, exact = 0;
        if (a.shard_cands) {
            // global k-th best key: k rounds of a merge of the shards'
            // descending lists (lane r walks shard r's list; keys are unique)
            const uint64_t *cl = cand_s + (int64_t)h * a.num_shards * kk;
            int ptr = 0;
            uint64_t thr = 1ull;  // fewer than k keys in all: every real key passes
            for (int it = 0; it < kk; ++it) {
                const uint64_t v = (lane < a.num_shards && ptr < kk) ? cl[lane * kk + ptr] : 0ull;
                const uint32_t vh = (uint32_t)(v >> 32);
                const uint32_t mh = __reduce_max_sync(0xffffffffu, vh);
                const uint32_t ml = __reduce_max_sync(0xffffffffu, vh == mh ? (uint32_t)v : 0u);
                if (mh == 0u && ml == 0u) break;
                thr = ((uint64_t)mh << 32) | ml;
                if (v == thr) ++ptr;
            }
            // local clusters at or above it: a prefix of every lane's sorted keys
            int cnt = 0;
#pragma unroll
            for (int j = 0; j < KPL; ++j) cnt += (key[j] != 0ull && key[j] >= thr) ? 1 : 0;
            int x = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            int pos = x - cnt;
#pragma unroll
            for (int j = 0; j < KPL; ++j)
                if (j < cnt)
                    gapcum[h * (2 * kcap + 1) + pos++] =
                        (int)(0xFFFFFFFFu - (uint32_t)key[j]) - cbase;
            nsel = __shfl_sync(0xffffffffu, x, 31);
        }
        bool ranked = false;
        if constexpr (KPL == 8) {
            // hybrid with k <= 16: one merge network instead of k extraction rounds
            if (!a.shard_cands && mode == SANTA_MODE_HYBRID && kmax <= 16) {
                uint64_t t[16];
                warp_top16(key, t);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (j < kmax && t[j] != 0ull) {
                        if (lane == j) {
                            gapcum[h * (2 * kcap + 1) + j] =
                                (int)(0xFFFFFFFFu - (uint32_t)t[j]) - cbase;
                            if (a.cand_out) store_key(a, ((int64_t)bh * g + h) * kk + j, t[j]);
                        }
                        ++nsel;
                    }
                }
                ranked = true;
            }
        }
        while (!a.shard_cands && !ranked && nsel < kmax) {
            const uint32_t bhi = (uint32_t)(key[0] >> 32);
            const uint32_t mhi = __reduce_max_sync(0xffffffffu, bhi);
            const uint32_t mlo = __reduce_max_sync(0xffffffffu, bhi == mhi ? (uint32_t)key[0] : 0u);
            if (mhi == 0u && mlo == 0u) break;  // no cluster left
            const int c = (int)(0xFFFFFFFFu - mlo) - cbase;
            if (a.cand_out && lane == 0)
                store_key(a, ((int64_t)bh * g + h) * kk + nsel, ((uint64_t)mhi << 32) | mlo);
            if (lane == (c & 31)) {
#pragma unroll
                for (int j = 0; j + 1 < KPL; ++j) key[j] = key[j + 1];
                key[KPL - 1] = 0ull;
            }
            if (mode == SANTA_MODE_HYBRID) {
                // chosen list in the (still unused) gap table; mask bits and
                // lengths are applied after the loop, off its critical path
                if (lane == 0) gapcum[h * (2 * kcap + 1) + nsel] = c;
            } else {
                if (lane == (c & 31)) atomicOr(&mask_s[c], 1 << h);
                exact += len_s[c];
            }
            ++nsel;
            // budget walk (santapp.py:404-410): stop once the chosen clusters
            // hold at least token_budget tokens
            if (mode == SANTA_MODE_TOPK && exact >= a.p.token_budget) break;
        }
        if (mode == SANTA_MODE_HYBRID) {
            __syncwarp();
            int ex = 0;
            for (int j = lane; j < nsel; j += 32) {
                const int c = gapcum[h * (2 * kcap + 1) + j];
                atomicOr(&mask_s[c], 1 << h);
                ex += len_s[c];
            }
            exact = warp_sum_int(ex);
        }
        if (lane == 0) {
            head_sel[h] = nsel;
            head_exact[h] = exact;
        }
    }
    __syncthreads();
    if (a.cand_out) {  // shard candidates only: pad the key lists and stop
        if (warp < g)
            for (int j = head_sel[warp] + lane; j < kk; j += 32)
                store_key(a, ((int64_t)bh * g + warp) * kk + j, 0ull);
        return;
    }

    // ---- 4. union of the group's selections (ascending cluster order) ----
    int n_union = 0, U = 0;
    {
        // union entries kept in the (now free) centroid tile area
        int *ue_start = (int *)ct;
        int *ue_off = ue_start + Gmax;
        int *ue_mask = ue_off + Gmax;
        int base = 0, rows = 0;
        for (int c0 = 0; c0 < n_groups; c0 += kSelThreads) {
            const int c = c0 + tid;
            const int m = c < n_groups ? mask_s[c] : 0;
            int cnt;
            const int ui = sel_block_exclusive_scan(m ? 1 : 0, sw, &cnt);
            int rtot;
            const int ro = sel_block_exclusive_scan(m ? len_s[c] : 0, sw, &rtot);
            if (m) {
                a.ws.u_start[(int64_t)bh * Gmax + base + ui] = starts_s[c];
                a.ws.u_mask[(int64_t)bh * Gmax + base + ui] = m;
                a.ws.u_cid[(int64_t)bh * Gmax + base + ui] = c;
                a.ws.u_off[(int64_t)bh * (Gmax + 1) + base + ui] = rows + ro;
                ue_start[base + ui] = starts_s[c];
                ue_off[base + ui] = rows + ro;
                ue_mask[base + ui] = m;
            }
            base += cnt;
            rows += rtot;
        }
        n_union = base;
        U = rows;
        if (tid == 0) a.ws.u_off[(int64_t)bh * (Gmax + 1) + n_union] = U;
        __syncthreads();
        // expanded row list of the union: entry v = sorted row | (head mask << 24),
        // so the attention kernel resolves a row with one coalesced load
        int32_t *wr = a.ws.w_row + (int64_t)bh * sample_end;
        for (int j = warp; j < n_union; j += kSelThreads / 32) {
            const int off = ue_off[j];
            const int len = (j + 1 < n_union ? ue_off[j + 1] : U) - off;
            const int tag = ue_mask[j] << 24;
            for (int r = lane; r < len; r += 32) wr[off + r] = (ue_start[j] + r) | tag;
        }
    }

    // ---- per-head sample counts ----
    const int R = a.geo.n_total - sample_end;
    if (tid < g) {
        int ns = 0;
        if (mode == SANTA_MODE_HYBRID) ns = (sample_end - head_exact[tid] > 0) ? S : 0;
        else if (mode == SANTA_MODE_GUIDED) ns = n_groups > 0 ? S : 0;
        else if (mode == SANTA_MODE_UNIFORM || mode == SANTA_MODE_SANTA) ns = S;
        head_ns[tid] = ns;
    }
    __syncthreads();  // also: the union expansion is done with the tile area
    if (tid == 0) {
        int acc = 0;
        for (int h = 0; h < g; ++h) {
            head_sbase[h] = acc;
            acc += head_ns[h];
        }
        int32_t *meta = a.ws.meta + (int64_t)bh * 8;
        meta[0] = n_union;
        meta[1] = U;
        meta[2] = R;
        meta[3] = acc;
        meta[4] = U + R + acc;
    }
    if (tid < g) {
        a.ws.head_meta[((int64_t)bh * 8 + tid) * 2 + 0] = head_exact[tid];
        a.ws.head_meta[((int64_t)bh * 8 + tid) * 2 + 1] = head_ns[tid];
        if (a.n_exact) a.n_exact[(int64_t)bh * g + tid] = head_exact[tid];
    }

    // ---- 5a. per-head tables for the draws (one warp per head) ----
    float *cdf_all = ct;  // guided CDF [8][Gmax], in the free tile area
    if (warp < g && head_ns[warp] > 0) {
        const int h = warp;
        if (mode == SANTA_MODE_HYBRID) {
            // selected clusters of this head in ascending start order, as
            // gap[j] = non-selected positions before cluster j and cum[j] =
            // selected positions before it: rank r maps to r + cum[J] with
            // J = #{j : gap[j] <= r}
            int *gap = gapcum + h * (2 * kcap + 1);
            int *cum = gap + kcap;
            int cnt = 0, carry = 0;
            for (int c0 = 0; c0 < n_groups; c0 += 32) {
                const int c = c0 + lane;
                const bool on = c < n_groups && ((mask_s[c] >> h) & 1);
                const unsigned bal = __ballot_sync(0xffffffffu, on);
                const int l = on ? len_s[c] : 0;
                int x = l;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x += y;
                }
                if (on) {
                    const int j = cnt + __popc(bal & ((1u << lane) - 1u));
                    const int before = carry + x - l;
                    gap[j] = starts_s[c] - before;
                    cum[j] = before;
                }
                cnt += __popc(bal);
                carry += __shfl_sync(0xffffffffu, x, 31);
            }
            if (lane == 0) {
                cum[cnt] = carry;
                head_cnt[h] = cnt;
            }
        } else if (mode == SANTA_MODE_GUIDED) {
            float mx = -INFINITY;
            for (int c = lane; c < n_groups; c += 32) mx = fmaxf(mx, guess_s[h * Gmax + c]);
            mx = warp_max(mx);
            float z = 0.0f;
            for (int c = lane; c < n_groups; c += 32) z += expf(guess_s[h * Gmax + c] - mx);
            z = warp_sum(z);
            if (lane == 0) {
                head_f[h * 4 + 0] = mx;
                head_f[h * 4 + 1] = logf(z);
            }
            float *cdf = cdf_all + h * Gmax;
            float carry = 0.0f;
            for (int c0 = 0; c0 < n_groups; c0 += 32) {
                const int c = c0 + lane;
                float v = c < n_groups ? expf(guess_s[h * Gmax + c] - mx) : 0.0f;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, v, o);
                    if (lane >= o) v += y;
                }
                if (c < n_groups) cdf[c] = carry + v;
                carry += __shfl_sync(0xffffffffu, v, 31);
            }
        }
    }
    __syncthreads();

    // ---- 5b. draws: two warps per query head, 32-draw chunks alternating ----
    const int h = warp & 7, half = warp >> 3;
    if (h < g && head_ns[h] > 0) {
        const int ns = head_ns[h];
        const int sbase = head_sbase[h];
        const int gh = kv * g + h;  // global query head
        int32_t *spos = a.ws.s_pos + (int64_t)bh * g * S + sbase;
        float *soff = a.ws.s_off + (int64_t)bh * g * S + sbase;
        const int64_t inj = ((int64_t)b * a.geo.num_kv_heads * g + gh) * S;
        const uint2 key = make_uint2((uint32_t)a.p.seed, (uint32_t)(a.p.seed >> 32));
        const uint32_t stepw = (uint32_t)decode_step_word(a.p);
        const float logS = logf((float)ns);
        if (mode == SANTA_MODE_HYBRID) {
            const int *gap = gapcum + h * (2 * kcap + 1);
            const int *cum = gap + kcap;
            const int cnt = head_cnt[h];
            const int n_rest = sample_end - head_exact[h];
            const float off = (logf((float)n_rest) - logS) * kLog2e;
            for (int i = half * 32 + lane; i < ns; i += 64) {
                uint32_t r;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    int v = a.sample_a[inj + i];
                    if (v < 0 || v >= n_rest) {
                        a.ws.flag[bh] = 1;
                        v = min(max(v, 0), n_rest - 1);
                    }
                    r = (uint32_t)v;
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 2), (uint32_t)gh, (uint32_t)b, stepw),
                        key);
                    r = (uint32_t)(((uint64_t)uint4_word(w, i & 3) * (uint64_t)n_rest) >> 32);
                }
                int lo = 0, hi = cnt;  // J = first j with gap[j] > r
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (gap[mid] <= (int)r) lo = mid + 1;
                    else hi = mid;
                }
                const int p = (int)r + cum[lo];
                spos[i] = (int32_t)((uint32_t)p | ((uint32_t)h << kHeadShift));
                soff[i] = off;
            }
        } else if (mode == SANTA_MODE_GUIDED) {
            const float mx = head_f[h * 4 + 0], logz = head_f[h * 4 + 1];
            const float *cdf = cdf_all + h * Gmax;
            const float total = cdf[n_groups - 1];
            const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
            for (int i = half * 32 + lane; i < ns; i += 64) {
                int grp, within;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    grp = a.sample_a[inj + i];
                    within = a.sample_b[inj + i];
                    if (grp < 0 || grp >= n_groups) {
                        a.ws.flag[bh] = 1;
                        grp = min(max(grp, 0), n_groups - 1);
                    }
                    if (within < 0 || within >= len_s[grp]) {
                        a.ws.flag[bh] = 1;
                        within = min(max(within, 0), len_s[grp] - 1);
                    }
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 1), (uint32_t)gh, (uint32_t)b, stepw),
                        key);
                    const uint32_t w0 = (i & 1) ? w.z : w.x, w1 = (i & 1) ? w.w : w.y;
                    const float u = (float)(w0 >> 8) * (1.0f / 16777216.0f) * total;
                    int lo = 0, hi = n_groups - 1;
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (cdf[mid] > u) hi = mid;
                        else lo = mid + 1;
                    }
                    grp = lo;
                    within = (int)(((uint64_t)w1 * (uint64_t)len_s[grp]) >> 32);
                }
                const int p = starts_s[grp] + within;
                // log r = log p_g - log n_g ; offset = -log r - log S
                const float logp = guess_s[h * Gmax + grp] - mx - logz;
                const float off = (logn[grp] - logp - logS) * kLog2e;
                spos[i] = (int32_t)((uint32_t)p | ((uint32_t)h << kHeadShift));
                soff[i] = off;
            }
        } else {  // UNIFORM / SANTA: token ids over the old prefix
            const int32_t *posmap = a.sum.positions + (int64_t)bh * sample_end;
            const float off_u = (logf((float)sample_end) - logS) * kLog2e;
            const float lse_o = (mode == SANTA_MODE_SANTA) ? a.ws.lse_old[(int64_t)bh * 8 + h] : 0.f;
            for (int i = half * 32 + lane; i < ns; i += 64) {
                int t;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    t = a.sample_a[inj + i];
                    if (t < 0 || t >= sample_end) {
                        a.ws.flag[bh] = 1;
                        t = min(max(t, 0), sample_end - 1);
                    }
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 2), (uint32_t)gh, (uint32_t)b, stepw),
                        key);
                    t = (int)(((uint64_t)uint4_word(w, i & 3) * (uint64_t)sample_end) >> 32);
                }
                const int p = posmap[t];
                if (mode == SANTA_MODE_SANTA) {
                    // lw = s - log r = s - (s - lse_old) = lse_old : absolute weight
                    spos[i] = (int32_t)((uint32_t)p | ((uint32_t)h << kHeadShift) | kAbsBit);
                    soff[i] = lse_o - logS * kLog2e;
                } else {
                    spos[i] = (int32_t)((uint32_t)p | ((uint32_t)h << kHeadShift));
                    soff[i] = off_u;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// santa mode: log2-sum-exp2 of every old-prefix score (the oracle proposal
// reads all old keys, santapp.py:450-458).  One CTA per (batch, KV head).
// ---------------------------------------------------------------------------
template <int D, typename T>
__global__ void __launch_bounds__(256) decode_old_lse_kernel(DecodeArgs a) {
    const int bh = blockIdx.x;
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const int g = a.geo.group;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float qs[SANTA_MAX_GROUP][D];
    __shared__ float wm[8][SANTA_MAX_GROUP], wl[8][SANTA_MAX_GROUP];
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    for (int i = threadIdx.x; i < g * D; i += 256) qs[i / D][i % D] = qb[i] * a.p.scale * kLog2e;
    __syncthreads();
    constexpr int PER = D / 32;
    float m[SANTA_MAX_GROUP], l[SANTA_MAX_GROUP];
#pragma unroll
    for (int h = 0; h < SANTA_MAX_GROUP; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
    }
    for (int t = warp; t < a.geo.sample_end; t += 8) {
        const T *kb = (const T *)a.key_cache + cache_row(a.geo, bh, t) * D;
        float kr[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) kr[j] = to_f32<T>(kb[lane + 32 * j]);
#pragma unroll
        for (int h = 0; h < SANTA_MAX_GROUP; ++h) {
            if (h < g) {
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < PER; ++j) s = fmaf(kr[j], qs[h][lane + 32 * j], s);
                s = warp_sum(s);
                if (s > m[h]) {
                    l[h] = l[h] * exp2f(m[h] - s) + 1.0f;
                    m[h] = s;
                } else {
                    l[h] += exp2f(s - m[h]);
                }
            }
        }
    }
    if (lane == 0)
        for (int h = 0; h < g; ++h) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
    __syncthreads();
    if (threadIdx.x < g) {
        const int h = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < 8; ++w) M = fmaxf(M, wm[w][h]);
        float L = 0.f;
        for (int w = 0; w < 8; ++w)
            if (wl[w][h] > 0.f) L += wl[w][h] * exp2f(wm[w][h] - M);
        a.ws.lse_old[(int64_t)bh * 8 + h] = M + log2f(L);
    }
}

// ---------------------------------------------------------------------------
// selection read-out (tests, traffic accounting): per query head, the set of
// exact clusters and the sorted-row position of every sample
// ---------------------------------------------------------------------------
__global__ void decode_expand_kernel(DecodeArgs a, uint8_t *selected, int32_t *sample_rows) {
    const int bh = blockIdx.x;
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const int g = a.geo.group, Gmax = a.sum.max_groups, S = a.p.samples;
    const int32_t *meta = a.ws.meta + (int64_t)bh * 8;
    const int n_union = meta[0], ns_total = meta[3];
    for (int h = 0; h < g; ++h) {
        const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
        if (selected)
            for (int c = threadIdx.x; c < Gmax; c += blockDim.x) selected[oh * Gmax + c] = 0;
        if (sample_rows && S > 0)
            for (int i = threadIdx.x; i < S; i += blockDim.x) sample_rows[oh * S + i] = -1;
    }
    __syncthreads();
    if (selected) {
        for (int j = threadIdx.x; j < n_union; j += blockDim.x) {
            const int m = a.ws.u_mask[(int64_t)bh * Gmax + j];
            const int c = a.ws.u_cid[(int64_t)bh * Gmax + j];
            for (int h = 0; h < g; ++h)
                if ((m >> h) & 1) {
                    const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
                    selected[oh * Gmax + c] = 1;
                }
        }
    }
    if (sample_rows && S > 0) {
        // samples are stored head-major with S per sampling head
        for (int j = threadIdx.x; j < ns_total; j += blockDim.x) {
            const uint32_t pk = (uint32_t)a.ws.s_pos[(int64_t)bh * g * S + j];
            const int h = (int)((pk >> kHeadShift) & 7u);
            int base = 0;
            for (int hh = 0; hh < h; ++hh) base += a.ws.head_meta[((int64_t)bh * 8 + hh) * 2 + 1];
            const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
            sample_rows[oh * S + (j - base)] = (int32_t)(pk & kPosMask);
        }
    }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int D, int KPL>
static size_t select_smem_bytes(int Gmax, int kcap) {
    size_t b = 0;
    b += SANTA_MAX_GROUP * D * 4;                                 // q
    b += (size_t)SelSmem<D, KPL>::CT_FLOATS * 4;                  // centroid area
    b += 3 * (size_t)Gmax * 4;                                    // starts, lengths, masks
    b += SANTA_MAX_GROUP * (size_t)Gmax * 4;                      // guesses
    b += SANTA_MAX_GROUP * (2 * (size_t)kcap + 1) * 4;            // gap / cum
    b += 40 * 4 + 5 * 8 * 4 + 32 * 4;                             // scan + per-head
    return b;
}

template <int D, int KPL>
static int launch_select(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int kcap = (a.p.mode == SANTA_MODE_HYBRID) ? (a.p.topk_clusters > 0 ? a.p.topk_clusters : 1) : 1;
    const size_t smem = select_smem_bytes<D, KPL>(a.sum.max_groups, kcap);
    if (smem > 227 * 1024) return SANTA_ERR_UNSUPPORTED;
    if (int st = ensure_dyn_smem((const void *)decode_select_kernel<D, KPL>, smem)) return st;
    decode_select_kernel<D, KPL><<<BH, kSelThreads, smem, stream>>>(a);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

template <int D>
static int launch_plan_d(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    if (a.p.mode == SANTA_MODE_SANTA) {
        if (a.geo.kv_dtype == SANTA_DTYPE_BF16)
            decode_old_lse_kernel<D, __nv_bfloat16><<<BH, 256, 0, stream>>>(a);
        else
            decode_old_lse_kernel<D, float><<<BH, 256, 0, stream>>>(a);
        SANTA_LAUNCH_CHECK();
    }
    if (select_group_supported(a)) return launch_select_group(a, stream);
    return a.sum.max_groups <= 256 ? launch_select<D, 8>(a, stream) : launch_select<D, 32>(a, stream);
}

int launch_plan(DecodeArgs &a, cudaStream_t stream) {
    return a.geo.head_dim == 64 ? launch_plan_d<64>(a, stream) : launch_plan_d<128>(a, stream);
}

int launch_expand(DecodeArgs &a, uint8_t *selected, int32_t *sample_rows, cudaStream_t stream) {
    decode_expand_kernel<<<a.geo.batch * a.geo.num_kv_heads, 256, 0, stream>>>(a, selected,
                                                                             sample_rows);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

}  // namespace santa
