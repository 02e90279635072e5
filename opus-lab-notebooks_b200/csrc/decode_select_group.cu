// SANTA++ decode, hybrid selection on a thread-block cluster: one CTA per
// query head, the g CTAs of a (batch, KV head) segment form one cluster and
// exchange their intermediate results through distributed shared memory.
//
// Computes exactly what decode_select_kernel computes in hybrid mode (the same
// guesses bit for bit, the same selected clusters, union, work list and
// draws), for k <= 32 selected clusters per head and at most 1024 clusters.
// It exists for latency: the one-CTA-per-segment form runs load, score,
// rank, union, tables and draws one after another on one SM; here each phase
// is spread over g SMs and the ranking is a bitonic network over all warps.
//
// Reference: the ranking of santapp.py:397-401 (descending guess, lowest
// cluster first on ties) restricted to the k best clusters, and the uniform
// importance draws of santapp.py:459-468 over the tokens outside them.
//
// Phases (cluster barriers between them):
//   1. CTA r scores centroid rows [r*per, (r+1)*per), per = ceil(Gmax / g),
//      for every query head of the group (a sequential fmaf chain over
//      head_dim, then fl32(dot * scale), then fl32(log_n + that)) and keeps
//      the keys (order bits of the guess << 32 | ~global cluster id).
//   2. CTA h ranks head h: every warp sorts batches of 32 keys (read from the
//      owning CTAs) with a bitonic network across its lanes and merges them
//      into a running descending top 32; the 8 warp lists are merged in a
//      tree.  Sharded threshold mode first runs the same network over the
//      gathered shard keys to find the global k-th key.
//   3. Every CTA reads all heads' selections, builds the union in ascending
//      cluster order and expands its share of the union's rows; CTA h writes
//      head h's counts.
//   4. CTA h draws head h's samples.
#include "decode_common.cuh"

#include <math.h>

namespace santa {

// 1-D bulk copy (TMA engine, no multicast) of this GPU's global memory into
// this CTA's shared memory: 16-byte aligned addresses, size a multiple of 16
__device__ __forceinline__ void grp_bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                             uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
constexpr int kGrpThreads = 256;
constexpr int kGrpWarps = kGrpThreads / 32;
constexpr int kGrpMaxK = 32;
constexpr int kGrpQPitch = 4;  // floats of padding per q row (distinct bank groups)

// ---- cluster / distributed shared memory helpers ---------------------------
__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
// address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cl_map(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ uint64_t cl_ld_u64(uint32_t addr) {
    uint64_t v;
    asm volatile("ld.shared::cluster.u64 %0, [%1];\n" : "=l"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ int cl_ld_s32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
// every thread of every CTA of the cluster calls these, in matching pairs
__device__ __forceinline__ void cl_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cl_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cl_sync() {
    cl_arrive();
    cl_wait();
}

// ---- warp-wide bitonic networks on unique 64-bit keys -----------------------
__device__ __forceinline__ uint64_t grp_shfl_xor_u64(uint64_t v, int o) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, o);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), o);
    return ((uint64_t)hi << 32) | lo;
}
__device__ __forceinline__ uint64_t grp_shfl_u64(uint64_t v, int src) {
    const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
    const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
    return ((uint64_t)hi << 32) | lo;
}

// one key per lane -> sorted descending in lane order
__device__ __forceinline__ uint64_t warp_sort32_desc(uint64_t x, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint64_t p = grp_shfl_xor_u64(x, j);
            // blocks of k alternate direction; the last level (k = 32) is
            // one descending block
            const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
            const bool gt = x > p;
            x = (gt == keep_max) ? x : p;
        }
    }
    return x;
}

// a bitonic sequence (one key per lane) -> sorted descending
__device__ __forceinline__ uint64_t warp_bitonic_clean_desc(uint64_t x, int lane) {
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        const uint64_t p = grp_shfl_xor_u64(x, j);
        const bool keep_max = (lane & j) == 0;
        const bool gt = x > p;
        x = (gt == keep_max) ? x : p;
    }
    return x;
}

// The 32 largest of the n keys key_at(i), i in [0, n), descending, left in
// lists[0..31] (0 = no key).  Every thread of the CTA calls it; lists is
// [kGrpWarps][32] in shared memory.  The elementwise maximum of a descending
// list and an ascending one holds the 32 largest of both as a bitonic
// sequence, which the half-cleaner stages sort.
template <typename F>
__device__ __forceinline__ void block_top32(int n, F key_at, uint64_t *lists, int warp,
                                            int lane) {
    uint64_t run = 0ull;
    bool any = false;
    for (int base = warp * 32; base < n; base += kGrpThreads) {
        const int i = base + lane;
        uint64_t x = i < n ? key_at(i) : 0ull;
        x = warp_sort32_desc(x, lane);
        if (any) {
            const uint64_t rev = grp_shfl_u64(x, 31 - lane);
            x = warp_bitonic_clean_desc(run > rev ? run : rev, lane);
        }
        run = x;
        any = true;
    }
    lists[warp * 32 + lane] = run;
    __syncthreads();
#pragma unroll
    for (int s = kGrpWarps / 2; s > 0; s >>= 1) {
        if (warp < s) {
            const uint64_t rev = lists[(warp + s) * 32 + 31 - lane];
            run = warp_bitonic_clean_desc(run > rev ? run : rev, lane);
            lists[warp * 32 + lane] = run;
        }
        __syncthreads();
    }
}

// exclusive block scan of two counters at once
__device__ __forceinline__ int2 grp_block_scan2(int a, int b, int2 *sw, int2 &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int xa = a, xb = b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ya = __shfl_up_sync(0xffffffffu, xa, o);
        const int yb = __shfl_up_sync(0xffffffffu, xb, o);
        if (lane >= o) {
            xa += ya;
            xb += yb;
        }
    }
    if (lane == 31) sw[warp] = make_int2(xa, xb);
    __syncthreads();
    int pa = 0, pb = 0, ta = 0, tb = 0;
#pragma unroll
    for (int w = 0; w < kGrpWarps; ++w) {
        const int2 v = sw[w];
        if (w < warp) {
            pa += v.x;
            pb += v.y;
        }
        ta += v.x;
        tb += v.y;
    }
    total = make_int2(ta, tb);
    return make_int2(pa + xa - a, pb + xb - b);
}

// One centroid row (cluster c, slice row i) against NH query heads part ..
// part + NH - 1 (heads >= g are padding: q rows past the group, no key):
// one fmaf chain per head in ascending d, the FMAs component-major across
// the NH chains, the row read from the staged slice in shared memory.  The
// keys go to keys[head * per + i].
template <int NH, int D, int QP>
__device__ __forceinline__ void grp_score_row(const float *row, const float *qs, int part, int g,
                                              float log_n, float scale, int c, int n_groups,
                                              int cbase, uint64_t *keys, int per, int i) {
    float acc[NH];
#pragma unroll
    for (int j = 0; j < NH; ++j) acc[j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; d += 4) {
        const float4 x = *(const float4 *)(row + d);
        float4 u[NH];
#pragma unroll
        for (int j = 0; j < NH; ++j) u[j] = *(const float4 *)(qs + (part + j) * QP + d);
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.x, u[j].x, acc[j]);
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.y, u[j].y, acc[j]);
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.z, u[j].z, acc[j]);
#pragma unroll
        for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.w, u[j].w, acc[j]);
    }
    const uint64_t low = (uint64_t)(0xFFFFFFFFu - (uint32_t)(c + cbase));
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        if (part + j < g) {  // a padded head set computes its spare chain for nothing
            const float gs = __fadd_rn(log_n, __fmul_rn(acc[j], scale));
            keys[(part + j) * per + i] =
                c < n_groups ? (((uint64_t)float_order_key(gs) << 32) | low) : 0ull;
        }
    }
}

// Unstaged slice: the warp scores the rows of its 32 lanes (lane row r, heads
// part .. part + NH - 1), the rows streamed through the warp's two 2 KB
// buffers [32 rows][16 floats] one 16-dim piece at a time.  Each piece is one batch
// of coalesced cp.async copies (four lanes per row, 8 rows per instruction),
// 16-byte slot k of row j held at slot k ^ ((j >> 1) & 3), so a quarter
// warp reading its eight rows hits eight distinct bank groups.  The chains
// are those of grp_score_row: one fmaf chain per head in ascending d.
constexpr int kGrpPiece = 16;  // floats of a row per piece
template <int NH, int D, int QP>
__device__ __forceinline__ void grp_score_pieces(const float *cent, float *buf, const float *qs,
                                                 bool active, int r, int part, int g,
                                                 float log_n, float scale, int c, int n_groups,
                                                 int cbase, uint64_t *keys, int per) {
    const int lane = threadIdx.x & 31;
    // the copies of this lane: rows of lanes 8i + lane / 4, slot lane % 4
    const float *src[4];
    int dst[4];
    bool cp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int j = 8 * i + (lane >> 2), k = lane & 3;
        const int rj = __shfl_sync(0xffffffffu, r, j);
        cp[i] = __shfl_sync(0xffffffffu, active ? 1 : 0, j) != 0;
        src[i] = cent + (int64_t)rj * D + 4 * k;
        dst[i] = j * kGrpPiece + 4 * (k ^ ((j >> 1) & 3));
    }
    const int swz = (lane >> 1) & 3;
    constexpr int NP = D / kGrpPiece;   // pieces per row
    constexpr int PB = 32 * kGrpPiece;  // floats of one piece buffer
    // piece p goes to buffer p & 1: the copies of piece p + 1 are in flight
    // while piece p is scored
    auto issue = [&](int p) {
        float *bp = buf + (p & 1) * PB;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (cp[i]) cp_async16(bp + dst[i], src[i] + p * kGrpPiece);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    float acc[NH];
#pragma unroll
    for (int j = 0; j < NH; ++j) acc[j] = 0.f;
    issue(0);
#pragma unroll 1
    for (int p = 0; p < NP; ++p) {
        if (p + 1 < NP) {
            issue(p + 1);
            asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        }
        __syncwarp();
        if (active) {
            const float *bp = buf + (p & 1) * PB;
#pragma unroll
            for (int e = 0; e < kGrpPiece / 4; ++e) {
                const float4 x = *(const float4 *)(bp + lane * kGrpPiece + 4 * (e ^ swz));
                const int d = p * kGrpPiece + 4 * e;
                float4 u[NH];
#pragma unroll
                for (int j = 0; j < NH; ++j) u[j] = *(const float4 *)(qs + (part + j) * QP + d);
#pragma unroll
                for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.x, u[j].x, acc[j]);
#pragma unroll
                for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.y, u[j].y, acc[j]);
#pragma unroll
                for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.z, u[j].z, acc[j]);
#pragma unroll
                for (int j = 0; j < NH; ++j) acc[j] = fmaf(x.w, u[j].w, acc[j]);
            }
        }
        __syncwarp();  // buffer p & 1 is refilled by piece p + 2
    }
    if (!active) return;
    const uint64_t low = (uint64_t)(0xFFFFFFFFu - (uint32_t)(c + cbase));
#pragma unroll
    for (int j = 0; j < NH; ++j) {
        if (part + j < g) {
            const float gs = __fadd_rn(log_n, __fmul_rn(acc[j], scale));
            keys[(part + j) * per + r] =
                c < n_groups ? (((uint64_t)float_order_key(gs) << 32) | low) : 0ull;
        }
    }
}

// Dynamic shared memory of one CTA:
//   keys  [g][per] u64       the guesses' keys of this CTA's rows (the
//                            cluster's CTAs read them in the ranking)
//   mask  [Gmax] int32       union masks
//   qs    [nq][D + 4] fp32   the group's q rows (nq = g, or 8 when g > 4:
//                            the second head set is padded to four)
//   work  during the scoring: the CTA's slice of per = ceil(Gmax / g)
//         centroid rows ([per][D + 4] fp32) when it fits the budget, else
//         two 2 KB piece buffers per warp (the rows streamed from global
//         memory, one piece in flight while the other is scored); after the
//         scoring the same bytes hold starts / lengths [Gmax] int32 (one bulk
//         copy each), the ranking lists [8][32] u64 and the union tables.
// The budget keeps four CTAs on an SM (the static part is ~2 KB).
constexpr int kGrpDynBudget = 53 * 1024;
constexpr int kGrpUnion = SANTA_MAX_GROUP * kGrpMaxK;  // union entries at most
struct GrpLayout {
    int per, nq;
    bool staged;
    size_t keys, mask, qs, work, len, lists, ue, bytes;
};
__host__ __device__ inline size_t grp_al16(size_t v) { return (v + 15) / 16 * 16; }
__host__ __device__ inline GrpLayout grp_layout(int Gmax, int g, int D) {
    GrpLayout L;
    L.per = (Gmax + g - 1) / g;
    L.nq = g <= 4 ? g : 8;
    L.keys = 0;
    L.mask = grp_al16((size_t)g * L.per * 8);
    L.qs = L.mask + grp_al16((size_t)Gmax * 4);
    L.work = L.qs + grp_al16((size_t)L.nq * (D + kGrpQPitch) * 4);
    // offsets inside work, after the scoring
    L.len = grp_al16((size_t)Gmax * 4);
    L.lists = 2 * L.len;
    L.ue = L.lists + (size_t)kGrpWarps * 32 * 8;
    const size_t post = L.ue + grp_al16((size_t)(4 * kGrpUnion + 1) * 4);
    const size_t slice = (size_t)L.per * (D + kGrpQPitch) * 4;
    const size_t pieces = (size_t)2 * kGrpWarps * 32 * kGrpPiece * 4;
    L.staged = L.work + (slice > post ? slice : post) <= (size_t)kGrpDynBudget;
    const size_t scoring = L.staged ? slice : pieces;
    L.bytes = L.work + (scoring > post ? scoring : post);
    return L;
}

template <int D>
__global__ void __launch_bounds__(kGrpThreads, 4) decode_select_group_kernel(DecodeArgs a) {
    constexpr int QP = D + kGrpQPitch;
    extern __shared__ __align__(16) unsigned char grp_dyn[];
    __shared__ int sel_s[kGrpMaxK];             // this head's clusters, descending key
    __shared__ int info_s[4];                   // this head: n_sel, n_exact, n_samples
    __shared__ int all_sel[SANTA_MAX_GROUP][kGrpMaxK];
    __shared__ int all_info[SANTA_MAX_GROUP][4];
    __shared__ int sid[kGrpMaxK], gap[kGrpMaxK], cum[kGrpMaxK + 1];
    __shared__ int2 sw[kGrpWarps];
    __shared__ int s_nunion, s_U;
    __shared__ uint64_t own_s[kGrpMaxK];        // peer exchange: this shard's own top-k
    __shared__ uint64_t meta_bar;               // the starts / lengths bulk copies

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = a.geo.group;
    const int rank = (int)cl_rank();  // = blockIdx.x = the local query head
    const int h = rank;
    const int bh = blockIdx.y;
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups;
    const GrpLayout L = grp_layout(Gmax, g, D);
    const int per = L.per;
    uint64_t *keys_s = (uint64_t *)(grp_dyn + L.keys);  // [g][per]
    int *mask_s = (int *)(grp_dyn + L.mask);
    float *qs = (float *)(grp_dyn + L.qs);
    unsigned char *work = grp_dyn + L.work;
    float *stage = (float *)work;  // staged: [rows][QP]; else [warps][2][32][kGrpPiece]
    // after the scoring (pointers formed where they are used)
    int *starts_s = (int *)work;
    const int c0 = rank * per;
    const int nrows = max(0, min(per, Gmax - c0));
    const int S = a.p.samples;
    const int sample_end = a.geo.sample_end;
    const int cbase = a.cluster_base;
    const int kk = a.p.topk_clusters;
    // Sharded threshold form: the clusters of this shard that reach the global
    // k-th key are all among this shard's own top-k keys (the candidates pass
    // over the same q wrote them, sorted, into the gathered key list: a key at
    // or above the global k-th has fewer than k larger keys anywhere), so the
    // centroids are not scored again.
    const bool thr_mode = a.shard_cands != nullptr;
    // Peer-memory exchange: this launch also scores and ranks the shard's own
    // clusters (as the candidates form), sends its top-k keys straight into
    // every rank's exchange buffer and reads every rank's keys of the same
    // (sequence, query head) from its own buffer as they arrive, so that one
    // launch replaces candidates -> all-gather -> threshold selection.
    const bool fused = a.p2p.peers != nullptr;

    // ---- loads: q rows and (staged layout) the slice ---------------------------
    // 16-byte cp.async copies by every thread; centroid rows and q rows land
    // in padded rows (pitch D + 4 floats: rows read at one offset by a
    // quarter warp sit on distinct bank groups).  The starts and lengths are
    // first read after the scoring: they come later, by bulk copy.
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    const float *cent = a.sum.centroids + (int64_t)(bh * Gmax + c0) * D;  // the slice
    const float *logn_g = a.sum.log_n + (int64_t)bh * Gmax;
    for (int i = tid; i < g * (D / 4); i += kGrpThreads) {
        const int hh = i / (D / 4), d = 4 * (i - hh * (D / 4));
        cp_async16(qs + hh * QP + d, qb + (int64_t)hh * D + d);
    }
    if (L.staged && !thr_mode) {
        for (int i = tid; i < nrows * (D / 4); i += kGrpThreads) {
            const int r = i / (D / 4), d = 4 * (i - r * (D / 4));
            cp_async16(stage + r * QP + d, cent + (int64_t)r * D + d);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    for (int i = tid; i < Gmax; i += kGrpThreads) mask_s[i] = 0;
    if (tid == 0) {
        mbar_init(&meta_bar, 1);
        mbar_fence_init();
    }
    if (rank == 0 && tid == 0) a.ws.flag[bh] = 0;  // draws set it after two cluster barriers
    const int n_groups = a.sum.n_groups[bh];
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();

    // ---- 1. guesses of this CTA's centroid rows for every head -------------
    // work item t takes row t % nrows and head set t / nrows: all heads when
    // g <= 4, else two sets of 4 (the second padded to 4), so the chain count
    // per item is uniform and warps are full
    if (!thr_mode) {
        const int nsets = g <= 4 ? 1 : 2;
        const int nh = g <= 4 ? g : 4;
        const int total = nrows * nsets;
        if (L.staged) {
            for (int t = tid; t < total; t += kGrpThreads) {
                const int set = t / nrows, r = t - set * nrows;
                const int c = c0 + r;
#define GRP_SCORE(N)                                                                           \
    grp_score_row<N, D, QP>(stage + r * QP, qs, set * 4, g, __ldg(logn_g + c), a.p.scale, c,   \
                            n_groups, cbase, keys_s, per, r)
                switch (nh) {
                    case 1: GRP_SCORE(1); break;
                    case 2: GRP_SCORE(2); break;
                    case 3: GRP_SCORE(3); break;
                    default: GRP_SCORE(4); break;
                }
#undef GRP_SCORE
            }
        } else {
            float *buf = stage + warp * 2 * 32 * kGrpPiece;  // two pieces
            for (int t0 = warp * 32; t0 < total; t0 += kGrpThreads) {  // warp-uniform
                const int t = t0 + lane;
                const bool active = t < total;
                const int set = active ? t / nrows : 0, r = active ? t - set * nrows : 0;
                const int c = c0 + r;
                const float log_n = active ? __ldg(logn_g + c) : 0.f;
#define GRP_SCORE(N)                                                                           \
    grp_score_pieces<N, D, QP>(cent, buf, qs, active, r, set * 4, g, log_n, a.p.scale, c,       \
                               n_groups, cbase, keys_s, per)
                switch (nh) {
                    case 1: GRP_SCORE(1); break;
                    case 2: GRP_SCORE(2); break;
                    case 3: GRP_SCORE(3); break;
                    default: GRP_SCORE(4); break;
                }
#undef GRP_SCORE
            }
        }
    }
    // starts and lengths into the work bytes, now free (the copies' async
    // proxy writes follow this CTA's generic accesses of those bytes)
    __syncthreads();
    if (tid == 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&meta_bar, 2u * (uint32_t)Gmax * 4u);
        grp_bulk_g2s(starts_s, a.sum.starts + (int64_t)bh * Gmax, (uint32_t)Gmax * 4u, &meta_bar);
        grp_bulk_g2s(work + grp_al16((size_t)Gmax * 4), a.sum.lengths + (int64_t)bh * Gmax,
                     (uint32_t)Gmax * 4u, &meta_bar);
    }
    cl_sync();  // every CTA's keys are in place

    // ---- 2. ranking of head h ---------------------------------------------------
    uint64_t *lists = (uint64_t *)(work + 2 * grp_al16((size_t)Gmax * 4));
    uint64_t thr = 1ull;  // threshold mode: the global k-th key
    if (a.shard_cands) {
        const int64_t rows = (int64_t)a.geo.batch * a.geo.num_kv_heads * g;
        const uint64_t *cand = a.shard_cands + ((int64_t)bh * g + h) * kk;
        block_top32(
            a.num_shards * kk,
            [&](int i) {
                const int r = i / kk, j = i - r * kk;
                return cand[(int64_t)r * rows * kk + j];
            },
            lists, warp, lane);
        // fewer than k keys in all: the smallest real key (every real key passes)
        int last = -1;
        for (int j = 0; j < kk; ++j)
            if (lists[j] != 0ull) last = j;
        thr = last >= 0 ? lists[last] : 1ull;
        __syncthreads();  // lists is reused below
        // this shard's own top-k keys, descending and zero-padded
        const uint64_t *own = a.shard_cands + (int64_t)a.shard_index * rows * kk +
                              ((int64_t)bh * g + h) * kk;
        if (tid < 32) lists[tid] = tid < kk ? own[tid] : 0ull;
        __syncthreads();
    } else {
        const uint32_t kbase = smem_u32(keys_s) + (uint32_t)(h * per) * 8u;
        block_top32(
            n_groups,
            [&](int c) {
                const int r = c / per, i = c - r * per;
                uint32_t addr;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n"
                             : "=r"(addr)
                             : "r"(kbase + (uint32_t)i * 8u), "r"((uint32_t)r));
                return cl_ld_u64(addr);
            },
            lists, warp, lane);
    }
    if (fused) {
        // send this shard's top-k keys (zero-padded, as the candidates form
        // writes them) to every rank, each word tagged with the epoch
        const int64_t row0 = ((int64_t)bh * g + h) * kk;
        const uint32_t tag = ll_key_tag(a.p2p.epoch);
        if (warp == 0) {
            const uint64_t key = lane < kk ? lists[lane] : 0ull;
            own_s[lane] = key;
            if (lane < kk) {
                const uint64_t w = ll_key_encode(key, tag);
                for (int r = 0; r < a.p2p.n; ++r)
                    st_relaxed_sys(p2p_key_slot(a.p2p, a.p2p.peers[r], a.p2p.rank) + row0 + lane, w);
            }
        }
        __syncthreads();  // lists is reused
        // every rank's keys of this row, polled in this rank's buffer
        const uint64_t t0 = p2p_now_ns();
        bool ok = true;
        block_top32(
            a.p2p.n * kk,
            [&](int i) {
                const int r = i / kk, j = i - r * kk;
                return ll_key_wait(a.p2p, p2p_key_slot(a.p2p, a.p2p.local, r) + row0 + j, tag,
                                   t0, ok);
            },
            lists, warp, lane);
        int last = -1;
        for (int j = 0; j < kk; ++j)
            if (lists[j] != 0ull) last = j;
        thr = last >= 0 ? lists[last] : 1ull;
        __syncthreads();
        if (tid < 32) lists[tid] = own_s[tid];
        __syncthreads();
    }
    // the starts / lengths bulk copies (bounded wait; a local copy always lands)
    if (!mbar_wait(&meta_bar, 0)) a.ws.flag[bh] = 2;
    const int *len_s = (const int *)(work + grp_al16((size_t)Gmax * 4));
    if (warp == 0) {
        const uint64_t key = lists[lane];
        const int kmax = min(kk, n_groups);
        const bool on = key != 0ull && ((a.shard_cands || fused) ? key >= thr : lane < kmax);
        const int c = on ? (int)(0xFFFFFFFFu - (uint32_t)key) - cbase : 0;
        const unsigned bal = __ballot_sync(0xffffffffu, on);
        const int nsel = __popc(bal);  // a prefix of the sorted list
        sel_s[lane] = on ? c : -1;
        const int exact = warp_sum_int(on ? len_s[c] : 0);
        if (a.cand_out) {  // shard candidates: the local top-k keys, zero-padded
            if (lane < kk) {
                const int64_t idx = ((int64_t)bh * g + h) * kk + lane;
                a.cand_out[idx] = on ? key : 0ull;
            }
        }
        if (lane == 0) {
            info_s[0] = nsel;
            info_s[1] = exact;
            info_s[2] = (sample_end - exact > 0) ? S : 0;
        }
    }
    if (a.cand_out) {  // the others may still read this CTA's keys
        cl_sync();
        return;
    }
    cl_sync();  // every head's selection is in place

    // ---- 3. union of the group's selections ------------------------------------
    int *ue_start = (int *)(work + 2 * grp_al16((size_t)Gmax * 4) + kGrpWarps * 32 * 8);
    int *ue_mask = ue_start + kGrpUnion, *ue_cid = ue_mask + kGrpUnion;
    int *ue_off = ue_cid + kGrpUnion;  // [kGrpUnion + 1]
    if (tid < g * 32) {
        const int hh = tid >> 5, j = tid & 31;
        all_sel[hh][j] = cl_ld_s32(cl_map(sel_s + j, (uint32_t)hh));
        if (j < 3) all_info[hh][j] = cl_ld_s32(cl_map(info_s + j, (uint32_t)hh));
    }
    __syncthreads();
    cl_arrive();  // done reading the other CTAs; the matching wait is at the end
    if (tid < g * 32) {
        const int hh = tid >> 5, j = tid & 31;
        if (j < all_info[hh][0]) atomicOr(&mask_s[all_sel[hh][j]], 1 << hh);
    }
    __syncthreads();
    {
        int m[4], cnt = 0, rows = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = 4 * tid + i;
            m[i] = c < n_groups ? mask_s[c] : 0;
            cnt += m[i] ? 1 : 0;
            rows += m[i] ? len_s[c] : 0;
        }
        int2 tot;
        const int2 ex = grp_block_scan2(cnt, rows, sw, tot);
        int ui = ex.x, ro = ex.y;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (m[i]) {
                const int c = 4 * tid + i;
                ue_start[ui] = starts_s[c];
                ue_mask[ui] = m[i];
                ue_cid[ui] = c;
                ue_off[ui] = ro;
                ++ui;
                ro += len_s[c];
            }
        }
        if (tid == 0) {
            s_nunion = tot.x;
            s_U = tot.y;
            ue_off[tot.x] = tot.y;
        }
    }
    __syncthreads();
    const int n_union = s_nunion, U = s_U;
    {
        // this CTA's share of the union entries; entry v of the expanded
        // row list = sorted row | (head mask << 24)
        int32_t *wr = a.ws.w_row + (int64_t)bh * sample_end;
        for (int j = rank * kGrpWarps + warp; j < n_union; j += g * kGrpWarps) {
            const int off = ue_off[j], len = ue_off[j + 1] - off;
            const int st = ue_start[j], tag = ue_mask[j] << 24;
            for (int r = lane; r < len; r += 32) wr[off + r] = (st + r) | tag;
            if (lane == 0) {
                a.ws.u_start[(int64_t)bh * Gmax + j] = st;
                a.ws.u_mask[(int64_t)bh * Gmax + j] = ue_mask[j];
                a.ws.u_cid[(int64_t)bh * Gmax + j] = ue_cid[j];
                a.ws.u_off[(int64_t)bh * (Gmax + 1) + j] = off;
            }
        }
    }
    const int R = a.geo.n_total - sample_end;
    int sbase = 0, ns_all = 0;
    for (int hh = 0; hh < g; ++hh) {
        if (hh < h) sbase += all_info[hh][2];
        ns_all += all_info[hh][2];
    }
    if (tid == 0) {
        if (rank == 0) {
            a.ws.u_off[(int64_t)bh * (Gmax + 1) + n_union] = U;
            int32_t *meta = a.ws.meta + (int64_t)bh * 8;
            meta[0] = n_union;
            meta[1] = U;
            meta[2] = R;
            meta[3] = ns_all;
            meta[4] = U + R + ns_all;
            a.ws.counters[bh] = 0;  // arrival counter of the attention merge
        }
        a.ws.head_meta[((int64_t)bh * 8 + h) * 2 + 0] = info_s[1];
        a.ws.head_meta[((int64_t)bh * 8 + h) * 2 + 1] = info_s[2];
        if (a.n_exact) a.n_exact[(int64_t)bh * g + h] = info_s[1];
    }

    // ---- 4. draws of head h -------------------------------------------------------
    const int ns = info_s[2];
    if (ns > 0) {
        const int cnt = info_s[0];
        if (warp == 0) {
            // selected clusters in ascending order (= ascending start) as
            // gap[j] = non-selected positions before cluster j and cum[j] =
            // selected positions before it: rank r maps to r + cum[J] with
            // J = #{j : gap[j] <= r}
            const int c = lane < cnt ? sel_s[lane] : 0x7FFFFFFF;
            int pos = 0;
            for (int i = 0; i < cnt; ++i) pos += __shfl_sync(0xffffffffu, c, i) < c ? 1 : 0;
            if (lane < cnt) sid[pos] = c;
            __syncwarp();
            const int cs = lane < cnt ? sid[lane] : 0;
            const int l = lane < cnt ? len_s[cs] : 0;
            int x = l;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (lane < cnt) {
                gap[lane] = starts_s[cs] - (x - l);
                cum[lane] = x - l;
            }
            if (lane == 31) cum[cnt] = x;
        }
        __syncthreads();
        const int gh = kv * g + h;  // global query head
        int32_t *spos = a.ws.s_pos + (int64_t)bh * g * S + sbase;
        float *soff = a.ws.s_off + (int64_t)bh * g * S + sbase;
        const int64_t inj = ((int64_t)b * a.geo.num_kv_heads * g + gh) * S;
        const uint2 key = make_uint2((uint32_t)a.p.seed, (uint32_t)(a.p.seed >> 32));
        const uint32_t stepw = (uint32_t)decode_step_word(a.p);
        const float logS = logf((float)ns);
        const int n_rest = sample_end - info_s[1];
        const float off = (logf((float)n_rest) - logS) * kLog2e;
        for (int i = tid; i < ns; i += kGrpThreads) {
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
    }
    // the attention kernel may be scheduled once every CTA of this grid got
    // here (its griddepcontrol.wait still waits for this grid's completion
    // and memory flush); triggered at the start instead, the attention CTAs
    // sat on the SMs this grid left free and the step measured 4-12 us slower
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    cl_wait();  // no CTA leaves while another may still read its shared memory
}

// The bulk copies need 16-byte aligned q rows and metadata rows.
bool select_group_supported(const DecodeArgs &a) {
    const uintptr_t al = (uintptr_t)a.q | (uintptr_t)a.sum.starts | (uintptr_t)a.sum.lengths |
                         (uintptr_t)a.sum.log_n | (uintptr_t)a.sum.centroids;
    return a.p.mode == SANTA_MODE_HYBRID && a.p.topk_clusters >= 1 &&
           a.p.topk_clusters <= kGrpMaxK && a.sum.max_groups <= SANTA_MAX_CLUSTERS &&
           (a.sum.max_groups & 3) == 0 && (al & 15) == 0 && a.geo.group >= 1 &&
           a.geo.group <= SANTA_MAX_GROUP && (a.geo.head_dim == 64 || a.geo.head_dim == 128);
}

template <int D>
static int launch_select_group_d(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.geo.group, (unsigned)BH, 1);
    cfg.blockDim = dim3(kGrpThreads, 1, 1);
    const GrpLayout L = grp_layout(a.sum.max_groups, a.geo.group, D);
    // at most ceil(CTAs / SMs) CTAs per SM: extra dynamic shared memory keeps
    // the cluster scheduler from packing CTAs onto a few SMs
    // (the kernel's static shared memory is a property of the code, the same
    // on every device; a thread-safe one-time initialisation)
    static const int static_smem = [] {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, decode_select_group_kernel<D>) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        return (int)fa.sharedSizeBytes;
    }();
    const int smem_sm = static_smem < 0 ? 0 : device_attr(cudaDevAttrMaxSharedMemoryPerMultiprocessor);
    const int smem_reserved = device_attr(cudaDevAttrReservedSharedMemoryPerBlock);
    size_t dyn = L.bytes;
    const int ctas = a.geo.group * BH;
    const int per_sm = (ctas + num_sms() - 1) / num_sms();
    if (smem_sm > 0 && per_sm <= 3) {
        const long cap = (long)smem_sm / per_sm - smem_reserved - static_smem - 256;
        const long lim = 227L * 1024 - static_smem;
        if (cap > (long)dyn) dyn = (size_t)(cap < lim ? cap : lim);
    }
    if (int st = ensure_dyn_smem((const void *)decode_select_group_kernel<D>, dyn)) return st;
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)a.geo.group;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (a.p2p.peers) {
        // The peer-memory form waits inside the kernel for the peers' keys of
        // each (sequence, query head): every cluster must be resident at once,
        // or a waiting cluster could hold the SMs that a cluster the peers
        // wait for needs.
        int max_clusters = 0;
        SANTA_CUDA_CHECK(
            cudaOccupancyMaxActiveClusters(&max_clusters, decode_select_group_kernel<D>, &cfg));
        if (max_clusters < BH) return SANTA_ERR_UNSUPPORTED;
    }
    SANTA_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_select_group_kernel<D>, a));
    return SANTA_OK;
}

int launch_select_group(DecodeArgs &a, cudaStream_t stream) {
    return a.geo.head_dim == 64 ? launch_select_group_d<64>(a, stream)
                                : launch_select_group_d<128>(a, stream);
}

}  // namespace santa
