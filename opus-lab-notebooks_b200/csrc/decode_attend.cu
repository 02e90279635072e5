// SANTA++ decode, attention phase over the work lists written by the
// selection phase (santapp_ruler/attention/santapp.py:412-427 for topk,
// :472-506 for the importance-sampled modes):
//
//   s      = k . q * scale                 per selected / sampled / recent row
//   lw     = s - log r (sampled rows), s (exact rows)
//   out    = sum_j exp(lw_j - m) v_j / sum_j exp(lw_j - m)   (with the 1/S
//            factor folded into the sampled rows' log weights)
//
// Two kernels:
//   decode_attend_gather_kernel  bf16 caches.  One CTA of 8 warps per SM; the
//       virtual row spaces of all (batch, KV head) segments are concatenated
//       and split over the CTAs in equal shares of a row cost (sampled rows,
//       scattered over the cache, cost 1.5x a contiguous cluster row).
//       Inside a CTA every warp works alone on every 8th 16-row tile: it
//       loads the tile's row entries (expanded union rows, the recent window,
//       sampled rows) three tiles ahead, gathers the K/V rows with
//       row-cooperative coalesced 16-byte cp.async copies into its own
//       3-stage ring of padded shared-memory tiles, and runs mma.sync
//       m16n8k16 with an online softmax.  GQA heads fill M rows 0-7 with the
//       bf16 hi part of q (or p) and rows 8-15 with the lo part, so one MMA
//       gives fp32-level accuracy.  No barrier crosses warps inside a
//       segment.  At a segment end each warp leaves its partial
//       (m, l, o[D]) in its drained ring, the CTA folds the 8 partials into
//       one CTA partial in global memory, and after the last segment the
//       last CTA of each segment (atomic counter) stages the segment's CTA
//       partials into shared memory and LSE-merges them into the output.
//       (Two earlier designs were measured slower on B200: one bulk copy per
//       256-byte row through the TMA engine is request-bound, and a single
//       producer warp cannot keep enough 16-byte copies in flight.)
//   decode_attend_simt_kernel  fp32 caches, a warp per row.
#include "decode_common.cuh"

#include <cuda.h>  // CUtensorMap (the encode entry point is fetched at run time)

#include <math.h>

namespace santa {

// ---------------------------------------------------------------------------
// SIMT kernel (fp32 caches): NSPLIT CTAs per segment
// ---------------------------------------------------------------------------
constexpr int kSimtThreads = 128;
constexpr int kSimtTileRows = 64;

template <int D, typename T>
__global__ void __launch_bounds__(kSimtThreads) decode_attend_simt_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int split = blockIdx.x, bh = blockIdx.y;
    const int g = a.geo.group, Gmax = a.sum.max_groups;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kSimtThreads / 32;
    WarpState<D> *ws4 = (WarpState<D> *)smem_raw;
    int *u_off = (int *)(ws4 + NW);
    int *u_start = u_off + Gmax + 1;
    int *u_mask = u_start + Gmax;
    float *qs = (float *)(u_mask + Gmax);  // [8][D], scaled by scale*log2e
    __shared__ int s_last;

    const int32_t *meta = a.ws.meta + (int64_t)bh * 8;
    const int n_union = meta[0], U = meta[1], R = meta[2], total = meta[4];
    for (int i = tid; i <= n_union; i += kSimtThreads)
        u_off[i] = a.ws.u_off[(int64_t)bh * (Gmax + 1) + i];
    for (int i = tid; i < n_union; i += kSimtThreads) {
        u_start[i] = a.ws.u_start[(int64_t)bh * Gmax + i];
        u_mask[i] = a.ws.u_mask[(int64_t)bh * Gmax + i];
    }
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    const float qscale = a.p.scale * kLog2e;
    for (int i = tid; i < g * D; i += kSimtThreads) qs[i] = qb[i] * qscale;
    __syncthreads();

    constexpr int PER = D / 32;
    float m[SANTA_MAX_GROUP], l[SANTA_MAX_GROUP], ms[SANTA_MAX_GROUP], e1[SANTA_MAX_GROUP],
        e2[SANTA_MAX_GROUP], o[SANTA_MAX_GROUP][PER];
#pragma unroll
    for (int h = 0; h < SANTA_MAX_GROUP; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
        ms[h] = -INFINITY;
        e1[h] = 0.f;
        e2[h] = 0.f;
#pragma unroll
        for (int j = 0; j < PER; ++j) o[h][j] = 0.f;
    }
    const int per = ceil_div(ceil_div(total, a.nsplit), kSimtTileRows) * kSimtTileRows;
    const int r0 = min(total, split * per), r1 = min(total, r0 + per);
    const int row_bytes = D * (int)sizeof(T);
    for (int v = r0 + warp; v < r1; v += NW) {
        const RowInfo ri = resolve_row(a, bh, v, U, R, total, n_union, u_off, u_start, u_mask,
                                       row_bytes);
        const T *kr = (const T *)ri.k;
        const T *vr = (const T *)ri.v;
        float kx[PER], vx[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            kx[j] = to_f32<T>(kr[lane + 32 * j]);
            vx[j] = to_f32<T>(vr[lane + 32 * j]);
        }
#pragma unroll
        for (int h = 0; h < SANTA_MAX_GROUP; ++h) {
            if (h < g && ((ri.mask >> h) & 1)) {
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < PER; ++j) s = fmaf(kx[j], qs[h * D + lane + 32 * j], s);
                s = warp_sum(s);
                const float lw = (ri.mask & kMaskAbs) ? ri.off : s + ri.off;
                float p;
                if (lw > m[h]) {
                    const float alpha = exp2f(m[h] - lw);
                    l[h] = l[h] * alpha + 1.f;
#pragma unroll
                    for (int j = 0; j < PER; ++j) o[h][j] *= alpha;
                    m[h] = lw;
                    p = 1.f;
                } else {
                    p = exp2f(lw - m[h]);
                    l[h] += p;
                }
#pragma unroll
                for (int j = 0; j < PER; ++j) o[h][j] = fmaf(p, vx[j], o[h][j]);
                if (ri.mask & kMaskSample) {
                    if (lw > ms[h]) {
                        const float f = exp2f(ms[h] - lw);
                        e1[h] = e1[h] * f + 1.f;
                        e2[h] = e2[h] * f * f + 1.f;
                        ms[h] = lw;
                    } else {
                        const float f = exp2f(lw - ms[h]);
                        e1[h] += f;
                        e2[h] += f * f;
                    }
                }
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int h = 0; h < SANTA_MAX_GROUP; ++h) {
            ws4[warp].m[h] = m[h];
            ws4[warp].l[h] = l[h];
            ws4[warp].ms[h] = ms[h];
            ws4[warp].e1[h] = e1[h];
            ws4[warp].e2[h] = e2[h];
        }
    }
#pragma unroll
    for (int h = 0; h < SANTA_MAX_GROUP; ++h)
#pragma unroll
        for (int j = 0; j < PER; ++j) ws4[warp].o[h][lane + 32 * j] = o[h][j];
    __syncthreads();
    const int PSTR = partial_stride(D);
    float *part = a.ws.partial + ((int64_t)bh * a.nsplit + split) * g * PSTR;
    merge_warp_states<D>(ws4, NW, g, part, tid, kSimtThreads);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.ws.counters[bh], 1) == a.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    merge_partials_to_output<D>(a, bh, a.ws.partial + (int64_t)bh * a.nsplit * g * PSTR,
                                a.nsplit, tid, kSimtThreads);
    if (tid == 0) a.ws.counters[bh] = 0;
}

// ---------------------------------------------------------------------------
// warp-independent gather kernel (bf16 caches)
// ---------------------------------------------------------------------------
constexpr int kGW = 8;        // warps per CTA
constexpr int kGRows = 16;    // rows per warp tile (the mma N/K granule)
constexpr int kGStages = 3;   // cp.async ring depth per warp
constexpr int kGThreads = 32 * kGW;
// balancing costs kCostRow / kCostSample / kCostSegment: decode_common.cuh

template <int D>
struct GatherGeom {
    static constexpr int ROWB = D * 2;                // bytes of one bf16 row
    static constexpr int BLOCKS = D / 64;             // 128-byte column blocks of a row
    static constexpr int TILE = kGRows * ROWB;        // one K (or V) warp tile
    static constexpr int STAGE = 2 * TILE;            // K + V; stages are 1024-byte aligned
    static constexpr int META = 2 * kGRows * 4;       // row masks + offsets of a stage
    static constexpr int WARP = (kGStages * (STAGE + META) + 1023) / 1024 * 1024;
    static constexpr int CPR = ROWB / 16;             // 16-byte chunks per row
    static constexpr int RPI = 32 / CPR;              // rows per copy instruction
};

// Tile layout in shared memory: column block b (bytes [128 b, 128 b + 128) of
// every row) is a [16 rows][128 bytes] block, and row r holds its 16-byte
// chunk j of the block at slot j ^ (r % 8) -- the 128-byte swizzle a tensor
// copy writes, which also keeps the eight rows of an ldmatrix phase on eight
// distinct bank groups.  Byte offset of chunk c (0 .. D / 8 - 1) of row r:
__device__ __forceinline__ int tile_off(int r, int c) {
    return (c >> 3) * (kGRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// 2-D tensor copy (TMA engine) of one [16 rows][64 bf16] box of this GPU's
// cluster-sorted K or V copy into shared memory, completing on an mbarrier;
// no multicast.  x = first column (0 or 64: 128-byte aligned), y = first row.
__device__ __forceinline__ void tma_box_g2s(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;\n"
        ::"r"(smem_u32(dst)), "l"((uint64_t)(uintptr_t)map), "r"(x), "r"(y), "r"(smem_u32(bar)),
        "l"(policy)
        : "memory");
}

template <int D>
inline size_t gather_smem_bytes(int BH) {
    // 1024-byte alignment, rings, segment prefix [BH + 1], completed-segment
    // bitmap [ceil(BH / 32)]
    return 1024 + (size_t)kGW * GatherGeom<D>::WARP + ((size_t)BH + 1) * 4 +
           (size_t)((BH + 31) / 32) * 4;
}

// One merged output element (head hh, dim dd) of segment bh: out / lse / ess,
// or the unnormalised partial for a sequence shard (ns: the head's sample
// count, used where dd == 0).
template <int D>
__device__ __forceinline__ void write_merged(const DecodeArgs &a, int bh, int hh, int dd, float acc,
                                             float M, float L, float MS, float E1, float E2,
                                             int ns, float inv_l) {
    const int g = a.geo.group, PSTR = partial_stride(D);
    const int64_t oh = (int64_t)bh * g + hh;  // (b * Hkv + kv) * g + hh
    if (a.part_out) {  // sequence shard: the unnormalised partial
        float *po = a.part_out + oh * PSTR;
        po[8 + dd] = acc;
        if (dd == 0) {
            po[0] = M;
            po[1] = L;
            po[2] = MS;
            po[3] = E1;
            po[4] = E2;
            po[5] = (float)ns;
            po[6] = 0.f;
            po[7] = 0.f;
        }
        return;
    }
    a.out[oh * D + dd] = acc * inv_l;
    if (dd == 0) {
        if (a.lse) a.lse[oh] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
        if (a.ess) a.ess[oh] = (ns > 0 && E2 > 0.f) ? (E1 * E1 / E2) / (float)ns : 0.f;
    }
}

// LSE merge of `count` partials (header m, l, ms, e1, e2 at [0, 5), values
// at [8, 8 + D) per head, heads PSTR floats apart) that lie `wstride` floats
// apart from `src`, into out / lse / ess of segment bh.  The whole CTA
// (kGThreads threads) calls it.  Up to 32 partials at a time are staged into
// `stage` with one batch of 16-byte cp.async; one thread per head then
// computes that head's factors for the batch (a short sequential loop, no
// warp reductions on the critical path) into shared memory, and after one
// barrier every thread runs the FMA pass over its output elements.
template <int D>
__device__ void merge_staged_to_output(const DecodeArgs &a, int bh, const float *src, int count,
                                       int wstride, float *stage, int stage_floats) {
    constexpr int NT = kGThreads;
    constexpr int OPT = (SANTA_MAX_GROUP * D + NT - 1) / NT;
    __shared__ float s_f[SANTA_MAX_GROUP][32], s_r[SANTA_MAX_GROUP];
    __shared__ float s_M[SANTA_MAX_GROUP], s_L[SANTA_MAX_GROUP], s_MS[SANTA_MAX_GROUP];
    __shared__ float s_E1[SANTA_MAX_GROUP], s_E2[SANTA_MAX_GROUP];
    const int g = a.geo.group, PSTR = partial_stride(D);
    const int tid = threadIdx.x;
    const int cap = min(32, stage_floats / wstride);
    float acc[OPT];
#pragma unroll
    for (int k = 0; k < OPT; ++k) acc[k] = 0.f;
    if (tid < g) {
        s_M[tid] = -INFINITY;
        s_MS[tid] = -INFINITY;
        s_L[tid] = s_E1[tid] = s_E2[tid] = 0.f;
    }
    for (int s0 = 0; s0 < count; s0 += cap) {
        const int n = min(cap, count - s0);
        const int n16 = n * wstride / 4;
        for (int i = tid; i < n16; i += NT)
            cp_async16(stage + 4 * i, src + (int64_t)s0 * wstride + 4 * i);
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();
        if (tid < g) {  // this batch's factors of head tid
            const int hh = tid;
            float Mn = s_M[hh], MSn = s_MS[hh];
            for (int s = 0; s < n; ++s) {
                const float *hs = stage + s * wstride + hh * PSTR;
                if (hs[1] > 0.f) Mn = fmaxf(Mn, hs[0]);
                if (hs[3] > 0.f) MSn = fmaxf(MSn, hs[2]);
            }
            const float r = s_M[hh] == -INFINITY ? 0.f : exp2f(s_M[hh] - Mn);
            const float re = s_MS[hh] == -INFINITY ? 0.f : exp2f(s_MS[hh] - MSn);
            float L = s_L[hh] * r, E1 = s_E1[hh] * re, E2 = s_E2[hh] * re * re;
            for (int s = 0; s < n; ++s) {
                const float *hs = stage + s * wstride + hh * PSTR;
                const float f = hs[1] > 0.f ? exp2f(hs[0] - Mn) : 0.f;
                s_f[hh][s] = f;
                L = fmaf(hs[1], f, L);
                if (hs[3] > 0.f) {
                    const float fe = exp2f(hs[2] - MSn);
                    E1 = fmaf(hs[3], fe, E1);
                    E2 = fmaf(hs[4], fe * fe, E2);
                }
            }
            s_r[hh] = r;
            s_M[hh] = Mn;
            s_MS[hh] = MSn;
            s_L[hh] = L;
            s_E1[hh] = E1;
            s_E2[hh] = E2;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < OPT; ++k) {
            const int i = tid + k * NT;
            if (i < g * D) {
                const int hh = i / D, col = hh * PSTR + 8 + (i - hh * D);
                float v = acc[k] * s_r[hh];
                for (int s = 0; s < n; ++s) v = fmaf(s_f[hh][s], stage[s * wstride + col], v);
                acc[k] = v;
            }
        }
        __syncthreads();  // the next batch overwrites the stage and the factors
    }
    float M[OPT], L[OPT], MS[OPT], E1[OPT], E2[OPT];
#pragma unroll
    for (int k = 0; k < OPT; ++k) {
        const int hh = min(tid + k * NT, g * D - 1) / D;
        M[k] = s_M[hh];
        L[k] = s_L[hh];
        MS[k] = s_MS[hh];
        E1[k] = s_E1[hh];
        E2[k] = s_E2[hh];
    }
#pragma unroll
    for (int k = 0; k < OPT; ++k) {
        const int i = tid + k * NT;
        if (i < g * D) {
            const int hh = i / D;
            write_merged<D>(a, bh, hh, i - hh * D, acc[k], M[k], L[k], MS[k], E1[k], E2[k],
                            i - hh * D == 0 ? a.ws.head_meta[((int64_t)bh * 8 + hh) * 2 + 1] : 0,
                            L[k] > 0.f ? 1.f / L[k] : 0.f);
        }
    }
}

// All the segments a CTA completes, merged together: their partials staged
// in one cp.async batch (segment i's `count[i]` partials from `first[i]`);
// the factors of each (segment, head) computed by one warp, a lane per
// partial (maxima and sums by shuffles); then every thread forms its output
// elements' sums (factor-weighted, ascending partial order) before any of its
// stores.  The caller checks that every count is at most 32, that there are
// at most kMergeSegs segments and that all partials fit the stage.
constexpr int kMergeSegs = 4;
template <int D>
__device__ void merge_segments_to_output(const DecodeArgs &a, const int *seg, const int *first,
                                         const int *count, int nseg, int wstride, float *stage) {
    constexpr int NT = kGThreads;
    constexpr int IPT = (SANTA_MAX_GROUP * D + NT - 1) / NT;  // output elements per thread
    __shared__ float s_f[kMergeSegs][SANTA_MAX_GROUP][32];
    __shared__ float s_hdr[kMergeSegs][SANTA_MAX_GROUP][8];  // M L MS E1 E2 n_samples 1/L
    const int g = a.geo.group, PSTR = partial_stride(D);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npairs = nseg * g;
    auto off_of = [&](int si) {  // stage slot of segment si's first partial
        int o = 0;
        for (int i = 0; i < si; ++i) o += count[i];
        return o;
    };
    // the sample counts of this warp's (segment, head) pairs warp + 8k, lane
    // k requesting pair k's before the staging round trip so the two overlap
    int my_ns = 0;
    if (lane < 4 && warp + kGW * lane < npairs) {
        const int p = warp + kGW * lane, si = p / g;
        my_ns = a.ws.head_meta[((int64_t)seg[si] * 8 + (p - si * g)) * 2 + 1];
    }
    // stage every segment's partials (stage slot off[i] + j = partial j of segment i)
    for (int i = 0, o = 0; i < nseg; o += count[i++]) {
        const float *src = a.ws.partial + ((int64_t)first[i] + seg[i]) * wstride;
        const int n16 = count[i] * wstride / 4;
        for (int c = tid; c < n16; c += NT) cp_async16(stage + o * wstride + 4 * c, src + 4 * c);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // npairs <= kMergeSegs * 8 = 4 * kGW
        const int p = warp + kGW * k;
        const int ns = __shfl_sync(0xffffffffu, my_ns, k);
        if (p >= npairs) break;  // warp-uniform
        const int si = p / g, hh = p - si * g, n = count[si];
        float m = -INFINITY, l = 0.f, ms = -INFINITY, e1 = 0.f, e2 = 0.f;
        if (lane < n) {
            const float *hs = stage + (off_of(si) + lane) * wstride + hh * PSTR;
            m = hs[0];
            l = hs[1];
            ms = hs[2];
            e1 = hs[3];
            e2 = hs[4];
        }
        float M = l > 0.f ? m : -INFINITY, MS = e1 > 0.f ? ms : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            MS = fmaxf(MS, __shfl_xor_sync(0xffffffffu, MS, o));
        }
        const float f = l > 0.f ? exp2f(m - M) : 0.f;
        const float fe = e1 > 0.f ? exp2f(ms - MS) : 0.f;
        float L = l * f, E1 = e1 * fe, E2 = e2 * fe * fe;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            L += __shfl_xor_sync(0xffffffffu, L, o);
            E1 += __shfl_xor_sync(0xffffffffu, E1, o);
            E2 += __shfl_xor_sync(0xffffffffu, E2, o);
        }
        s_f[si][hh][lane] = f;
        if (lane == 0) {
            float *hd = s_hdr[si][hh];
            hd[0] = M;
            hd[1] = L;
            hd[2] = MS;
            hd[3] = E1;
            hd[4] = E2;
            hd[5] = (float)ns;
            hd[6] = L > 0.f ? 1.f / L : 0.f;
        }
    }
    __syncthreads();
    for (int si = 0; si < nseg; ++si) {
        const int n = count[si], bh = seg[si];
        const float *sb = stage + off_of(si) * wstride + 8;
        float acc[IPT];
#pragma unroll
        for (int k = 0; k < IPT; ++k) {
            const int j = tid + k * NT;
            acc[k] = 0.f;
            if (j < g * D) {
                const int hh = j / D, dd = j - hh * D;
                const float *v = sb + hh * PSTR + dd;
                const float *fs = s_f[si][hh];
                float x = 0.f;
                for (int s = 0; s < n; ++s) x = fmaf(fs[s], v[s * wstride], x);
                acc[k] = x;
            }
        }
#pragma unroll
        for (int k = 0; k < IPT; ++k) {
            const int j = tid + k * NT;
            if (j < g * D) {
                const int hh = j / D;
                const float *hd = s_hdr[si][hh];
                write_merged<D>(a, bh, hh, j - hh * D, acc[k], hd[0], hd[1], hd[2], hd[3], hd[4],
                                (int)hd[5], hd[6]);
            }
        }
    }
}

// The segments a CTA completes when each has at most kDirectMax partials:
// one warp per (segment, head), a lane per VPL = D / 32 consecutive dims.
// Every header and value of the pair is loaded in one batch straight from
// the partial slots (no staging, no barrier: the whole merge is one L2 round
// trip), then the factors and sums are formed in ascending partial order as
// in the staged merges (the maximum over the non-empty partials,
// f_s = 2^(m_s - M), L = sum f_s l_s, acc = sum f_s v_s).  One pair per
// pass: the merge runs once per kernel, as the last code a CTA fetches, and
// a second unrolled pair doubled the instructions it fetched.
constexpr int kDirectMax = 8;
template <int D>
__device__ void merge_pairs_direct(const DecodeArgs &a, const int *seg, const int *first,
                                   const int *count, int nseg, int wstride) {
    constexpr int VPL = D / 32;
    const int g = a.geo.group, PSTR = partial_stride(D);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npairs = nseg * g;
    for (int p = warp; p < npairs; p += kGW) {
        const int si = p / g, hh = p - si * g;
        const int n = count[si], bh = seg[si];
        const int ns = lane == 0 ? a.ws.head_meta[((int64_t)bh * 8 + hh) * 2 + 1] : 0;
        const float *src = a.ws.partial + ((int64_t)first[si] + bh) * wstride + hh * PSTR;
        float mv[kDirectMax], lv[kDirectMax], vv[kDirectMax][VPL];
        float xs[kDirectMax][3];  // ms e1 e2 (lane 0)
#pragma unroll
        for (int s = 0; s < kDirectMax; ++s) {
            mv[s] = -INFINITY;
            lv[s] = 0.f;
            xs[s][0] = -INFINITY;
            xs[s][1] = xs[s][2] = 0.f;
#pragma unroll
            for (int e = 0; e < VPL; ++e) vv[s][e] = 0.f;
            if (s < n) {
                const float *ps = src + (int64_t)s * wstride;
                mv[s] = ps[0];
                lv[s] = ps[1];
                if constexpr (VPL == 4) {
                    const float4 x = *(const float4 *)(ps + 8 + 4 * lane);
                    vv[s][0] = x.x;
                    vv[s][1] = x.y;
                    vv[s][2] = x.z;
                    vv[s][3] = x.w;
                } else {
                    const float2 x = *(const float2 *)(ps + 8 + 2 * lane);
                    vv[s][0] = x.x;
                    vv[s][1] = x.y;
                }
                if (lane == 0) {
                    xs[s][0] = ps[2];
                    xs[s][1] = ps[3];
                    xs[s][2] = ps[4];
                }
            }
        }
        float M = -INFINITY, MS = -INFINITY;
#pragma unroll
        for (int s = 0; s < kDirectMax; ++s) {
            if (lv[s] > 0.f) M = fmaxf(M, mv[s]);
            if (xs[s][1] > 0.f) MS = fmaxf(MS, xs[s][0]);
        }
        float L = 0.f, E1 = 0.f, E2 = 0.f, acc[VPL];
#pragma unroll
        for (int e = 0; e < VPL; ++e) acc[e] = 0.f;
#pragma unroll
        for (int s = 0; s < kDirectMax; ++s) {
            const float f = lv[s] > 0.f ? exp2f(mv[s] - M) : 0.f;
            L = fmaf(lv[s], f, L);
#pragma unroll
            for (int e = 0; e < VPL; ++e) acc[e] = fmaf(f, vv[s][e], acc[e]);
            if (xs[s][1] > 0.f) {
                const float fe = exp2f(xs[s][0] - MS);
                E1 = fmaf(xs[s][1], fe, E1);
                E2 = fmaf(xs[s][2], fe * fe, E2);
            }
        }
        const float inv_l = L > 0.f ? 1.f / L : 0.f;
        if (!a.part_out && ((uintptr_t)a.out & 15) == 0) {
            // one vector store per lane: the warp writes the head's row whole
            float *o = a.out + ((int64_t)bh * g + hh) * D + VPL * lane;
            if constexpr (VPL == 4)
                *(float4 *)o = make_float4(acc[0] * inv_l, acc[1] * inv_l, acc[2] * inv_l,
                                           acc[3] * inv_l);
            else
                *(float2 *)o = make_float2(acc[0] * inv_l, acc[1] * inv_l);
            if (lane == 0)  // lse / ess (and the dim-0 value again, identical)
                write_merged<D>(a, bh, hh, 0, acc[0], M, L, MS, E1, E2, ns, inv_l);
        } else {
#pragma unroll
            for (int e = 0; e < VPL; ++e)
                write_merged<D>(a, bh, hh, VPL * lane + e, acc[e], M, L, MS, E1, E2, ns, inv_l);
        }
    }
}

// Peer-memory exchange of the shard partials, fused into the attention
// kernel (the segments `done` marks, which this CTA merged into this rank's
// partial rows in the stage area).  Every CTA first sends all of its rows to
// every rank (16-byte lines, each 8-byte word tagged with the epoch), and
// only then waits for the other ranks' rows of the same segments: no CTA
// waits before it has sent, so every wait ends once the peers' kernels reach
// their own tails (all CTAs of this kernel are resident: one per SM).  Then
// one warp per (segment, query head) merges the ranks' partials in ascending
// rank order (the merge kernel's arithmetic, so both exchange paths give the
// same bits) into out / lse / ess.  A wait that runs out of time sets the
// error flag and the rows it could not complete, and every row after it in
// this CTA, come out NaN.
template <int D>
__device__ void fused_shard_exchange(const DecodeArgs &a, const unsigned *done, int BH,
                                     float *hdr_smem) {
    constexpr int VPL = D / 32, LPL = VPL / 2;
    const int g = a.geo.group, pf = partial_stride(D), pl = pf / 2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = a.p2p.n;
    const uint32_t tag = (uint32_t)a.p2p.epoch;
    const uint64_t tg = (uint64_t)tag << 32;
    const float *stage = a.part_out;
    // 1. send: lines of each completed segment's g rows, to every rank
    for (int w = 0; w < (BH + 31) / 32; ++w) {
        for (unsigned m = done[w]; m; m &= m - 1) {
            const int bh = 32 * w + __ffs(m) - 1;
            const int nl = g * pl;  // lines of the segment (rows bh*g .. bh*g+g-1 are contiguous)
            const float2 *src = (const float2 *)(stage + (int64_t)bh * g * pf);
            for (int i = tid; i < n * nl; i += kGThreads) {
                const int r = i / nl, j = i - r * nl;
                const float2 v = src[j];
                st_relaxed_sys_v2(p2p_part_slot(a.p2p, a.p2p.peers[r], a.p2p.rank) +
                                      (int64_t)bh * g * pl + j,
                                  tg | __float_as_uint(v.x), tg | __float_as_uint(v.y));
            }
        }
    }
    // 2. wait and merge: one warp per (segment, head)
    volatile int32_t *errp = a.p2p.err;
    bool ok = *errp == 0;  // a wait of the selection already gave up: NaN rows
    const uint64_t t0 = p2p_now_ns();
    float *sh = hdr_smem + warp * (SANTA_MAX_SHARDS * 8);  // [rank][8] headers
    int k = 0;
    for (int w = 0; w < (BH + 31) / 32; ++w) {
        for (unsigned m = done[w]; m; m &= m - 1) {
            const int bh = 32 * w + __ffs(m) - 1;
            for (int hh = 0; hh < g; ++hh, ++k) {
                if ((k % kGW) != warp) continue;
                const int64_t oh = (int64_t)bh * g + hh;
                // headers: lane -> rank r0 + lane / 4, line lane % 4 (lines 0-2
                // hold m l ms e1 e2 samples)
                for (int r0 = 0; r0 < n; r0 += 8) {
                    const int r = r0 + (lane >> 2), j = lane & 3;
                    if (r < n && j < 3) {
                        const float2 v = ll_part_wait(
                            a.p2p, p2p_part_slot(a.p2p, a.p2p.local, r) + oh * pl + j, tag, t0, ok);
                        sh[r * 8 + 2 * j] = v.x;
                        sh[r * 8 + 2 * j + 1] = v.y;
                    }
                }
                __syncwarp();
                const ShardMerged s =
                    shard_merge_header(n, [&](int r, int j) { return sh[r * 8 + j]; });
                float acc[VPL];
#pragma unroll
                for (int e = 0; e < VPL; ++e) acc[e] = 0.f;
                for (int r0 = 0; r0 < n; r0 += 8) {
                    ulonglong2 v[8][LPL];
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr) {  // one batch of loads
                        if (r0 + rr < n) {
                            const ulonglong2 *p = p2p_part_slot(a.p2p, a.p2p.local, r0 + rr) +
                                                  oh * pl + 4 + LPL * lane;
#pragma unroll
                            for (int e = 0; e < LPL; ++e) v[rr][e] = ld_relaxed_sys_v2(p + e);
                        }
                    }
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr) {
                        const int r = r0 + rr;
                        if (r >= n || !(sh[r * 8 + 1] > 0.f)) continue;
                        const float f = exp2f(sh[r * 8] - s.M);
                        const ulonglong2 *p =
                            p2p_part_slot(a.p2p, a.p2p.local, r) + oh * pl + 4 + LPL * lane;
#pragma unroll
                        for (int e = 0; e < LPL; ++e) {
                            float2 x;
                            if ((uint32_t)(v[rr][e].x >> 32) == tag &&
                                (uint32_t)(v[rr][e].y >> 32) == tag)
                                x = make_float2(__uint_as_float((uint32_t)v[rr][e].x),
                                                __uint_as_float((uint32_t)v[rr][e].y));
                            else
                                x = ll_part_wait(a.p2p, p + e, tag, t0, ok);
                            acc[2 * e] = fmaf(x.x, f, acc[2 * e]);
                            acc[2 * e + 1] = fmaf(x.y, f, acc[2 * e + 1]);
                        }
                    }
                }
                ok = __all_sync(0xffffffffu, ok);
                const float sc = shard_out_scale(s);
                const float nan = __int_as_float(0x7FC00000);
                float *o = a.out + oh * D + VPL * lane;
                if constexpr (VPL == 4)
                    *(float4 *)o = ok ? make_float4(acc[0] * sc, acc[1] * sc, acc[2] * sc,
                                                    acc[3] * sc)
                                      : make_float4(nan, nan, nan, nan);
                else
                    *(float2 *)o = ok ? make_float2(acc[0] * sc, acc[1] * sc)
                                      : make_float2(nan, nan);
                if (lane == 0) {
                    if (a.lse) a.lse[oh] = ok ? shard_lse(s) : nan;
                    if (a.ess) a.ess[oh] = ok ? shard_ess(s) : nan;
                }
                __syncwarp();  // sh is rewritten by the warp's next row
            }
        }
    }
}

// A row entry prefetched ahead of its copy.
struct RowEntry {
    int kind;   // 0 none, 1 union row, 2 recent row, 3 sampled row
    int32_t e;  // union: row | mask << 24; recent: cache row; sampled: packed sample word
    float off;
};

__device__ __forceinline__ RowEntry load_entry(const DecodeArgs &a, int bh, int v, int s1, int U,
                                               int R) {
    RowEntry r;
    r.kind = 0;
    r.e = 0;
    r.off = 0.f;
    if (v >= s1) return r;
    if (v < U) {
        r.kind = 1;
        r.e = a.ws.w_row[(int64_t)bh * a.geo.sample_end + v];
    } else if (v < U + R) {
        r.kind = 2;
        r.e = (int32_t)cache_row(a.geo, bh, a.geo.sample_end + (v - U));
    } else {
        const int64_t j = (int64_t)bh * a.geo.group * a.p.samples + (v - U - R);
        r.kind = 3;
        r.e = a.ws.s_pos[j];
        r.off = a.ws.s_off[j];
    }
    return r;
}

template <int D>
__global__ void __launch_bounds__(kGThreads, 1)
    decode_attend_gather_kernel(DecodeArgs a, const __grid_constant__ CUtensorMap tmap_k,
                                const __grid_constant__ CUtensorMap tmap_v) {
    using GG = GatherGeom<D>;
    constexpr int NT_O = D / 8;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int g = a.geo.group;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gid = lane >> 2, tig = lane & 3;

    unsigned char *base = (unsigned char *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char *wbase = base + warp * GG::WARP;     // this warp's ring: stages, then metas
    // one mbarrier per stage of every warp: completion of a stage's tensor copies
    __shared__ __align__(8) uint64_t s_tma_bar[kGW][kGStages];
    uint64_t *wbar = s_tma_bar[warp];
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < kGStages; ++st) mbar_init(&wbar[st], 1);
        mbar_fence_init();
    }
    __syncwarp();
    uint32_t tma_pending = 0u, tma_phase = 0u;  // per stage: copies in flight, barrier parity
    int *pre = (int *)(base + kGW * GG::WARP);         // segment prefix [BH + 1]
    unsigned *done_bits = (unsigned *)(pre + BH + 1);  // segments this CTA merged (p2p)
    const bool fused = a.p2p.peers != nullptr;
    __shared__ float s_wfac[SANTA_MAX_GROUP][kGW];     // CTA fold: factor per head and warp
    // The merge path reads the arguments from a shared-memory copy: after the
    // row loops the constant cache no longer holds the fields only it uses
    // (outputs, counters, partial slots), and each first touch of one costs a
    // round trip on the tail's critical path.
    __shared__ __align__(16) DecodeArgs s_args;
    if (tid == kGThreads - 1) s_args = a;
    // the tensor maps are kernel parameters, not outputs of the selection
    if (a.tma && tid == 0) {
        asm volatile("prefetch.tensormap [%0];\n" ::"l"((uint64_t)(uintptr_t)&tmap_k) : "memory");
        asm volatile("prefetch.tensormap [%0];\n" ::"l"((uint64_t)(uintptr_t)&tmap_v) : "memory");
    }
    // Launched as a programmatic dependent of the selection kernel, which
    // triggers it as its CTAs finish: everything below reads what the
    // selection wrote, so wait for that grid to complete (a no-op when the
    // launch had no such dependency).
    asm volatile("griddepcontrol.wait;\n" ::: "memory");

    {
        // segment cost prefix, 256 segments per round over the whole CTA
        // (one round of loads instead of a warp walking the segments)
        __shared__ int s_wtot[kGW];
        int carry = 0;
        for (int c0 = 0; c0 < BH; c0 += kGThreads) {
            const int i = c0 + tid;
            // segment cost: kCostRow per union / recent row, kCostSample per
            // sampled row (scattered rows stream ~1.5x slower than contiguous
            // cluster rows)
            const int rows = i < BH ? a.ws.meta[(int64_t)i * 8 + 4] : 0;
            int x = i < BH ? kCostRow * rows +
                                 (kCostSample - kCostRow) * a.ws.meta[(int64_t)i * 8 + 3] +
                                 (rows > 0 ? kCostSegment : 0)
                           : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (lane == 31) s_wtot[warp] = x;
            __syncthreads();
            int before = 0, total = 0;
#pragma unroll
            for (int w = 0; w < kGW; ++w) {
                const int v = s_wtot[w];
                before += w < warp ? v : 0;
                total += v;
            }
            if (i < BH) pre[i + 1] = carry + before + x;
            carry += total;
            __syncthreads();  // s_wtot is rewritten by the next round
        }
        if (tid == 0) pre[0] = 0;
        if (fused)
            for (int i = tid; i < (BH + 31) / 32; i += kGThreads) done_bits[i] = 0u;
    }
    __syncthreads();  // the prefix and the done bits are in place

    // every CTA takes an equal share [r0, r1) of the total cost; within a
    // segment (after its kCostSegment start charge), row v starts at cost
    // kCostRow * v (union and recent rows) or kCostRow * (U + R) +
    // kCostSample * (v - U - R) (sampled rows), and belongs to the CTA whose
    // share holds that start
    const int T_all = pre[BH];
    const int P = max(1, ceil_div(T_all, (int)gridDim.x));
    const int r0 = min(T_all, (int)blockIdx.x * P);
    const int r1 = min(T_all, r0 + P);
    auto row_at_cost = [](int c, int ur) {  // first row whose cost start is >= c
        return c <= kCostRow * ur ? ceil_div(c, kCostRow)
                                  : ur + ceil_div(c - kCostRow * ur, kCostSample);
    };
    // first segment whose cost range ends after r0 (pre is non-decreasing; a
    // binary search: a walk from segment 0 put the CTAs of the last segments
    // microseconds behind the first ones)
    int bh0 = 0;
    {
        int hi = BH;
        while (bh0 < hi) {
            const int mid = (bh0 + hi) >> 1;
            if (pre[mid + 1] <= r0) bh0 = mid + 1;
            else hi = mid;
        }
    }
    // U and R of the next segment the loop meets, loaded one segment ahead
    int nx_bh = bh0, nx_U = 0, nx_R = 0;
    if (bh0 < BH) {
        nx_U = a.ws.meta[(int64_t)bh0 * 8 + 1];
        nx_R = a.ws.meta[(int64_t)bh0 * 8 + 2];
    }

    const float qscale = a.p.scale * kLog2e;
    const int PSTR = partial_stride(D);
    // K / V rows are read once per step: their copies carry an L2 evict-first
    // policy, so the streaming does not push the CTA partials (written as
    // segments end, read by the merging CTA up to a whole loop later) and the
    // row tables out of L2
    uint64_t kv_policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(kv_policy));
    const char *sk_all = (const char *)a.sum.sorted_key;
    const char *sv_all = (const char *)a.sum.sorted_value;
    int k_base = 0;  // CTA tiles before the current segment
    for (int bh = bh0; bh < BH && pre[bh] < r1; ++bh) {
        const int seg0 = pre[bh], total = pre[bh + 1] - seg0;
        const int c0 = max(r0, seg0) - seg0, c1 = min(r1, seg0 + total) - seg0;
        // a CTA whose share meets the segment takes part in its merge even
        // when the share holds no row start (its warps write empty partials)
        if (c0 >= c1) continue;
        int U, R;
        if (bh == nx_bh) {
            U = nx_U;
            R = nx_R;
        } else {
            U = a.ws.meta[(int64_t)bh * 8 + 1];
            R = a.ws.meta[(int64_t)bh * 8 + 2];
        }
        if (bh + 1 < BH && pre[bh + 1] < r1) {  // the next segment's, while this one runs
            nx_bh = bh + 1;
            nx_U = a.ws.meta[(int64_t)(bh + 1) * 8 + 1];
            nx_R = a.ws.meta[(int64_t)(bh + 1) * 8 + 2];
        }
        const int s0 = row_at_cost(max(0, c0 - kCostSegment), U + R);
        const int s1 = row_at_cost(max(0, c1 - kCostSegment), U + R);
        const int nt = ceil_div(s1 - s0, kGRows);
        const int j0 = ((warp - k_base) % kGW + kGW) % kGW;  // my first tile in the segment
        const int n_my = nt > j0 ? ceil_div(nt - j0, kGW) : 0;
        k_base += nt;
        const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
        const char *sk = sk_all + (int64_t)bh * a.geo.sample_end * GG::ROWB;
        const char *sv = sv_all + (int64_t)bh * a.geo.sample_end * GG::ROWB;
        const char *ck = a.key_cache, *cv = a.value_cache;  // recent rows: cache_row codes

        // q fragments of this (batch, KV head): rows = heads, split bf16 hi + lo
        const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
        uint32_t qh[D / 16][2], ql[D / 16][2];
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int d = 16 * ks + 8 * half + 2 * tig;
                float x0 = 0.f, x1 = 0.f;
                if (gid < g) {
                    const float2 v = *(const float2 *)(qb + gid * D + d);
                    x0 = v.x * qscale;
                    x1 = v.y * qscale;
                }
                const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
                qh[ks][half] = pack_bf16(__bfloat162float(h0), __bfloat162float(h1));
                ql[ks][half] = pack_bf16(x0 - __bfloat162float(h0), x1 - __bfloat162float(h1));
            }
        }
        float m_run = -INFINITY, l_run = 0.f, ms_run = -INFINITY, e1_run = 0.f, e2_run = 0.f;
        float o[NT_O][4];
#pragma unroll
        for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

        // first virtual row of my i-th tile
        auto tile_row0 = [&](int i) { return s0 + (j0 + i * kGW) * kGRows; };
        // issue the copies of my i-th tile into stage st from its prefetched entry
        auto issue = [&](int i, int st, const RowEntry &en) {
            unsigned char *stg = wbase + st * GG::STAGE;
            int *mk = (int *)(wbase + kGStages * GG::STAGE + st * GG::META);
            float *of = (float *)(mk + kGRows);
            // row code: >= 0 row of the cluster-sorted copy, -1 - x row x of
            // the cache (a recent-window token), INT_MIN no row
            int code = INT_MIN, mask = 0;
            if (en.kind == 1) {
                code = en.e & (int)kPosMask;
                mask = (int)((uint32_t)en.e >> 24);
            } else if (en.kind == 2) {
                code = -1 - en.e;
                mask = (1 << g) - 1;
            } else if (en.kind == 3) {
                const uint32_t pk = (uint32_t)en.e;
                code = (int)(pk & kPosMask);
                mask = (1 << ((pk >> kHeadShift) & 7u)) | kMaskSample |
                       ((pk & kAbsBit) ? kMaskAbs : 0);
            }
            if (lane < kGRows) {
                mk[lane] = mask;
                of[lane] = en.off;
            }
            // sixteen consecutive rows of the cluster-sorted copy (a run of
            // adjacent selected clusters): the tile moves as 2 * D / 64 tensor
            // copies issued by one lane, completing on the stage's mbarrier
            const int code0 = __shfl_sync(0xffffffffu, code, 0);
            const bool run = a.tma && __all_sync(0xffffffffu, lane >= kGRows ||
                                                               (en.kind == 1 && code == code0 + lane));
            if (run) {
                if (lane == 0) {
                    uint64_t *bar = &wbar[st];
                    // the stage's earlier generic-proxy reads and writes come first
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(bar, (uint32_t)GG::STAGE);
                    const int y = bh * a.geo.sample_end + code0;
#pragma unroll
                    for (int blk = 0; blk < GG::BLOCKS; ++blk) {
                        tma_box_g2s(stg + blk * kGRows * 128, &tmap_k, 64 * blk, y, bar, kv_policy);
                        tma_box_g2s(stg + GG::TILE + blk * kGRows * 128, &tmap_v, 64 * blk, y, bar,
                                    kv_policy);
                    }
                }
                tma_pending |= 1u << st;
                (void)i;
                return;
            }
            // otherwise row-cooperative 16-byte copies: CPR lanes cover one
            // row, so every instruction moves RPI whole rows (few cache lines
            // per request; mapping a lane pair to each row instead measured
            // 40% slower)
            const int c = lane % GG::CPR;
#pragma unroll
            for (int it = 0; it < kGRows / GG::RPI; ++it) {
                const int r = it * GG::RPI + lane / GG::CPR;
                const int rc = __shfl_sync(0xffffffffu, code, r);
                const char *ks = rc >= 0 ? sk + (int64_t)rc * GG::ROWB
                                         : ck + (int64_t)(rc == INT_MIN ? 0 : -1 - rc) * GG::ROWB;
                // byte distance from the K row to the V row of the same source
                const int64_t dv = rc >= 0 ? (int64_t)((uintptr_t)sv - (uintptr_t)sk)
                                           : (int64_t)((uintptr_t)cv - (uintptr_t)ck);
                const int ok = rc == INT_MIN ? 0 : 16;
                const uint32_t kd = smem_u32(stg + tile_off(r, c));
                asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(kd),
                             "l"(ks + c * 16), "r"(ok), "l"(kv_policy)
                             : "memory");
                asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(kd + GG::TILE),
                             "l"(ks + dv + c * 16), "r"(ok), "l"(kv_policy)
                             : "memory");
            }
            (void)i;
        };
        auto entry_of = [&](int i) {
            RowEntry en;
            en.kind = 0;
            en.e = 0;
            en.off = 0.f;
            if (i < n_my && lane < kGRows) en = load_entry(a, bh, tile_row0(i) + lane, s1, U, R);
            return en;
        };

        // Row entries are loaded three tiles before their copies are issued
        // (a register ring e0..e2), copies two tiles before their compute, so
        // neither the entry loads nor the row copies stall the warp.
        // prologue: entries of tiles 0..4 requested, copies of tiles 0..1 issued
        RowEntry e0 = entry_of(0), e1 = entry_of(1), e2 = entry_of(2);
#pragma unroll
        for (int i = 0; i < kGStages - 1; ++i) {
            const RowEntry en = e0;
            e0 = e1;
            e1 = e2;
            e2 = entry_of(i + 3);
            if (i < n_my) issue(i, i % kGStages, en);
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        }
        for (int i = 0; i < n_my; ++i) {
            const int ni = i + kGStages - 1;
            if (ni < n_my) {
                const RowEntry en = e0;
                e0 = e1;
                e1 = e2;
                e2 = entry_of(ni + 3);
                issue(ni, ni % kGStages, en);
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
            asm volatile("cp.async.wait_group %0;\n" ::"n"(kGStages - 1) : "memory");
            __syncwarp();

            const int st = i % kGStages;
            // a stage filled by tensor copies: wait for its mbarrier (bounded;
            // a local copy always lands -- a wait that gave up is reported in
            // the segment's error word and the tile is used as it is)
            if (tma_pending & (1u << st)) {
                if (!mbar_wait(&wbar[st], (tma_phase >> st) & 1u) && lane == 0)
                    atomicExch(&a.ws.flag[bh], 3);
                tma_phase ^= 1u << st;
                tma_pending &= ~(1u << st);
            }
            const unsigned char *stg = wbase + st * GG::STAGE;
            const char *ks_ = (const char *)stg;
            const char *vs_ = (const char *)stg + GG::TILE;
            const int *mk = (const int *)(wbase + kGStages * GG::STAGE + st * GG::META);
            const float *of = (const float *)(mk + kGRows);
            const int mat = lane >> 3, mrow = lane & 7;
            float s0v[4] = {0.f, 0.f, 0.f, 0.f}, s1v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                uint32_t b0, b1, b2, b3;
                const int r = ((mat >> 1) << 3) + mrow;
                const int c = 2 * kk + (mat & 1);
                ldmatrix_x4(smem_u32(ks_ + tile_off(r, c)), b0, b1, b2, b3);
                // A rows 0-7 = q hi parts, rows 8-15 = q lo parts (GQA heads
                // fill at most 8 rows): one mma yields both halves
                mma_bf16(s0v, qh[kk][0], ql[kk][0], qh[kk][1], ql[kk][1], b0, b1);
                mma_bf16(s1v, qh[kk][0], ql[kk][0], qh[kk][1], ql[kk][1], b2, b3);
            }
            const int rr[4] = {2 * tig, 2 * tig + 1, 8 + 2 * tig, 9 + 2 * tig};
            const float raw[4] = {s0v[0] + s0v[2], s0v[1] + s0v[3], s1v[0] + s1v[2],
                                  s1v[1] + s1v[3]};
            float sv4[4];
            bool any_sample = false;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int mm = mk[rr[q]];
                const bool on = gid < g && ((mm >> gid) & 1);
                sv4[q] = on ? ((mm & kMaskAbs) ? of[rr[q]] : raw[q] + of[rr[q]]) : -INFINITY;
                any_sample |= on && (mm & kMaskSample);
            }
            float tmax = fmaxf(fmaxf(sv4[0], sv4[1]), fmaxf(sv4[2], sv4[3]));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
            const float m_new = fmaxf(m_run, tmax);
            float pr[4];
            float alpha = 1.f;
            if (m_new == -INFINITY) {
                pr[0] = pr[1] = pr[2] = pr[3] = 0.f;
            } else {
                alpha = exp2f(m_run - m_new);
#pragma unroll
                for (int q = 0; q < 4; ++q) pr[q] = exp2f(sv4[q] - m_new);
                m_run = m_new;
            }
            l_run = l_run * alpha + (pr[0] + pr[1] + pr[2] + pr[3]);
            // once the running maxima settle most tiles leave them unchanged:
            // skip the accumulator rescale then (warp-uniform branch)
            if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
                for (int q = 0; q < NT_O; ++q) {
                    o[q][0] *= alpha;
                    o[q][1] *= alpha;
                    o[q][2] *= alpha;
                    o[q][3] *= alpha;
                }
            }
            if (__any_sync(0xffffffffu, any_sample)) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int mm = mk[rr[q]];
                    if (gid < g && ((mm >> gid) & 1) && (mm & kMaskSample)) {
                        const float lw = sv4[q];
                        if (lw > ms_run) {
                            const float f = exp2f(ms_run - lw);
                            e1_run = e1_run * f + 1.f;
                            e2_run = e2_run * f * f + 1.f;
                            ms_run = lw;
                        } else {
                            const float f = exp2f(lw - ms_run);
                            e1_run += f;
                            e2_run += f * f;
                        }
                    }
                }
            }
            const uint32_t ph0 = pack_bf16(pr[0], pr[1]);
            const uint32_t ph2 = pack_bf16(pr[2], pr[3]);
            const float2 f0 = __bfloat1622float2(*(const __nv_bfloat162 *)&ph0);
            const float2 f2 = __bfloat1622float2(*(const __nv_bfloat162 *)&ph2);
            const uint32_t pl0 = pack_bf16(pr[0] - f0.x, pr[1] - f0.y);
            const uint32_t pl2 = pack_bf16(pr[2] - f2.x, pr[3] - f2.y);
#pragma unroll
            for (int j = 0; j < D / 16; ++j) {
                uint32_t b0, b1, b2, b3;
                const int r = ((mat & 1) << 3) + mrow;
                const int c = 2 * j + (mat >> 1);
                ldmatrix_x4_trans(smem_u32(vs_ + tile_off(r, c)), b0, b1, b2, b3);
                // A rows 0-7 = p hi, rows 8-15 = p lo: accumulator rows gid
                // and gid + 8 hold the two halves of head gid's output
                mma_bf16(o[2 * j], ph0, pl0, ph2, pl2, b0, b1);
                mma_bf16(o[2 * j + 1], ph0, pl0, ph2, pl2, b2, b3);
            }
            __syncwarp();  // stage st is refilled by the next iteration's issue
        }
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");

        // ---- this warp is done with segment bh: write its partial ----
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
        {
            float MS = fmaxf(ms_run, __shfl_xor_sync(0xffffffffu, ms_run, 1));
            MS = fmaxf(MS, __shfl_xor_sync(0xffffffffu, MS, 2));
            const float f = (e1_run > 0.f) ? exp2f(ms_run - MS) : 0.f;
            float E1 = e1_run * f, E2 = e2_run * f * f;
            E1 += __shfl_xor_sync(0xffffffffu, E1, 1);
            E1 += __shfl_xor_sync(0xffffffffu, E1, 2);
            E2 += __shfl_xor_sync(0xffffffffu, E2, 1);
            E2 += __shfl_xor_sync(0xffffffffu, E2, 2);
            ms_run = MS;
            e1_run = E1;
            e2_run = E2;
        }
        // the ring is drained (wait_group 0 above): the warp's partial goes
        // into its first bytes
        float *wpart = (float *)wbase;
        if (gid < g) {
            if (tig == 0) {
                wpart[gid * PSTR + 0] = m_run;
                wpart[gid * PSTR + 1] = l_run;
                wpart[gid * PSTR + 2] = ms_run;
                wpart[gid * PSTR + 3] = e1_run;
                wpart[gid * PSTR + 4] = e2_run;
            }
#pragma unroll
            for (int q = 0; q < NT_O; ++q) {
                wpart[gid * PSTR + 8 + q * 8 + 2 * tig] = o[q][0] + o[q][2];
                wpart[gid * PSTR + 8 + q * 8 + 2 * tig + 1] = o[q][1] + o[q][3];
            }
        }
        // ---- CTA fold: the kGW warp partials of this segment -> one CTA
        // partial in slot c + bh, unique because the segments a CTA meets form
        // an increasing range and consecutive CTAs' shares overlap in at most
        // one segment.  Every warp of the CTA walks the same segments (the
        // loop bounds are CTA-uniform), so the block barriers line up ----
        __syncthreads();
        float *cpart = a.ws.partial + ((int64_t)blockIdx.x + bh) * g * PSTR;
        if (tid < g) {  // per head: maxima, denominators, the warps' factors
            const int h = tid;
            float M = -INFINITY, MS = -INFINITY;
#pragma unroll
            for (int w = 0; w < kGW; ++w) {
                const float *pw = (const float *)(base + w * GG::WARP) + h * PSTR;
                if (pw[1] > 0.f) M = fmaxf(M, pw[0]);
                if (pw[3] > 0.f) MS = fmaxf(MS, pw[2]);
            }
            float L = 0.f, E1 = 0.f, E2 = 0.f;
#pragma unroll
            for (int w = 0; w < kGW; ++w) {
                const float *pw = (const float *)(base + w * GG::WARP) + h * PSTR;
                const float f = pw[1] > 0.f ? exp2f(pw[0] - M) : 0.f;
                s_wfac[h][w] = f;
                L = fmaf(pw[1], f, L);
                if (pw[3] > 0.f) {
                    const float fe = exp2f(pw[2] - MS);
                    E1 = fmaf(pw[3], fe, E1);
                    E2 = fmaf(pw[4], fe * fe, E2);
                }
            }
            cpart[h * PSTR + 0] = M;
            cpart[h * PSTR + 1] = L;
            cpart[h * PSTR + 2] = MS;
            cpart[h * PSTR + 3] = E1;
            cpart[h * PSTR + 4] = E2;
        }
        __syncthreads();
        for (int i = tid; i < g * D; i += kGThreads) {
            const int hh = i / D, dd = i - hh * D;
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < kGW; ++w)
                acc = fmaf(s_wfac[hh][w],
                           ((const float *)(base + w * GG::WARP))[hh * PSTR + 8 + dd], acc);
            cpart[hh * PSTR + 8 + dd] = acc;
        }
        __syncthreads();  // the rings are refilled by the next segment
    }

    // ---- LSE merge.  Every warp reaches this barrier (the loops above have
    // no early exit and no waits that can time out), so the stage rings are
    // free and every CTA partial of this CTA is written.  The arrivals are
    // acq_rel atomics at GPU scope, one lane per segment: the release covers
    // this CTA's partials (ordered before it by the barrier), the acquire of
    // the last arrival covers every other CTA's, and the barrier after the
    // arrivals passes that on to the whole CTA ----
    __syncthreads();
    const DecodeArgs &ma = s_args;
    __shared__ unsigned s_lastmask;
    __shared__ int m_seg[kMergeSegs], m_first[kMergeSegs], m_cnt[kMergeSegs];
    __shared__ int m_n, m_mode;  // merge form: 2 direct, 1 staged together, 0 one by one
    const int wstride = g * PSTR;  // floats between partial slots
    // arrivals at up to 32 segments at once (one atomic round trip), then
    // the merges of the segments this CTA completed
    for (int b0 = bh0; b0 < BH && pre[b0] < r1; b0 += 32) {
        if (warp == 0) {
            const int bh = b0 + lane;
            bool done = false;
            int first = 0, cnt = 0;
            if (bh < BH && pre[bh] < r1) {
                const int seg0 = pre[bh], total = pre[bh + 1] - seg0;
                if (max(r0, seg0) < min(r1, seg0 + total)) {
                    first = seg0 / P;
                    cnt = (seg0 + total - 1) / P - first + 1;
                    unsigned old;
                    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;\n"
                                 : "=r"(old)
                                 : "l"(ma.ws.counters + bh)
                                 : "memory");
                    done = (int)old == cnt - 1;
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, done);
            // the completed segments, listed in lane order
            const int rank = __popc(m & ((1u << lane) - 1u));
            const bool fit = !done || (rank < kMergeSegs && cnt <= 32);
            const bool small = !done || (rank < kMergeSegs && cnt <= kDirectMax);
            int tot = done ? cnt : 0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
            const bool all_fit = __all_sync(0xffffffffu, fit);
            const bool all_small = __all_sync(0xffffffffu, small);
            if (done) {
                ma.ws.counters[bh] = 0;  // every CTA of the segment has arrived
                if (fused) atomicOr(done_bits + (bh >> 5), 1u << (bh & 31));
                if (rank < kMergeSegs) {
                    m_seg[rank] = bh;
                    m_first[rank] = first;
                    m_cnt[rank] = cnt;
                }
            }
            if (lane == 0) {
                s_lastmask = m;
                m_n = __popc(m);
                m_mode = all_small ? 2
                         : (all_fit && (int64_t)tot * wstride <= (int64_t)kGW * GG::WARP / 4) ? 1
                                                                                               : 0;
            }
        }
        __syncthreads();
        if (s_lastmask) {
            if (m_mode == 2) {
                merge_pairs_direct<D>(ma, m_seg, m_first, m_cnt, m_n, wstride);
            } else if (m_mode == 1) {
                merge_segments_to_output<D>(ma, m_seg, m_first, m_cnt, m_n, wstride, (float *)base);
            } else {
                for (unsigned m = s_lastmask; m; m &= m - 1) {
                    const int bh = b0 + __ffs(m) - 1;
                    const int seg0 = pre[bh], total = pre[bh + 1] - seg0;
                    const int f0 = seg0 / P, last = (seg0 + total - 1) / P;
                    merge_staged_to_output<D>(ma, bh, ma.ws.partial + ((int64_t)f0 + bh) * wstride,
                                              last - f0 + 1, wstride, (float *)base,
                                              kGW * GG::WARP / 4);
                    __syncthreads();  // the stage is reused by the next segment
                }
            }
        }
        __syncthreads();  // s_lastmask and the merge list are rewritten by the next batch
    }
    // segments with no rows at all (every head empty) still get an output
    if (blockIdx.x == 0) {
        for (int bh = 0; bh < BH; ++bh) {
            if (pre[bh + 1] != pre[bh]) continue;
            const int b = bh / ma.geo.num_kv_heads, kv = bh - b * ma.geo.num_kv_heads;
            if (fused && tid == 0) atomicOr(done_bits + (bh >> 5), 1u << (bh & 31));
            for (int i = tid; i < g * D; i += kGThreads) {
                const int h = i / D, d = i - h * D;
                const int64_t oh = (int64_t)b * ma.geo.num_kv_heads * g + (int64_t)kv * g + h;
                if (ma.part_out) {
                    float *po = ma.part_out + oh * PSTR;
                    po[8 + d] = 0.f;
                    if (d < 8) po[d] = (d == 0 || d == 2) ? -INFINITY : 0.f;
                    continue;
                }
                ma.out[oh * D + d] = 0.f;
                if (d == 0) {
                    if (ma.lse) ma.lse[oh] = -INFINITY;
                    if (ma.ess) ma.ess[oh] = 0.f;
                }
            }
        }
    }
    if (fused) {
        __syncthreads();  // this CTA's partial rows and done bits are in place
        fused_shard_exchange<D>(ma, done_bits, BH, (float *)base);
    }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
template <int D>
static size_t simt_smem_bytes(int Gmax) {
    return sizeof(WarpState<D>) * (kSimtThreads / 32) + (3 * (size_t)Gmax + 1) * 4 +
           SANTA_MAX_GROUP * D * 4;
}

int attend_partial_slots(const SantaGeometry *geo, int nsplit) {
    const int BH = geo->batch * geo->num_kv_heads;
    const int simt = BH * nsplit;
    const int gather = num_sms() + BH;  // one CTA partial per (CTA, segment met)
    return simt > gather ? simt : gather;
}

// cuTensorMapEncodeTiled from the driver, fetched once through the runtime
// (no link against the driver library)
typedef CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                         const cuuint64_t *, const cuuint64_t *,
                                         const cuuint32_t *, const cuuint32_t *,
                                         CUtensorMapInterleave, CUtensorMapSwizzle,
                                         CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static TensorMapEncodeTiled tensor_map_encoder() {
    static const TensorMapEncodeTiled fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (TensorMapEncodeTiled) nullptr;
        }
        return (TensorMapEncodeTiled)p;
    }();
    return fn;
}

// The [rows][D] bf16 cluster-sorted copy as a 2-D tensor of [16][64] boxes
// with the 128-byte swizzle of the attention kernel's tile layout.
template <int D>
static bool sorted_copy_map(CUtensorMap *m, const void *base, int64_t rows) {
    const TensorMapEncodeTiled enc = tensor_map_encoder();
    if (!enc || !base || ((uintptr_t)base & 15) || rows <= 0 || rows >= ((int64_t)1 << 31))
        return false;
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kGRows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

template <int D>
static int launch_execute_d(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups;
    // the segment counters are zeroed by the selection kernel and put back
    // to zero by each segment's merging CTA
    if (a.geo.kv_dtype == SANTA_DTYPE_BF16) {
        const size_t sm = gather_smem_bytes<D>(BH);
        if (sm > 227 * 1024) return SANTA_ERR_UNSUPPORTED;
        if (int st = ensure_dyn_smem((const void *)decode_attend_gather_kernel<D>, sm)) return st;
        // Programmatic dependent launch: the grid is scheduled as the
        // selection kernel's CTAs finish (they trigger it at their end), so
        // its launch latency overlaps their exit (0.4-1 us per step).  With
        // the trigger at the selection's start instead, the attention CTAs
        // occupied the SMs the selection left free and the step measured
        // slower than a plain stream-ordered launch: 232.5 vs 223.7 us at
        // 128K, 81.1 vs 69.4 us at 32K.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)num_sms(), 1, 1);
        cfg.blockDim = dim3(kGThreads, 1, 1);
        cfg.dynamicSmemBytes = sm;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        // tensor maps of the two cluster-sorted copies; if either cannot be
        // made, every tile takes the 16-byte copy path
        CUtensorMap mk, mv;
        memset(&mk, 0, sizeof(mk));
        memset(&mv, 0, sizeof(mv));
        const int64_t rows = (int64_t)BH * a.geo.sample_end;
        a.tma = sorted_copy_map<D>(&mk, a.sum.sorted_key, rows) &&
                        sorted_copy_map<D>(&mv, a.sum.sorted_value, rows)
                    ? 1
                    : 0;
        SANTA_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_attend_gather_kernel<D>, a, mk, mv));
    } else {
        const size_t sm = simt_smem_bytes<D>(Gmax);
        if (int st = ensure_dyn_smem((const void *)decode_attend_simt_kernel<D, float>, sm))
            return st;
        dim3 grid(a.nsplit, BH);
        decode_attend_simt_kernel<D, float><<<grid, kSimtThreads, sm, stream>>>(a);
    }
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

int launch_execute(DecodeArgs &a, cudaStream_t stream) {
    return a.geo.head_dim == 64 ? launch_execute_d<64>(a, stream)
                                : launch_execute_d<128>(a, stream);
}

}  // namespace santa
