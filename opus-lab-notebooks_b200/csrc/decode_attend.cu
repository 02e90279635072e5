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
//   decode_attend_pipe_kernel   bf16 caches.  One CTA per SM, the virtual row
//       spaces of all (batch, KV head) segments concatenated and split evenly
//       over the CTAs.  Warp 4 is a producer that resolves 64-row tiles from
//       tables in shared memory and streams the rows with row-cooperative,
//       coalesced 16-byte cp.async copies into a 4-stage ring of padded
//       shared-memory tiles, completing on mbarriers (cp.async.mbarrier.arrive);
//       per-row bulk copies through the TMA engine were measured 4x slower on
//       these 256-byte gathers: the engine is request-bound at that size;
//       warps 0-3 consume 16 rows each with mma.sync m16n8k16 (GQA heads on
//       the M dimension, q and p split into bf16 hi + lo for fp32-level
//       accuracy) and an online softmax.  At every segment end the CTA writes
//       one partial; the last CTA of a segment merges them (LSE merge).
//   decode_attend_simt_kernel  fp32 caches, a warp per row.
#include "decode_common.cuh"

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
// producer / consumer pipeline kernel (bf16 caches)
// ---------------------------------------------------------------------------
constexpr int kRows = 64;     // rows per tile
constexpr int kNS = 4;        // pipeline stages
constexpr int kCons = 4;      // consumer warps, 16 rows each
constexpr int kPipeThreads = 32 * (kCons + 1);
constexpr int kSampCap = 4096; // sample words of a segment kept in shared memory

template <int D>
struct PipeGeom {
    static constexpr int ROWB = D * 2;           // bytes of one bf16 row
    static constexpr int PITCH = ROWB + 16;      // padded smem pitch: 8 rows hit 8 bank groups
    static constexpr int TILE = kRows * PITCH;   // bytes of one K (or V) stage
};

template <int D>
__host__ __device__ inline size_t pipe_smem_bytes(int BH, int Gmax) {
    size_t b = 128;                                    // alignment slack
    b += 2 * (size_t)kNS * PipeGeom<D>::TILE;           // K and V stages
    b += 2 * (size_t)kNS * kRows * 4;                  // row mask + offset
    b += 2 * kNS * 8;                                  // full / empty mbarriers
    b += ((size_t)BH + 1) * 4;                         // segment prefix
    b += (3 * (size_t)Gmax + 1) * 4;                   // producer's union table
    b += 2 * (size_t)kSampCap * 4;                     // producer's sample table
    return b;
}

template <int D>
__global__ void __launch_bounds__(kPipeThreads, 1) decode_attend_pipe_kernel(DecodeArgs a) {
    using TG = PipeGeom<D>;
    constexpr int NT_O = D / 8;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups, g = a.geo.group;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    unsigned char *p = (unsigned char *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    char *kbuf = (char *)p;                  p += kNS * TG::TILE;
    char *vbuf = (char *)p;                  p += kNS * TG::TILE;
    int *rmask = (int *)p;                   p += kNS * kRows * 4;
    float *roff = (float *)p;                p += kNS * kRows * 4;
    uint64_t *full = (uint64_t *)p;          p += kNS * 8;
    uint64_t *empty = (uint64_t *)p;         p += kNS * 8;
    int *pre = (int *)p;                     p += (BH + 1) * 4;
    int *u_off = (int *)p;                   p += (Gmax + 1) * 4;
    int *u_start = (int *)p;                 p += Gmax * 4;
    int *u_mask = (int *)p;                  p += Gmax * 4;
    int32_t *s_tab = (int32_t *)p;           p += kSampCap * 4;
    float *s_offt = (float *)p;              p += kSampCap * 4;
    constexpr int CPR = TG::ROWB / 16;           // 16-byte chunks per row
    constexpr int kRowsPerIter = 32 / CPR;

    // ---- set-up: zero the stages (rows past a tile's end are multiplied by
    // p = 0 and must hold finite values), barriers, segment prefix ----
    for (int i = tid; i < 2 * kNS * TG::TILE / 16; i += kPipeThreads)
        ((int4 *)kbuf)[i] = make_int4(0, 0, 0, 0);
    if (tid == 0) {
        for (int s = 0; s < kNS; ++s) {
            mbar_init(&full[s], 32);  // one cp.async arrival per producer lane
            mbar_init(&empty[s], kCons);
        }
        mbar_fence_init();
    }
    if (warp == 0) {
        int carry = 0;
        for (int i0 = 0; i0 < BH; i0 += 32) {
            const int i = i0 + lane;
            int x = i < BH ? a.ws.meta[(int64_t)i * 8 + 4] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (i < BH) pre[i + 1] = carry + x;
            carry += __shfl_sync(0xffffffffu, x, 31);
        }
        if (lane == 0) pre[0] = 0;
    }
    fence_proxy_async_smem();  // order the generic zero-fill before async-proxy copies
    __syncthreads();

    const int T_all = pre[BH];
    const int P = max(1, ceil_div(T_all, (int)gridDim.x));
    const int r0 = min(T_all, (int)blockIdx.x * P);
    const int r1 = min(T_all, r0 + P);
    int bh0 = 0;
    while (bh0 < BH && pre[bh0 + 1] <= r0) ++bh0;

    if (warp == kCons) {
        // ===================== producer warp =====================
        int it = 0;
        bool err = false;
        for (int bh = bh0; bh < BH && pre[bh] < r1 && !err; ++bh) {
            const int seg0 = pre[bh], total = pre[bh + 1] - seg0;
            const int s0 = max(r0, seg0) - seg0, s1 = min(r1, seg0 + total) - seg0;
            if (s0 >= s1) continue;
            const int32_t *meta = a.ws.meta + (int64_t)bh * 8;
            const int n_union = meta[0], U = meta[1], R = meta[2];
            for (int i = lane; i <= n_union; i += 32)
                u_off[i] = a.ws.u_off[(int64_t)bh * (Gmax + 1) + i];
            for (int i = lane; i < n_union; i += 32) {
                u_start[i] = a.ws.u_start[(int64_t)bh * Gmax + i];
                u_mask[i] = a.ws.u_mask[(int64_t)bh * Gmax + i];
            }
            // the segment's sample table, so row resolution never waits on HBM
            const int nsamp = min(meta[3], kSampCap);
            const int64_t sbase = (int64_t)bh * g * a.p.samples;
            for (int i = lane; i < nsamp; i += 32) {
                s_tab[i] = a.ws.s_pos[sbase + i];
                s_offt[i] = a.ws.s_off[sbase + i];
            }
            __syncwarp();
            for (int t0 = s0; t0 < s1; t0 += kRows, ++it) {
                const int st = it % kNS;
                const uint32_t ph = (uint32_t)(it / kNS) & 1u;
                if (it >= kNS && !mbar_wait(&empty[st], ph ^ 1u)) {
                    err = true;
                    break;
                }
                const int nrows = min(kRows, s1 - t0);
                const char *kp[2], *vp[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int row = lane + 32 * j;
                    RowInfo ri;
                    ri.k = ri.v = nullptr;
                    ri.mask = 0;
                    ri.off = 0.f;
                    if (row < nrows)
                        ri = resolve_row(a, bh, t0 + row, U, R, total, n_union, u_off, u_start,
                                         u_mask, TG::ROWB, s_tab, s_offt, nsamp);
                    kp[j] = ri.k;
                    vp[j] = ri.v;
                    rmask[st * kRows + row] = ri.mask;
                    roff[st * kRows + row] = ri.off;
                }
                // row-cooperative 16-byte copies: CPR lanes cover one row, so a
                // warp instruction moves 32 / CPR whole rows, fully coalesced
                char *kd = kbuf + st * TG::TILE;
                char *vd = vbuf + st * TG::TILE;
#pragma unroll
                for (int i = 0; i < kRows / kRowsPerIter; ++i) {
                    const int r = i * kRowsPerIter + lane / CPR;   // tile row
                    const int c = lane % CPR;                      // 16-byte chunk
                    const int slot = (i * kRowsPerIter) / 32;      // uniform per iteration
                    const char *ks = (const char *)__shfl_sync(
                        0xffffffffu, (unsigned long long)(slot ? kp[1] : kp[0]), r & 31);
                    const char *vs = (const char *)__shfl_sync(
                        0xffffffffu, (unsigned long long)(slot ? vp[1] : vp[0]), r & 31);
                    if (r < nrows) {
                        cp_async16(kd + r * TG::PITCH + c * 16, ks + c * 16);
                        cp_async16(vd + r * TG::PITCH + c * 16, vs + c * 16);
                    }
                }
                __syncwarp();
                cp_async_mbar_arrive(&full[st]);
            }
        }
        if (err && lane == 0) atomicExch(a.ws.flag + kFlagWaitTimeout, 1);
        // no copy may still be landing in shared memory when the CTA exits
        for (int k = max(0, it - kNS); k < it; ++k)
            mbar_wait(&full[k % kNS], (uint32_t)(k / kNS) & 1u);
        return;
    }

    // ===================== consumer warps =====================
    const float qscale = a.p.scale * kLog2e;
    const int gid = lane >> 2, tig = lane & 3;
    const int rbase = warp * 16;  // this warp's rows inside a tile
    const int PSTR = partial_stride(D);
    int it = 0;
    bool err = false;
    for (int bh = bh0; bh < BH && pre[bh] < r1; ++bh) {
        const int seg0 = pre[bh], total = pre[bh + 1] - seg0;
        const int s0 = max(r0, seg0) - seg0, s1 = min(r1, seg0 + total) - seg0;
        if (s0 >= s1) continue;
        // q fragments of this (batch, KV head): rows = heads, split bf16 hi + lo
        const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
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

        for (int t0 = s0; t0 < s1; t0 += kRows, ++it) {
            const int st = it % kNS;
            const uint32_t ph = (uint32_t)(it / kNS) & 1u;
            if (!mbar_wait(&full[st], ph)) {
                err = true;
                break;
            }
            const int nrows = min(kRows, s1 - t0);
            if (rbase < nrows) {
                const char *ks_ = kbuf + st * TG::TILE;
                const char *vs_ = vbuf + st * TG::TILE;
                const int mat = lane >> 3, mrow = lane & 7;
                float s0v[4] = {0.f, 0.f, 0.f, 0.f}, s1v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    uint32_t b0, b1, b2, b3;
                    const int r = rbase + ((mat >> 1) << 3) + mrow;
                    const int c = 2 * ks + (mat & 1);
                    ldmatrix_x4(smem_u32(ks_ + r * TG::PITCH + c * 16), b0, b1, b2, b3);
                    mma_bf16(s0v, qh[ks][0], 0u, qh[ks][1], 0u, b0, b1);
                    mma_bf16(s0v, ql[ks][0], 0u, ql[ks][1], 0u, b0, b1);
                    mma_bf16(s1v, qh[ks][0], 0u, qh[ks][1], 0u, b2, b3);
                    mma_bf16(s1v, ql[ks][0], 0u, ql[ks][1], 0u, b2, b3);
                }
                const int *mk = rmask + st * kRows;
                const float *of = roff + st * kRows;
                const int rr[4] = {rbase + 2 * tig, rbase + 2 * tig + 1, rbase + 8 + 2 * tig,
                                   rbase + 9 + 2 * tig};
                const float raw[4] = {s0v[0], s0v[1], s1v[0], s1v[1]};
                float sv[4];
                bool any_sample = false;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int mm = mk[rr[i]];
                    const bool on = gid < g && ((mm >> gid) & 1);
                    sv[i] = on ? ((mm & kMaskAbs) ? of[rr[i]] : raw[i] + of[rr[i]]) : -INFINITY;
                    any_sample |= on && (mm & kMaskSample);
                }
                float tmax = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
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
                    for (int i = 0; i < 4; ++i) pr[i] = exp2f(sv[i] - m_new);
                    m_run = m_new;
                }
                l_run = l_run * alpha + (pr[0] + pr[1] + pr[2] + pr[3]);
#pragma unroll
                for (int i = 0; i < NT_O; ++i) {
                    o[i][0] *= alpha;
                    o[i][1] *= alpha;
                }
                if (__any_sync(0xffffffffu, any_sample)) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int mm = mk[rr[i]];
                        if (gid < g && ((mm >> gid) & 1) && (mm & kMaskSample)) {
                            const float lw = sv[i];
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
                    const int r = rbase + ((mat & 1) << 3) + mrow;
                    const int c = 2 * j + (mat >> 1);
                    ldmatrix_x4_trans(smem_u32(vs_ + r * TG::PITCH + c * 16), b0, b1, b2, b3);
                    mma_bf16(o[2 * j], ph0, 0u, ph2, 0u, b0, b1);
                    mma_bf16(o[2 * j], pl0, 0u, pl2, 0u, b0, b1);
                    mma_bf16(o[2 * j + 1], ph0, 0u, ph2, 0u, b2, b3);
                    mma_bf16(o[2 * j + 1], pl0, 0u, pl2, 0u, b2, b3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        if (err) break;

        // ---- this CTA is done with segment bh: write its partial ----
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
        // Each consumer warp writes its own partial (no intra-CTA barrier, so
        // a timed-out wait in one warp cannot stall the others).  Slot
        // (c + bh) * kCons + warp is unique: the segments a CTA meets form an
        // increasing range and the ranges of consecutive CTAs touch at most
        // at one segment.
        const int64_t slot = ((int64_t)blockIdx.x + bh) * kCons + warp;
        float *part = a.ws.partial + slot * g * PSTR;
        if (gid < g) {
            if (tig == 0) {
                part[gid * PSTR + 0] = m_run;
                part[gid * PSTR + 1] = l_run;
                part[gid * PSTR + 2] = ms_run;
                part[gid * PSTR + 3] = e1_run;
                part[gid * PSTR + 4] = e2_run;
            }
#pragma unroll
            for (int i = 0; i < NT_O; ++i) {
                part[gid * PSTR + 8 + i * 8 + 2 * tig] = o[i][0];
                part[gid * PSTR + 8 + i * 8 + 2 * tig + 1] = o[i][1];
            }
        }
        __threadfence();
        __syncwarp();
        const int first = seg0 / P, last = (seg0 + total - 1) / P;
        const int contributors = (last - first + 1) * kCons;
        int is_last = 0;
        if (lane == 0) is_last = (atomicAdd(&a.ws.counters[bh], 1) == contributors - 1);
        is_last = __shfl_sync(0xffffffffu, is_last, 0);
        if (is_last) {
            __threadfence();
            merge_partials_to_output<D>(
                a, bh, a.ws.partial + ((int64_t)first + bh) * kCons * g * PSTR, contributors, lane,
                32);
            if (lane == 0) a.ws.counters[bh] = 0;
        }
    }
    if (err && lane == 0) atomicExch(a.ws.flag + kFlagWaitTimeout, 1);
    // segments with no rows at all (every head empty) still get an output
    if (blockIdx.x == 0 && !err) {
        for (int bh = 0; bh < BH; ++bh) {
            if (pre[bh + 1] != pre[bh]) continue;
            const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
            for (int i = tid; i < g * D; i += 32 * kCons) {
                const int h = i / D, d = i - h * D;
                const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
                a.out[oh * D + d] = 0.f;
                if (d == 0) {
                    if (a.lse) a.lse[oh] = -INFINITY;
                    if (a.ess) a.ess[oh] = 0.f;
                }
            }
        }
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
    const int pipe = (num_sms() + BH) * kCons;
    return simt > pipe ? simt : pipe;
}

template <int D>
static int launch_execute_d(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups;
    SANTA_CUDA_CHECK(cudaMemsetAsync(a.ws.counters, 0, (size_t)BH * 4, stream));
    if (a.geo.kv_dtype == SANTA_DTYPE_BF16) {
        static size_t done = 0;
        const size_t sm = pipe_smem_bytes<D>(BH, Gmax);
        if (sm > 227 * 1024) return SANTA_ERR_UNSUPPORTED;
        if (done < sm) {
            SANTA_CUDA_CHECK(cudaFuncSetAttribute(decode_attend_pipe_kernel<D>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)sm));
            done = sm;
        }
        decode_attend_pipe_kernel<D><<<num_sms(), kPipeThreads, sm, stream>>>(a);
    } else {
        static size_t done = 0;
        const size_t sm = simt_smem_bytes<D>(Gmax);
        if (done < sm) {
            SANTA_CUDA_CHECK(cudaFuncSetAttribute(decode_attend_simt_kernel<D, float>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)sm));
            done = sm;
        }
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
