// SANTA++ sparse decode: cluster selection + split-KV gather attention.
//
// Replaces SantaPlusEngine._approximate_attention
// (santapp_ruler/attention/santapp.py:365-506), batched over every
// (batch, query head) instead of the per-head Python loop of :347-358.
//
// Two launches per decode step:
//   decode_select_kernel   one CTA per (batch, KV head): centroid guesses for
//                          the GQA group (santapp.py:397-400), ranking with a
//                          shared-memory bitonic sort (argsort at :401 with
//                          lowest-index tie-break), top-k / budget walk
//                          (:402-411), union of the group's selections, and
//                          the importance samples with their log weights
//                          (:429-468).  Output is a per-(b, kv) work list.
//   decode_attend_*        split-KV over the work list: NSPLIT CTAs per
//                          (b, kv) stream the selected clusters (contiguous
//                          row runs of the cluster-sorted copy), the exact
//                          recent window and the sampled rows, with an online
//                          softmax per query head; the last CTA of each
//                          (b, kv) merges the split partials (LSE merge) and
//                          writes out / lse / ess (:472-506).
#include "common.cuh"

#include <math.h>

namespace santa {

constexpr int kSelThreads = 512;
constexpr int kTileRows = 64;
constexpr int kAttThreads = 128;
constexpr int kStages = 3;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// packed sample word: bits 0-23 sorted row, 24-26 local head, 27 = absolute
// log weight (santa mode: lw does not depend on the row's score)
constexpr uint32_t kPosMask = 0xFFFFFFu;
constexpr int kHeadShift = 24;
constexpr uint32_t kAbsBit = 1u << 27;

struct DecodeWs {
    int32_t *counters;   // [BH]
    int32_t *flag;       // [4] invalid injected draws seen
    int32_t *meta;       // [BH][8]: 0 n_union, 1 U, 2 R, 3 n_samples, 4 total rows
    int32_t *head_meta;  // [BH][8][2]: n_exact, n_samples
    int32_t *u_start;    // [BH][G]
    int32_t *u_mask;     // [BH][G]
    int32_t *u_cid;      // [BH][G] cluster row of each union entry
    int32_t *u_off;      // [BH][G+1]
    int32_t *s_pos;      // [BH][g*S]
    float *s_off;        // [BH][g*S] log2-units offset (or absolute log2 weight)
    float *lse_old;      // [BH][8] santa mode: log-sum-exp (log2 units) of old scores
    float *partial;      // [BH][nsplit][g][PSTR]
};

__host__ __device__ inline int partial_stride(int D) { return D + 8; }

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static size_t decode_ws_layout(int BH, int G, int g, int S, int nsplit, int D, char *base,
                               DecodeWs *ws) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const int gs = g * (S > 0 ? S : 1);
    size_t o_cnt = take((size_t)BH * 4);
    size_t o_flag = take(16);
    size_t o_meta = take((size_t)BH * 8 * 4);
    size_t o_hm = take((size_t)BH * 16 * 4);
    size_t o_us = take((size_t)BH * G * 4);
    size_t o_um = take((size_t)BH * G * 4);
    size_t o_uc = take((size_t)BH * G * 4);
    size_t o_uo = take((size_t)BH * (G + 1) * 4);
    size_t o_sp = take((size_t)BH * gs * 4);
    size_t o_so = take((size_t)BH * gs * 4);
    size_t o_lo = take((size_t)BH * 8 * 4);
    size_t o_pa = take((size_t)BH * nsplit * g * partial_stride(D) * 4);
    if (base && ws) {
        ws->counters = (int32_t *)(base + o_cnt);
        ws->flag = (int32_t *)(base + o_flag);
        ws->meta = (int32_t *)(base + o_meta);
        ws->head_meta = (int32_t *)(base + o_hm);
        ws->u_start = (int32_t *)(base + o_us);
        ws->u_mask = (int32_t *)(base + o_um);
        ws->u_cid = (int32_t *)(base + o_uc);
        ws->u_off = (int32_t *)(base + o_uo);
        ws->s_pos = (int32_t *)(base + o_sp);
        ws->s_off = (float *)(base + o_so);
        ws->lse_old = (float *)(base + o_lo);
        ws->partial = (float *)(base + o_pa);
    }
    return off;
}

struct DecodeArgs {
    SantaGeometry geo;
    SantaDecodeParams p;
    SantaSummary sum;
    const float *q;
    const char *key_cache;
    const char *value_cache;
    const int32_t *sample_a;
    const int32_t *sample_b;
    float *out;
    float *lse;
    int32_t *n_exact;
    float *ess;
    int nsplit;
    DecodeWs ws;
};

// ---------------------------------------------------------------------------
// block-wide helpers (blockDim.x == kSelThreads)
// ---------------------------------------------------------------------------
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

// ---------------------------------------------------------------------------
// selection kernel
// ---------------------------------------------------------------------------
template <int D>
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

    // shared memory carve-up
    float *qs = (float *)smem_raw;                              // [8][D]
    float *ct = qs + SANTA_MAX_GROUP * D;                       // [64][D+1]
    int *starts_s = (int *)(ct + 64 * (D + 1));                 // [Gmax]
    int *len_s = starts_s + Gmax;                               // [Gmax]
    int *mask_s = len_s + Gmax;                                 // [Gmax]
    float *guess_s = (float *)(mask_s + Gmax);                  // [8][Gmax]
    int *selasc = (int *)(guess_s + SANTA_MAX_GROUP * Gmax);    // [8][Gmax]
    int *sw = selasc + SANTA_MAX_GROUP * Gmax;                  // [40]
    int *head_sel = sw + 40;                                    // [8] selected clusters per head
    int *head_exact = head_sel + 8;                             // [8]
    int *head_ns = head_exact + 8;                              // [8] samples per head
    int *head_sbase = head_ns + 8;                              // [8]
    float *head_f = (float *)(head_sbase + 8);                  // [8][4] misc floats
    uint64_t *keys = (uint64_t *)(((uintptr_t)(head_f + 32) + 15) & ~(uintptr_t)15);  // [8][Gp]

    const int n_groups = uses_clusters ? a.sum.n_groups[bh] : 0;
    int Gp = 1;
    while (Gp < n_groups) Gp <<= 1;

    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    for (int i = tid; i < g * D; i += kSelThreads) qs[i] = qb[i];
    for (int i = tid; i < n_groups; i += kSelThreads) {
        starts_s[i] = a.sum.starts[(int64_t)bh * Gmax + i];
        len_s[i] = a.sum.lengths[(int64_t)bh * Gmax + i];
        mask_s[i] = 0;
    }
    if (tid < 8) {
        head_sel[tid] = 0;
        head_exact[tid] = 0;
        head_ns[tid] = 0;
    }
    __syncthreads();

    // ---- centroid guesses: fl32(log_n + fl32(dot * scale)), dot = fmaf chain ----
    if (uses_clusters) {
        const float *cent = a.sum.centroids + (int64_t)bh * Gmax * D;
        const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
        for (int c0 = 0; c0 < n_groups; c0 += 64) {
            const int nc = min(64, n_groups - c0);
            for (int i = tid; i < nc * D; i += kSelThreads) {
                const int r = i / D, d = i - r * D;
                ct[r * (D + 1) + d] = cent[(int64_t)(c0 + r) * D + d];
            }
            __syncthreads();
            const int c = tid & 63, h = tid >> 6;  // 512 threads = 64 centroids x 8 heads
            if (c < nc && h < g) {
                const float *crow = ct + c * (D + 1);
                const float *qh = qs + h * D;
                float acc = 0.0f;
#pragma unroll 8
                for (int d = 0; d < D; ++d) acc = fmaf(crow[d], qh[d], acc);
                const float gs = __fadd_rn(logn[c0 + c], __fmul_rn(acc, a.p.scale));
                guess_s[h * Gmax + c0 + c] = gs;
            }
            __syncthreads();
        }
    }

    // ---- ranking (TOPK / HYBRID): bitonic sort of (guess, -index) descending ----
    if (mode == SANTA_MODE_TOPK || mode == SANTA_MODE_HYBRID) {
        for (int i = tid; i < g * Gp; i += kSelThreads) {
            const int h = i / Gp, c = i - h * Gp;
            uint64_t k = 0;
            if (c < n_groups)
                k = ((uint64_t)float_order_key(guess_s[h * Gmax + c]) << 32) |
                    (uint64_t)(0xFFFFFFFFu - (uint32_t)c);
            keys[i] = k;
        }
        __syncthreads();
        const int half = Gp >> 1;
        for (int kk = 2; kk <= Gp; kk <<= 1) {
            for (int j = kk >> 1; j > 0; j >>= 1) {
                for (int p = tid; p < g * half; p += kSelThreads) {
                    const int h = p / half, i = p - h * half;
                    const int lo = 2 * j * (i / j) + (i % j);
                    const int hi = lo + j;
                    uint64_t *arr = keys + h * Gp;
                    const uint64_t x = arr[lo], y = arr[hi];
                    const bool desc = (lo & kk) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        arr[lo] = y;
                        arr[hi] = x;
                    }
                }
                __syncthreads();
            }
        }
        // selection per head (one warp per head)
        if (warp < g) {
            const int h = warp;
            const uint64_t *arr = keys + h * Gp;
            int nsel = 0, exact = 0;
            if (mode == SANTA_MODE_HYBRID) {
                const int k = min(a.p.topk_clusters, n_groups);
                for (int i = lane; i < k; i += 32) {
                    const int c = (int)(0xFFFFFFFFu - (uint32_t)(arr[i] & 0xFFFFFFFFu));
                    atomicOr(&mask_s[c], 1 << h);
                    exact += len_s[c];
                }
                nsel = k;
            } else {
                int carry = 0;
                for (int i0 = 0; i0 < n_groups; i0 += 32) {
                    const int i = i0 + lane;
                    int c = 0, l = 0;
                    if (i < n_groups) {
                        c = (int)(0xFFFFFFFFu - (uint32_t)(arr[i] & 0xFFFFFFFFu));
                        l = len_s[c];
                    }
                    int x = l;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        int y = __shfl_up_sync(0xffffffffu, x, o);
                        if (lane >= o) x += y;
                    }
                    const int excl = carry + x - l;
                    const bool take = (i < n_groups) && (excl < a.p.token_budget);
                    if (take) {
                        atomicOr(&mask_s[c], 1 << h);
                        exact += l;
                    }
                    nsel += __popc(__ballot_sync(0xffffffffu, take));
                    carry += __shfl_sync(0xffffffffu, x, 31);
                    if (carry >= a.p.token_budget) break;
                }
            }
            exact = warp_sum_int(exact);
            if (lane == 0) {
                head_sel[h] = nsel;
                head_exact[h] = exact;
            }
        }
        __syncthreads();
    }

    // ---- union of the group's selections (ascending cluster order) ----
    int n_union = 0, U = 0;
    {
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
            }
            base += cnt;
            rows += rtot;
        }
        n_union = base;
        U = rows;
        if (tid == 0) a.ws.u_off[(int64_t)bh * (Gmax + 1) + n_union] = U;
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
    __syncthreads();
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

    // ---- guided: per-head softmax over guesses for the proposal ----
    if (mode == SANTA_MODE_GUIDED && warp < g) {
        const int h = warp;
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
        // inclusive cdf of unnormalised probabilities, stored over guess_s of a
        // scratch row: reuse keys[] as float storage
        float *cdf = (float *)keys + h * Gmax;
        float carry = 0.0f;
        for (int c0 = 0; c0 < n_groups; c0 += 32) {
            const int c = c0 + lane;
            float v = c < n_groups ? expf(guess_s[h * Gmax + c] - mx) : 0.0f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                float y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            if (c < n_groups) cdf[c] = carry + v;
            carry += __shfl_sync(0xffffffffu, v, 31);
        }
    }
    __syncthreads();

    // ---- samples ----
    if (warp < g && head_ns[warp] > 0) {
        const int h = warp;
        const int ns = head_ns[h];
        const int sbase = head_sbase[h];
        const int gh = kv * g + h;  // global query head
        int32_t *spos = a.ws.s_pos + (int64_t)bh * g * S + sbase;
        float *soff = a.ws.s_off + (int64_t)bh * g * S + sbase;
        const int64_t inj = ((int64_t)b * a.geo.num_kv_heads * g + gh) * S;
        const uint2 key = make_uint2((uint32_t)a.p.seed, (uint32_t)(a.p.seed >> 32));
        const float logS = logf((float)ns);
        if (mode == SANTA_MODE_HYBRID) {
            // selected clusters of this head in ascending cluster (= start) order
            int *sel = selasc + h * Gmax;
            int cnt = 0;
            for (int c0 = 0; c0 < n_groups; c0 += 32) {
                const int c = c0 + lane;
                const bool on = c < n_groups && ((mask_s[c] >> h) & 1);
                const unsigned bal = __ballot_sync(0xffffffffu, on);
                if (on) sel[cnt + __popc(bal & ((1u << lane) - 1u))] = c;
                cnt += __popc(bal);
            }
            __syncwarp();
            const int n_rest = sample_end - head_exact[h];
            const float off = (logf((float)n_rest) - logS) * kLog2e;
            for (int i = lane; i < ns; i += 32) {
                uint32_t r;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    int v = a.sample_a[inj + i];
                    if (v < 0 || v >= n_rest) {
                        atomicExch(a.ws.flag, 1);
                        v = min(max(v, 0), n_rest - 1);
                    }
                    r = (uint32_t)v;
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 2), (uint32_t)gh, (uint32_t)b, (uint32_t)a.p.step),
                        key);
                    r = (uint32_t)(((uint64_t)uint4_word(w, i & 3) * (uint64_t)n_rest) >> 32);
                }
                int p = (int)r;
                for (int j = 0; j < cnt; ++j) {
                    const int c = sel[j];
                    if (p >= starts_s[c]) p += len_s[c];
                    else break;
                }
                spos[i] = (int32_t)((uint32_t)p | ((uint32_t)h << kHeadShift));
                soff[i] = off;
            }
        } else if (mode == SANTA_MODE_GUIDED) {
            const float mx = head_f[h * 4 + 0], logz = head_f[h * 4 + 1];
            const float *cdf = (const float *)keys + h * Gmax;
            const float total = cdf[n_groups - 1];
            const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
            for (int i = lane; i < ns; i += 32) {
                int grp, within;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    grp = a.sample_a[inj + i];
                    within = a.sample_b[inj + i];
                    if (grp < 0 || grp >= n_groups) {
                        atomicExch(a.ws.flag, 1);
                        grp = min(max(grp, 0), n_groups - 1);
                    }
                    if (within < 0 || within >= len_s[grp]) {
                        atomicExch(a.ws.flag, 1);
                        within = min(max(within, 0), len_s[grp] - 1);
                    }
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 1), (uint32_t)gh, (uint32_t)b, (uint32_t)a.p.step),
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
            for (int i = lane; i < ns; i += 32) {
                int t;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    t = a.sample_a[inj + i];
                    if (t < 0 || t >= sample_end) {
                        atomicExch(a.ws.flag, 1);
                        t = min(max(t, 0), sample_end - 1);
                    }
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 2), (uint32_t)gh, (uint32_t)b, (uint32_t)a.p.step),
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
// santa mode: log-sum-exp of every old-prefix score (the oracle proposal
// reads all old keys, santapp.py:450-458).  One CTA per (b, kv, head chunk).
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
    const T *kb = (const T *)a.key_cache + (int64_t)bh * a.geo.capacity * D;
    for (int t = warp; t < a.geo.sample_end; t += 8) {
        float kr[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) kr[j] = to_f32<T>(kb[(int64_t)t * D + lane + 32 * j]);
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
// attend: shared pieces
// ---------------------------------------------------------------------------
struct RowInfo {
    const char *k;
    const char *v;
    float off;     // log2-units additive offset (or absolute weight when abs)
    int mask;      // bit h: row contributes to local head h; bit 8: sample row; bit 9: abs
};

__device__ __forceinline__ RowInfo resolve_row(const DecodeArgs &a, int bh, int v, int U, int R,
                                               int total, int n_union, const int *u_off,
                                               const int *u_start, const int *u_mask,
                                               int row_bytes) {
    RowInfo ri;
    const int g = a.geo.group;
    const int sample_end = a.geo.sample_end;
    const char *sk = (const char *)a.sum.sorted_key + (int64_t)bh * sample_end * row_bytes;
    const char *sv = (const char *)a.sum.sorted_value + (int64_t)bh * sample_end * row_bytes;
    if (v >= total) {
        ri.k = sk;
        ri.v = sv;
        ri.off = 0.f;
        ri.mask = 0;
    } else if (v < U) {
        int lo = 0, hi = n_union - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (u_off[mid] <= v) lo = mid;
            else hi = mid - 1;
        }
        const int row = u_start[lo] + (v - u_off[lo]);
        ri.k = sk + (int64_t)row * row_bytes;
        ri.v = sv + (int64_t)row * row_bytes;
        ri.off = 0.f;
        ri.mask = u_mask[lo];
    } else if (v < U + R) {
        const int64_t row = (int64_t)bh * a.geo.capacity + sample_end + (v - U);
        ri.k = a.key_cache + row * row_bytes;
        ri.v = a.value_cache + row * row_bytes;
        ri.off = 0.f;
        ri.mask = (1 << g) - 1;
    } else {
        const int j = v - U - R;
        const uint32_t pk = (uint32_t)a.ws.s_pos[(int64_t)bh * g * a.p.samples + j];
        const int row = (int)(pk & kPosMask);
        const int h = (int)((pk >> kHeadShift) & 7u);
        ri.k = sk + (int64_t)row * row_bytes;
        ri.v = sv + (int64_t)row * row_bytes;
        ri.off = a.ws.s_off[(int64_t)bh * g * a.p.samples + j];
        ri.mask = (1 << h) | 256 | ((pk & kAbsBit) ? 512 : 0);
    }
    return ri;
}

// Per-warp state in shared memory for the cross-warp and cross-split merge.
template <int D>
struct WarpState {
    float m[SANTA_MAX_GROUP], l[SANTA_MAX_GROUP];
    float ms[SANTA_MAX_GROUP], e1[SANTA_MAX_GROUP], e2[SANTA_MAX_GROUP];
    float o[SANTA_MAX_GROUP][D];
};

// Merge the 4 warps of this CTA, write the split partial, and let the last
// CTA of this (b, kv) merge every split into out / lse / ess.
template <int D>
__device__ void finish_cta(const DecodeArgs &a, int bh, WarpState<D> *ws4, int split) {
    const int g = a.geo.group;
    const int tid = threadIdx.x;
    constexpr int NW = kAttThreads / 32;
    const int PSTR = partial_stride(D);
    float *part = a.ws.partial + ((int64_t)bh * a.nsplit + split) * g * PSTR;
    __syncthreads();
    // scalars
    if (tid < g) {
        const int h = tid;
        float M = -INFINITY, MS = -INFINITY;
        for (int w = 0; w < NW; ++w) {
            M = fmaxf(M, ws4[w].m[h]);
            MS = fmaxf(MS, ws4[w].ms[h]);
        }
        float L = 0.f, E1 = 0.f, E2 = 0.f;
        for (int w = 0; w < NW; ++w) {
            if (ws4[w].l[h] > 0.f) L += ws4[w].l[h] * exp2f(ws4[w].m[h] - M);
            if (ws4[w].e1[h] > 0.f) {
                E1 += ws4[w].e1[h] * exp2f(ws4[w].ms[h] - MS);
                E2 += ws4[w].e2[h] * exp2f(2.f * (ws4[w].ms[h] - MS));
            }
        }
        part[h * PSTR + 0] = M;
        part[h * PSTR + 1] = L;
        part[h * PSTR + 2] = MS;
        part[h * PSTR + 3] = E1;
        part[h * PSTR + 4] = E2;
    }
    for (int i = tid; i < g * D; i += kAttThreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, ws4[w].m[h]);
        float acc = 0.f;
        for (int w = 0; w < NW; ++w)
            if (ws4[w].l[h] > 0.f) acc += ws4[w].o[h][d] * exp2f(ws4[w].m[h] - M);
        part[h * PSTR + 8 + d] = acc;
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) s_last = (atomicAdd(&a.ws.counters[bh], 1) == a.nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float *pall = a.ws.partial + (int64_t)bh * a.nsplit * g * PSTR;
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    for (int i = tid; i < g * D; i += kAttThreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
        for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, pall[(s * g + h) * PSTR + 0]);
        float L = 0.f, acc = 0.f;
        for (int s = 0; s < a.nsplit; ++s) {
            const float* ps = pall + (s * g + h) * PSTR;
            if (ps[1] > 0.f) {
                const float f = exp2f(ps[0] - M);
                L += ps[1] * f;
                acc += ps[8 + d] * f;
            }
        }
        const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
        a.out[oh * D + d] = L > 0.f ? acc / L : 0.f;
        if (d == 0) {
            if (a.lse) a.lse[oh] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
            if (a.ess) {
                float MS = -INFINITY;
                for (int s = 0; s < a.nsplit; ++s) MS = fmaxf(MS, pall[(s * g + h) * PSTR + 2]);
                float E1 = 0.f, E2 = 0.f;
                for (int s = 0; s < a.nsplit; ++s) {
                    const float* ps = pall + (s * g + h) * PSTR;
                    if (ps[3] > 0.f) {
                        E1 += ps[3] * exp2f(ps[2] - MS);
                        E2 += ps[4] * exp2f(2.f * (ps[2] - MS));
                    }
                }
                const int ns = a.ws.head_meta[((int64_t)bh * 8 + h) * 2 + 1];
                a.ess[oh] = (ns > 0 && E2 > 0.f) ? (E1 * E1 / E2) / (float)ns : 0.f;
            }
        }
    }
    if (tid == 0) a.ws.counters[bh] = 0;
}

__device__ __forceinline__ void split_range(const DecodeArgs &a, int total, int split, int *r0,
                                            int *r1) {
    const int per = ceil_div(ceil_div(total, a.nsplit), kTileRows) * kTileRows;
    *r0 = min(total, split * per);
    *r1 = min(total, *r0 + per);
}

// ---------------------------------------------------------------------------
// attend, SIMT (fp32 or bf16 caches): a warp per row, lanes over head_dim
// ---------------------------------------------------------------------------
template <int D, typename T>
__global__ void __launch_bounds__(kAttThreads) decode_attend_simt_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int split = blockIdx.x, bh = blockIdx.y;
    const int g = a.geo.group, Gmax = a.sum.max_groups;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    WarpState<D> *ws4 = (WarpState<D> *)smem_raw;
    int *u_off = (int *)(ws4 + kAttThreads / 32);
    int *u_start = u_off + Gmax + 1;
    int *u_mask = u_start + Gmax;
    float *qs = (float *)(u_mask + Gmax);  // [8][D], scaled by scale*log2e

    const int32_t *meta = a.ws.meta + (int64_t)bh * 8;
    const int n_union = meta[0], U = meta[1], R = meta[2], total = meta[4];
    for (int i = tid; i <= n_union; i += kAttThreads) u_off[i] = a.ws.u_off[(int64_t)bh * (Gmax + 1) + i];
    for (int i = tid; i < n_union; i += kAttThreads) {
        u_start[i] = a.ws.u_start[(int64_t)bh * Gmax + i];
        u_mask[i] = a.ws.u_mask[(int64_t)bh * Gmax + i];
    }
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    const float qscale = a.p.scale * kLog2e;
    for (int i = tid; i < g * D; i += kAttThreads) qs[i] = qb[i] * qscale;
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
    int r0, r1;
    split_range(a, total, split, &r0, &r1);
    const int row_bytes = D * (int)sizeof(T);
    for (int v = r0 + warp; v < r1; v += kAttThreads / 32) {
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
                const float lw = (ri.mask & 512) ? ri.off : s + ri.off;
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
                if (ri.mask & 256) {
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
    finish_cta<D>(a, bh, ws4, split);
}

// ---------------------------------------------------------------------------
// attend, tensor-core (bf16 caches): mma.sync m16n8k16, heads on M
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                            uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                                  uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t *)&v;
}

// Byte offset of 16-byte chunk c of row r in a swizzled tile with ROWB bytes
// per row: chunk index XOR (row mod 8), keeps 8-row ldmatrix reads
// bank-conflict free.
template <int ROWB>
__device__ __forceinline__ int swz(int r, int c) {
    return r * ROWB + ((c ^ (r & 7)) << 4);
}

template <int D>
struct MmaSmem {
    static constexpr int ROWB = D * 2;
    static constexpr int TILE_BYTES = kTileRows * ROWB;
    __nv_bfloat16 *k[kStages];
    __nv_bfloat16 *v[kStages];
    const char **kp[kStages];
    const char **vp[kStages];
    float *off[kStages];
    int *mask[kStages];
};

template <int D>
__global__ void __launch_bounds__(kAttThreads, 2) decode_attend_mma_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int ROWB = D * 2;
    constexpr int CPR = ROWB / 16;
    constexpr int TILE_BYTES = kTileRows * ROWB;
    constexpr int NT_O = D / 8;  // output n-tiles
    const int split = blockIdx.x, bh = blockIdx.y;
    const int g = a.geo.group, Gmax = a.sum.max_groups;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, tig = lane & 3;

    // carve shared memory
    // tiles start on a 128-byte boundary so the XOR swizzle maps to banks
    unsigned char *p = (unsigned char *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    __nv_bfloat16 *kt = (__nv_bfloat16 *)p;  p += kStages * TILE_BYTES;
    __nv_bfloat16 *vt = (__nv_bfloat16 *)p;  p += kStages * TILE_BYTES;
    __nv_bfloat16 *qhi = (__nv_bfloat16 *)p; p += 8 * ROWB;
    __nv_bfloat16 *qlo = (__nv_bfloat16 *)p; p += 8 * ROWB;
    const char **kp = (const char **)p;      p += kStages * kTileRows * sizeof(void *);
    const char **vp = (const char **)p;      p += kStages * kTileRows * sizeof(void *);
    float *roff = (float *)p;                p += kStages * kTileRows * 4;
    int *rmask = (int *)p;                   p += kStages * kTileRows * 4;
    int *u_off = (int *)p;                   p += (Gmax + 1) * 4;
    // the warp states of the final merge reuse the K stage buffers
    WarpState<D> *ws4 = (WarpState<D> *)kt;
    const int *u_start = a.ws.u_start + (int64_t)bh * Gmax;
    const int *u_mask = a.ws.u_mask + (int64_t)bh * Gmax;

    const int32_t *meta = a.ws.meta + (int64_t)bh * 8;
    const int n_union = meta[0], U = meta[1], R = meta[2], total = meta[4];
    for (int i = tid; i <= n_union; i += kAttThreads) u_off[i] = a.ws.u_off[(int64_t)bh * (Gmax + 1) + i];
    // q (scaled to log2 units) split into bf16 hi + lo, rows >= g are zero
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    const float *qb = a.q + ((int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g) * D;
    const float qscale = a.p.scale * kLog2e;
    for (int i = tid; i < 8 * D; i += kAttThreads) {
        const int h = i / D, d = i - h * D;
        const float x = h < g ? qb[h * D + d] * qscale : 0.f;
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
        const int off = swz<ROWB>(h, d >> 3) + (d & 7) * 2;
        *(__nv_bfloat16 *)((char *)qhi + off) = hi;
        *(__nv_bfloat16 *)((char *)qlo + off) = lo;
    }
    __syncthreads();

    int r0, r1;
    split_range(a, total, split, &r0, &r1);
    const int ntiles = ceil_div(r1 - r0, kTileRows);

    auto resolve_and_issue = [&](int t) {
        const int st = t % kStages;
        const int base = r0 + t * kTileRows;
        if (tid < kTileRows) {
            const int v = base + tid;
            RowInfo ri = resolve_row(a, bh, v, U, R, (v < r1) ? total : 0, n_union, u_off,
                                     u_start, u_mask, ROWB);
            kp[st * kTileRows + tid] = ri.k;
            vp[st * kTileRows + tid] = ri.v;
            roff[st * kTileRows + tid] = ri.off;
            rmask[st * kTileRows + tid] = ri.mask;
        }
        __syncthreads();
        const uint32_t kb = smem_u32((char *)kt + st * TILE_BYTES);
        const uint32_t vb = smem_u32((char *)vt + st * TILE_BYTES);
#pragma unroll
        for (int j = 0; j < (kTileRows * CPR) / kAttThreads; ++j) {
            const int q = tid + j * kAttThreads;
            const int r = q / CPR, c = q - r * CPR;
            const int valid = rmask[st * kTileRows + r] != 0 ? 16 : 0;
            const int so = swz<ROWB>(r, c);
            cp_async16(kb + so, kp[st * kTileRows + r] + c * 16, valid);
            cp_async16(vb + so, vp[st * kTileRows + r] + c * 16, valid);
        }
    };

    // per-thread softmax state for head gid (rows >= g of the M tile are padding)
    float m_run = -INFINITY, l_run = 0.f, ms_run = -INFINITY, e1_run = 0.f, e2_run = 0.f;
    float o[NT_O][4];
#pragma unroll
    for (int i = 0; i < NT_O; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    // prologue
#pragma unroll
    for (int t = 0; t < kStages - 1; ++t) {
        if (t < ntiles) resolve_and_issue(t);
        cp_async_commit();
    }

    for (int t = 0; t < ntiles; ++t) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        if (t + kStages - 1 < ntiles) resolve_and_issue(t + kStages - 1);
        cp_async_commit();

        const int st = t % kStages;
        const char *ks = (const char *)kt + st * TILE_BYTES;
        const char *vs = (const char *)vt + st * TILE_BYTES;
        const int rbase = warp * 16;  // this warp's 16 rows of the tile

        // S = Q K^T for 16 rows (two n8 tiles), q split hi + lo
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks16 = 0; ks16 < D / 16; ++ks16) {
            // A (q): rows 0-7 only; ldmatrix.x4 of rows gid, chunks 2ks, 2ks+1 for hi and lo
            uint32_t ah0, ah2, al0, al2;
            {
                const int mrow = lane & 7, which = lane >> 3;  // 0: hi c0, 1: hi c1, 2: lo c0, 3: lo c1
                const char *qbase = (which < 2) ? (const char *)qhi : (const char *)qlo;
                const uint32_t addr = smem_u32(qbase + swz<ROWB>(mrow, 2 * ks16 + (which & 1)));
                ldmatrix_x4(addr, ah0, ah2, al0, al2);
            }
            uint32_t b0, b1, b2, b3;
            {
                const int mat = lane >> 3, mrow = lane & 7;
                const int r = rbase + ((mat >> 1) << 3) + mrow;
                const int c = 2 * ks16 + (mat & 1);
                ldmatrix_x4(smem_u32(ks + swz<ROWB>(r, c)), b0, b1, b2, b3);
            }
            mma_bf16(s0, ah0, 0u, ah2, 0u, b0, b1);
            mma_bf16(s0, al0, 0u, al2, 0u, b0, b1);
            mma_bf16(s1, ah0, 0u, ah2, 0u, b2, b3);
            mma_bf16(s1, al0, 0u, al2, 0u, b2, b3);
        }
        // scores for head gid: rows rbase + {2tig, 2tig+1} (s0) and +8 (s1)
        const int *mk = rmask + st * kTileRows;
        const float *of = roff + st * kTileRows;
        float sv[4];
        int rr[4] = {rbase + 2 * tig, rbase + 2 * tig + 1, rbase + 8 + 2 * tig, rbase + 9 + 2 * tig};
        float raw[4] = {s0[0], s0[1], s1[0], s1[1]};
        bool any_sample = false;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int mm = mk[rr[i]];
            const bool on = gid < g && ((mm >> gid) & 1);
            sv[i] = on ? ((mm & 512) ? of[rr[i]] : raw[i] + of[rr[i]]) : -INFINITY;
            any_sample |= on && (mm & 256);
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
        // importance-sample diagnostics (ESS)
        if (__any_sync(0xffffffffu, any_sample)) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int mm = mk[rr[i]];
                if (gid < g && ((mm >> gid) & 1) && (mm & 256)) {
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
        // P (bf16 hi + lo) as the A operand: k = 16 rows of this warp
        const uint32_t ph0 = pack_bf16(pr[0], pr[1]);
        const uint32_t ph2 = pack_bf16(pr[2], pr[3]);
        const float2 f0 = __bfloat1622float2(*(const __nv_bfloat162 *)&ph0);
        const float2 f2 = __bfloat1622float2(*(const __nv_bfloat162 *)&ph2);
        const uint32_t pl0 = pack_bf16(pr[0] - f0.x, pr[1] - f0.y);
        const uint32_t pl2 = pack_bf16(pr[2] - f2.x, pr[3] - f2.y);
#pragma unroll
        for (int j = 0; j < D / 16; ++j) {
            uint32_t b0, b1, b2, b3;
            const int mat = lane >> 3, mrow = lane & 7;
            const int r = rbase + ((mat & 1) << 3) + mrow;
            const int c = 2 * j + (mat >> 1);
            ldmatrix_x4_trans(smem_u32(vs + swz<ROWB>(r, c)), b0, b1, b2, b3);
            mma_bf16(o[2 * j], ph0, 0u, ph2, 0u, b0, b1);
            mma_bf16(o[2 * j], pl0, 0u, pl2, 0u, b0, b1);
            mma_bf16(o[2 * j + 1], ph0, 0u, ph2, 0u, b2, b3);
            mma_bf16(o[2 * j + 1], pl0, 0u, pl2, 0u, b2, b3);
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    // reduce l / ess state over the 4 threads of the row group
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    {
        float MS = fmaxf(ms_run, __shfl_xor_sync(0xffffffffu, ms_run, 1));
        MS = fmaxf(MS, __shfl_xor_sync(0xffffffffu, MS, 2));
        float f = (e1_run > 0.f) ? exp2f(ms_run - MS) : 0.f;
        float E1 = e1_run * f, E2 = e2_run * f * f;
        E1 += __shfl_xor_sync(0xffffffffu, E1, 1);
        E1 += __shfl_xor_sync(0xffffffffu, E1, 2);
        E2 += __shfl_xor_sync(0xffffffffu, E2, 1);
        E2 += __shfl_xor_sync(0xffffffffu, E2, 2);
        ms_run = MS;
        e1_run = E1;
        e2_run = E2;
    }
    __syncthreads();
    if (gid < SANTA_MAX_GROUP) {
        if (tig == 0) {
            ws4[warp].m[gid] = m_run;
            ws4[warp].l[gid] = l_run;
            ws4[warp].ms[gid] = ms_run;
            ws4[warp].e1[gid] = e1_run;
            ws4[warp].e2[gid] = e2_run;
        }
#pragma unroll
        for (int i = 0; i < NT_O; ++i) {
            ws4[warp].o[gid][i * 8 + 2 * tig] = o[i][0];
            ws4[warp].o[gid][i * 8 + 2 * tig + 1] = o[i][1];
        }
    }
    finish_cta<D>(a, bh, ws4, split);
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
        if (selected) {
            for (int c = threadIdx.x; c < Gmax; c += blockDim.x) selected[oh * Gmax + c] = 0;
        }
        if (sample_rows && S > 0) {
            for (int i = threadIdx.x; i < S; i += blockDim.x) sample_rows[oh * S + i] = -1;
        }
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
// host side
// ---------------------------------------------------------------------------
static int g_num_sms = 0;

static int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

static int pick_splits(const SantaGeometry *geo, const SantaDecodeParams *p) {
    if (p->num_splits > 0) return p->num_splits;
    const int BH = geo->batch * geo->num_kv_heads;
    const int slots = 2 * num_sms();
    int s = slots / BH;
    if (s < 1) s = 1;
    if (s > 64) s = 64;
    return s;
}

static size_t select_smem_bytes(int D, int Gmax) {
    int Gp = 1;
    while (Gp < Gmax) Gp <<= 1;
    size_t b = 0;
    b += SANTA_MAX_GROUP * D * 4;
    b += 64 * (D + 1) * 4;
    b += 3 * (size_t)Gmax * 4;
    b += SANTA_MAX_GROUP * (size_t)Gmax * 4;  // guess
    b += SANTA_MAX_GROUP * (size_t)Gmax * 4;  // selasc
    b += 40 * 4 + 32 * 4 + 32 * 4 + 32;
    b += SANTA_MAX_GROUP * (size_t)Gp * 8;    // keys
    return b;
}

template <int D>
static size_t mma_smem_bytes(int Gmax) {
    size_t b = 0;
    b += 128;  // alignment slack for the tile base
    b += 2 * (size_t)kStages * kTileRows * D * 2;
    b += 2 * 8 * D * 2;
    b += 2 * (size_t)kStages * kTileRows * sizeof(void *);
    b += 2 * (size_t)kStages * kTileRows * 4;
    b += ((size_t)Gmax + 1) * 4;
    static_assert(sizeof(WarpState<D>) * (kAttThreads / 32) <= (size_t)kStages * kTileRows * D * 2,
                  "warp states must fit in the K stage buffers");
    return b;
}

template <int D>
static size_t simt_smem_bytes(int Gmax) {
    return sizeof(WarpState<D>) * (kAttThreads / 32) + (3 * (size_t)Gmax + 1) * 4 +
           SANTA_MAX_GROUP * D * 4;
}

// Raise the dynamic shared-memory limit of a kernel once per process and size.
template <typename K>
static int ensure_smem(K kernel, size_t bytes, size_t *done) {
    if (*done >= bytes) return SANTA_OK;
    SANTA_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)bytes));
    *done = bytes;
    return SANTA_OK;
}

// Selection phase: [santa: old-prefix LSE] + select kernel -> work list.
template <int D>
static int launch_plan(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups;
    SANTA_CUDA_CHECK(cudaMemsetAsync(a.ws.flag, 0, 16, stream));
    if (a.p.mode == SANTA_MODE_SANTA) {
        if (a.geo.kv_dtype == SANTA_DTYPE_BF16)
            decode_old_lse_kernel<D, __nv_bfloat16><<<BH, 256, 0, stream>>>(a);
        else
            decode_old_lse_kernel<D, float><<<BH, 256, 0, stream>>>(a);
        SANTA_LAUNCH_CHECK();
    }
    static size_t sel_done = 0;
    const size_t sel_smem = select_smem_bytes(D, Gmax);
    int st = ensure_smem(decode_select_kernel<D>, sel_smem, &sel_done);
    if (st) return st;
    decode_select_kernel<D><<<BH, kSelThreads, sel_smem, stream>>>(a);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

// Attention phase over the work list written by launch_plan.
template <int D>
static int launch_execute(DecodeArgs &a, cudaStream_t stream) {
    const int BH = a.geo.batch * a.geo.num_kv_heads;
    const int Gmax = a.sum.max_groups;
    SANTA_CUDA_CHECK(cudaMemsetAsync(a.ws.counters, 0, (size_t)BH * 4, stream));
    dim3 grid(a.nsplit, BH);
    if (a.geo.kv_dtype == SANTA_DTYPE_BF16) {
        static size_t done = 0;
        const size_t sm = mma_smem_bytes<D>(Gmax);
        int st = ensure_smem(decode_attend_mma_kernel<D>, sm, &done);
        if (st) return st;
        decode_attend_mma_kernel<D><<<grid, kAttThreads, sm, stream>>>(a);
    } else {
        static size_t done = 0;
        const size_t sm = simt_smem_bytes<D>(Gmax);
        int st = ensure_smem(decode_attend_simt_kernel<D, float>, sm, &done);
        if (st) return st;
        decode_attend_simt_kernel<D, float><<<grid, kAttThreads, sm, stream>>>(a);
    }
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

template <int D>
static int launch_decode(DecodeArgs &a, cudaStream_t stream, bool attend = true) {
    int st = launch_plan<D>(a, stream);
    if (st || !attend) return st;
    return launch_execute<D>(a, stream);
}

}  // namespace santa

using namespace santa;

extern "C" int santa_check_geometry(const SantaGeometry *geo);

static int check_decode(const SantaGeometry *geo, const SantaDecodeParams *p, int max_groups) {
    int st = santa_check_geometry(geo);
    if (st) return st;
    if (!p) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->mode < SANTA_MODE_TOPK || p->mode > SANTA_MODE_HYBRID) return SANTA_ERR_INVALID_ARGUMENT;
    if (max_groups <= 0 || max_groups > SANTA_MAX_CLUSTERS) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->samples < 0 || p->samples > SANTA_MAX_SAMPLES) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->mode != SANTA_MODE_TOPK && p->samples <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->mode == SANTA_MODE_TOPK && p->token_budget <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->mode == SANTA_MODE_HYBRID && (p->topk_clusters < 0 || p->topk_clusters > max_groups))
        return SANTA_ERR_INVALID_ARGUMENT;
    if (geo->sample_end >= (1 << 24)) return SANTA_ERR_UNSUPPORTED;
    if (!(p->scale > 0.f)) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->num_splits < 0 || p->num_splits > 256) return SANTA_ERR_INVALID_ARGUMENT;
    return SANTA_OK;
}

extern "C" int santa_decode_workspace_bytes(const SantaGeometry *geo, const SantaDecodeParams *p,
                                            int32_t max_groups, size_t *bytes) {
    int st = check_decode(geo, p, max_groups);
    if (st) return st;
    if (!bytes) return SANTA_ERR_INVALID_ARGUMENT;
    const int BH = geo->batch * geo->num_kv_heads;
    *bytes = decode_ws_layout(BH, max_groups, geo->group, p->samples, pick_splits(geo, p),
                              geo->head_dim, nullptr, nullptr);
    return SANTA_OK;
}

static int prepare_decode(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                          const void *key_cache, const void *value_cache,
                          const SantaSummary *summary, const int32_t *sample_a,
                          const int32_t *sample_b, void *workspace, size_t workspace_bytes,
                          cudaStream_t stream, DecodeArgs *a) {
    if (!summary) return SANTA_ERR_INVALID_ARGUMENT;
    int st = check_decode(geo, p, summary->max_groups);
    if (st) return st;
    if (!q || !key_cache || !value_cache) return SANTA_ERR_INVALID_ARGUMENT;
    const bool needs_summary = p->mode == SANTA_MODE_TOPK || p->mode == SANTA_MODE_GUIDED ||
                               p->mode == SANTA_MODE_HYBRID;
    if (needs_summary && (!summary->starts || !summary->lengths || !summary->log_n ||
                          !summary->centroids || !summary->n_groups))
        return SANTA_ERR_INVALID_ARGUMENT;
    if (!summary->sorted_key || !summary->sorted_value) return SANTA_ERR_INVALID_ARGUMENT;
    if ((p->mode == SANTA_MODE_UNIFORM || p->mode == SANTA_MODE_SANTA) && !summary->positions)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (p->sample_source == SANTA_SAMPLES_INJECTED && p->mode != SANTA_MODE_TOPK) {
        if (!sample_a) return SANTA_ERR_INVALID_ARGUMENT;
        if (p->mode == SANTA_MODE_GUIDED && !sample_b) return SANTA_ERR_INVALID_ARGUMENT;
    }
    const int BH = geo->batch * geo->num_kv_heads;
    const int nsplit = pick_splits(geo, p);
    const size_t need = decode_ws_layout(BH, summary->max_groups, geo->group, p->samples, nsplit,
                                         geo->head_dim, nullptr, nullptr);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    a->geo = *geo;
    a->p = *p;
    a->sum = *summary;
    a->q = q;
    a->key_cache = (const char *)key_cache;
    a->value_cache = (const char *)value_cache;
    a->sample_a = sample_a;
    a->sample_b = sample_b;
    a->out = nullptr;
    a->lse = nullptr;
    a->n_exact = nullptr;
    a->ess = nullptr;
    a->nsplit = nsplit;
    decode_ws_layout(BH, summary->max_groups, geo->group, p->samples, nsplit, geo->head_dim,
                     (char *)workspace, &a->ws);
    return SANTA_OK;
}

extern "C" int santa_decode_plan(const SantaGeometry *geo, const SantaDecodeParams *p,
                                 const float *q, const void *key_cache, const void *value_cache,
                                 const SantaSummary *summary, const int32_t *sample_a,
                                 const int32_t *sample_b, int32_t *n_exact, void *workspace,
                                 size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b,
                            workspace, workspace_bytes, stream, &a);
    if (st) return st;
    a.n_exact = n_exact;
    return geo->head_dim == 64 ? launch_plan<64>(a, stream) : launch_plan<128>(a, stream);
}

extern "C" int santa_decode_execute(const SantaGeometry *geo, const SantaDecodeParams *p,
                                    const float *q, const void *key_cache,
                                    const void *value_cache, const SantaSummary *summary,
                                    float *out, float *lse, float *ess, void *workspace,
                                    size_t workspace_bytes, cudaStream_t stream) {
    if (!out) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, nullptr, nullptr,
                            workspace, workspace_bytes, stream, &a);
    if (st == SANTA_ERR_INVALID_ARGUMENT && p && p->sample_source == SANTA_SAMPLES_INJECTED) {
        // execute does not read the draws; accept NULL for them
        SantaDecodeParams p2 = *p;
        p2.sample_source = SANTA_SAMPLES_DEVICE;
        st = prepare_decode(geo, &p2, q, key_cache, value_cache, summary, nullptr, nullptr,
                            workspace, workspace_bytes, stream, &a);
    }
    if (st) return st;
    a.out = out;
    a.lse = lse;
    a.ess = ess;
    return geo->head_dim == 64 ? launch_execute<64>(a, stream) : launch_execute<128>(a, stream);
}

extern "C" int santa_decode(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                            const void *key_cache, const void *value_cache,
                            const SantaSummary *summary, const int32_t *sample_a,
                            const int32_t *sample_b, float *out, float *lse, int32_t *n_exact,
                            float *ess, void *workspace, size_t workspace_bytes,
                            cudaStream_t stream) {
    if (!out) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b,
                            workspace, workspace_bytes, stream, &a);
    if (st) return st;
    a.out = out;
    a.lse = lse;
    a.n_exact = n_exact;
    a.ess = ess;
    if (geo->head_dim == 64) return launch_decode<64>(a, stream);
    return launch_decode<128>(a, stream);
}

extern "C" int santa_decode_select(const SantaGeometry *geo, const SantaDecodeParams *p,
                                   const float *q, const void *key_cache, const void *value_cache,
                                   const SantaSummary *summary, const int32_t *sample_a,
                                   const int32_t *sample_b, uint8_t *selected,
                                   int32_t *sample_rows, int32_t *n_exact, void *workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b,
                            workspace, workspace_bytes, stream, &a);
    if (st) return st;
    a.n_exact = n_exact;
    st = geo->head_dim == 64 ? launch_decode<64>(a, stream, false)
                             : launch_decode<128>(a, stream, false);
    if (st) return st;
    decode_expand_kernel<<<geo->batch * geo->num_kv_heads, 256, 0, stream>>>(a, selected,
                                                                          sample_rows);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}
