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
#include "decode_common.cuh"

#include <math.h>

namespace santa {

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
    int *selasc = (int *)(guess_s + SANTA_MAX_GROUP * Gmax);    // [8][2*Gmax+1] gap / cum
    int *sw = selasc + SANTA_MAX_GROUP * (2 * Gmax + 1);        // [40]
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
        // 64-centroid tiles, loaded as float4 into registers one tile ahead so
        // the HBM round trip of tile t+1 overlaps the dot products of tile t.
        constexpr int V4 = 64 * D / 4 / kSelThreads;  // float4 per thread per tile
        float4 pre[V4];
        auto load_tile = [&](int c0) {
            const int nc = min(64, n_groups - c0);
#pragma unroll
            for (int j = 0; j < V4; ++j) {
                const int i = tid + j * kSelThreads;  // float4 index in the tile
                const int r = (i * 4) / D;
                pre[j] = r < nc ? *(const float4 *)(cent + (int64_t)(c0 + r) * D + (i * 4 - r * D))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        };
        if (n_groups > 0) load_tile(0);
        for (int c0 = 0; c0 < n_groups; c0 += 64) {
            const int nc = min(64, n_groups - c0);
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
            if (c0 + 64 < n_groups) load_tile(c0 + 64);
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

    // ---- ranking (TOPK / HYBRID): one warp per query head extracts clusters
    // in descending (guess, -index) order by repeated warp arg-max; this is
    // the prefix of argsort(guess, descending, stable) that the selection uses.
    if (mode == SANTA_MODE_TOPK || mode == SANTA_MODE_HYBRID) {
        if (warp < g) {
            const int h = warp;
            uint64_t *arr = keys + h * Gp;
            uint64_t best = 0;  // lane-local maximum key
            for (int c = lane; c < n_groups; c += 32) {
                const uint64_t k = ((uint64_t)float_order_key(guess_s[h * Gmax + c]) << 32) |
                                   (uint64_t)(0xFFFFFFFFu - (uint32_t)c);
                arr[c] = k;
                best = k > best ? k : best;
            }
            const int kmax = (mode == SANTA_MODE_HYBRID) ? min(a.p.topk_clusters, n_groups)
                                                         : n_groups;
            int nsel = 0, exact = 0;
            while (nsel < kmax) {
                // 64-bit warp max in two redux.sync steps: the largest high
                // word, then the largest low word among the lanes holding it
                const uint32_t bhi = (uint32_t)(best >> 32);
                const uint32_t mhi = __reduce_max_sync(0xffffffffu, bhi);
                const uint32_t mlo =
                    __reduce_max_sync(0xffffffffu, bhi == mhi ? (uint32_t)best : 0u);
                const uint64_t m = ((uint64_t)mhi << 32) | mlo;
                if (m == 0) break;  // no cluster left
                const int c = (int)(0xFFFFFFFFu - (uint32_t)(m & 0xFFFFFFFFu));
                const int l = len_s[c];
                if (lane == (c & 31)) {
                    atomicOr(&mask_s[c], 1 << h);
                    arr[c] = 0;
                    best = 0;
                    for (int cc = lane; cc < n_groups; cc += 32)
                        best = arr[cc] > best ? arr[cc] : best;
                }
                exact += l;
                ++nsel;
                // budget walk (santapp.py:404-410): stop once the chosen
                // clusters hold at least token_budget tokens
                if (mode == SANTA_MODE_TOPK && exact >= a.p.token_budget) break;
            }
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
        // union entries also kept in shared memory (the centroid tile area is
        // free after scoring: 64 * (D + 1) floats >= 3 * 1024 ints)
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
        // inclusive cdf of the unnormalised probabilities (keys[] reused as floats)
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
            // Selected clusters of this head in ascending cluster (= start)
            // order, as gap[j] = non-selected positions before cluster j and
            // cum[j] = selected positions before cluster j.  Rank r maps to
            // position r + cum[J] with J = #{j : gap[j] <= r}.
            int *gap = selasc + h * (2 * Gmax + 1);
            int *cum = gap + Gmax;
            int cnt = 0, carry = 0;
            for (int c0 = 0; c0 < n_groups; c0 += 32) {
                const int c = c0 + lane;
                const bool on = c < n_groups && ((mask_s[c] >> h) & 1);
                const unsigned bal = __ballot_sync(0xffffffffu, on);
                int l = on ? len_s[c] : 0;
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
            if (lane == 0) cum[cnt] = carry;
            __syncwarp();
            const int n_rest = sample_end - head_exact[h];
            const float off = (logf((float)n_rest) - logS) * kLog2e;
            for (int i = lane; i < ns; i += 32) {
                uint32_t r;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    int v = a.sample_a[inj + i];
                    if (v < 0 || v >= n_rest) {
                        atomicExch(a.ws.flag + kFlagBadDraw, 1);
                        v = min(max(v, 0), n_rest - 1);
                    }
                    r = (uint32_t)v;
                } else {
                    const uint4 w = philox4x32_10(
                        make_uint4((uint32_t)(i >> 2), (uint32_t)gh, (uint32_t)b, (uint32_t)a.p.step),
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
            const float *cdf = (const float *)keys + h * Gmax;
            const float total = cdf[n_groups - 1];
            const float *logn = a.sum.log_n + (int64_t)bh * Gmax;
            for (int i = lane; i < ns; i += 32) {
                int grp, within;
                if (a.p.sample_source == SANTA_SAMPLES_INJECTED) {
                    grp = a.sample_a[inj + i];
                    within = a.sample_b[inj + i];
                    if (grp < 0 || grp >= n_groups) {
                        atomicExch(a.ws.flag + kFlagBadDraw, 1);
                        grp = min(max(grp, 0), n_groups - 1);
                    }
                    if (within < 0 || within >= len_s[grp]) {
                        atomicExch(a.ws.flag + kFlagBadDraw, 1);
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
                        atomicExch(a.ws.flag + kFlagBadDraw, 1);
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
static size_t select_smem_bytes(int D, int Gmax) {
    int Gp = 1;
    while (Gp < Gmax) Gp <<= 1;
    size_t b = 0;
    b += SANTA_MAX_GROUP * D * 4;
    b += 64 * (D + 1) * 4;
    b += 3 * (size_t)Gmax * 4;
    b += SANTA_MAX_GROUP * (size_t)Gmax * 4;  // guess
    b += SANTA_MAX_GROUP * (2 * (size_t)Gmax + 1) * 4;  // gap / cum per head
    b += 40 * 4 + 32 * 4 + 32 * 4 + 32;
    b += SANTA_MAX_GROUP * (size_t)Gp * 8;    // keys
    return b;
}

template <int D>
static int launch_plan_d(DecodeArgs &a, cudaStream_t stream) {
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
    static size_t done = 0;
    const size_t smem = select_smem_bytes(D, Gmax);
    if (done < smem) {
        SANTA_CUDA_CHECK(cudaFuncSetAttribute(decode_select_kernel<D>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem));
        done = smem;
    }
    decode_select_kernel<D><<<BH, kSelThreads, smem, stream>>>(a);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
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

static int g_num_sms = 0;

int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            g_num_sms <= 0) {
            cudaGetLastError();
            g_num_sms = 148;
        }
    }
    return g_num_sms;
}

}  // namespace santa
