// Cluster-summary build: stable counting sort of tokens by cluster label,
// cluster-sorted K/V copy, and key centroids.
//
// Replaces SantaPlusEngine._build_summary (santapp_ruler/attention/santapp.py:508-540).
//   counts   = bincount(labels)                      -> per-chunk histograms + scan
//   members  = argsort(labels) (stable)              -> warp-ranked scatter
//   starts   = exclusive cumsum(counts)[active]      -> same scan
//   centroid = index_add_(labels, keys)[active] / n  -> sequential fp32 sums in
//              ascending token order (CPU index_add_ order), IEEE division.
//
// Layout per (batch b, KV head kv) = segment bh = b * Hkv + kv; the old prefix
// has N = sample_end tokens split into chunks of kChunk tokens, one warp each.
#include "common.cuh"

namespace santa {

constexpr int kChunk = 1024;          // tokens per warp chunk
constexpr int kWarpsPerCta = 4;

struct SummaryWs {
    int32_t *flag;        // [4]: [0] = invalid label seen
    int32_t *chunk_off;   // [BH][G][nchunks]  histogram, then exclusive offsets
    int32_t *counts;      // [BH][G]
    int32_t *active_idx;  // [BH][G]  row of a non-empty cluster, -1 if empty
    int32_t *full_start;  // [BH][G]
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static size_t summary_ws_layout(int BH, int G, int nchunks, char *base, SummaryWs *ws) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    size_t o_flag = take(16);
    size_t o_hist = take((size_t)BH * G * nchunks * 4);
    size_t o_cnt = take((size_t)BH * G * 4);
    size_t o_act = take((size_t)BH * G * 4);
    size_t o_fs = take((size_t)BH * G * 4);
    if (base && ws) {
        ws->flag = (int32_t *)(base + o_flag);
        ws->chunk_off = (int32_t *)(base + o_hist);
        ws->counts = (int32_t *)(base + o_cnt);
        ws->active_idx = (int32_t *)(base + o_act);
        ws->full_start = (int32_t *)(base + o_fs);
    }
    return off;
}

// ---------------------------------------------------------------------------
// 1. per-chunk label histograms (integer atomics: exact, order-free)
// ---------------------------------------------------------------------------
__global__ void summary_count_kernel(const int32_t *__restrict__ labels, int N, int G,
                                     int nchunks, SummaryWs ws) {
    extern __shared__ int32_t hist[];  // [kWarpsPerCta][G]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int chunk = blockIdx.x * kWarpsPerCta + warp;
    int32_t *h = hist + warp * G;
    for (int i = lane; i < G; i += 32) h[i] = 0;
    __syncwarp();
    if (chunk < nchunks) {
        const int32_t *lab = labels + (int64_t)bh * N;
        const int t0 = chunk * kChunk;
        const int t1 = min(N, t0 + kChunk);
        for (int t = t0 + lane; t < t1; t += 32) {
            const int l = lab[t];
            if (l >= 0 && l < G) atomicAdd(&h[l], 1);
            else atomicExch(ws.flag, 1);
        }
    }
    __syncwarp();
    if (chunk < nchunks) {
        int32_t *dst = ws.chunk_off + (int64_t)bh * G * nchunks + chunk;
        for (int i = lane; i < G; i += 32) dst[(int64_t)i * nchunks] = h[i];
    }
}

// ---------------------------------------------------------------------------
// 2. exclusive scan over [G][nchunks] (label-major), cluster counts, active rows
// ---------------------------------------------------------------------------
__device__ int block_exclusive_scan_1024(int v, int *smem_warp, int *total) {
    // blockDim.x == 1024
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = smem_warp[lane];
        int s = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        smem_warp[lane] = s - w;  // exclusive warp offsets
        if (lane == 31) smem_warp[32] = s;
    }
    __syncthreads();
    int res = smem_warp[warp] + x - v;
    if (total) *total = smem_warp[32];
    __syncthreads();
    return res;
}

__global__ void __launch_bounds__(1024) summary_scan_kernel(int G, int nchunks, SummaryWs ws,
                                                            SantaSummary out) {
    __shared__ int sw[33];
    const int bh = blockIdx.x;
    int32_t *a = ws.chunk_off + (int64_t)bh * G * nchunks;
    const int64_t E = (int64_t)G * nchunks;
    const int per = (int)ceil_div64(E, 1024);
    const int64_t b0 = (int64_t)threadIdx.x * per;
    int local = 0;
    for (int i = 0; i < per; ++i)
        if (b0 + i < E) local += a[b0 + i];
    int tot;
    int run = block_exclusive_scan_1024(local, sw, &tot);
    for (int i = 0; i < per; ++i) {
        if (b0 + i < E) {
            int v = a[b0 + i];
            a[b0 + i] = run;
            run += v;
        }
    }
    __syncthreads();
    // counts and active rows; one thread per label (G <= 1024)
    const int g = threadIdx.x;
    int cnt = 0, fstart = 0;
    if (g < G) {
        fstart = a[(int64_t)g * nchunks];
        int next = (g + 1 < G) ? a[(int64_t)(g + 1) * nchunks] : tot;
        cnt = next - fstart;
    }
    int n_active;
    int rank = block_exclusive_scan_1024((g < G && cnt > 0) ? 1 : 0, sw, &n_active);
    if (g < G) {
        ws.counts[(int64_t)bh * G + g] = cnt;
        ws.full_start[(int64_t)bh * G + g] = fstart;
        ws.active_idx[(int64_t)bh * G + g] = cnt > 0 ? rank : -1;
        const int64_t o = (int64_t)bh * out.max_groups;
        if (cnt > 0) {
            out.starts[o + rank] = fstart;
            out.lengths[o + rank] = cnt;
            out.log_n[o + rank] = (float)log((double)cnt);
        }
    }
    if (threadIdx.x == 0) out.n_groups[bh] = n_active;
    // rows beyond n_groups are left untouched except a zero length marker
    if (g < G && g >= n_active) {
        const int64_t o = (int64_t)bh * out.max_groups;
        out.starts[o + g] = 0;
        out.lengths[o + g] = 0;
        out.log_n[o + g] = 0.0f;
    }
}

// ---------------------------------------------------------------------------
// 3. stable scatter: members / positions and the cluster-sorted K/V copy
// ---------------------------------------------------------------------------
template <int ROW_BYTES>
__global__ void summary_scatter_kernel(const int32_t *__restrict__ labels,
                                       const char *__restrict__ key_cache,
                                       const char *__restrict__ value_cache,
                                       int N, int G, int nchunks, SantaGeometry geo,
                                       SummaryWs ws, SantaSummary out) {
    extern __shared__ int32_t running_all[];  // [kWarpsPerCta][G]
    constexpr int CPR = ROW_BYTES / 16;        // 16-byte chunks per row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int chunk = blockIdx.x * kWarpsPerCta + warp;
    if (chunk >= nchunks) return;
    int32_t *running = running_all + warp * G;
    const int32_t *offs = ws.chunk_off + (int64_t)bh * G * nchunks + chunk;
    for (int i = lane; i < G; i += 32) running[i] = offs[(int64_t)i * nchunks];
    __syncwarp();

    const int32_t *lab = labels + (int64_t)bh * N;
    int32_t *members = out.members + (int64_t)bh * N;
    int32_t *positions = out.positions + (int64_t)bh * N;
    char *kdst = (char *)out.sorted_key + (int64_t)bh * N * ROW_BYTES;
    char *vdst = (char *)out.sorted_value + (int64_t)bh * N * ROW_BYTES;

    const int t0 = chunk * kChunk;
    const int t1 = min(N, t0 + kChunk);
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int base_t = t0; base_t < t1; base_t += 32) {
        const int t = base_t + lane;
        const bool valid = t < t1;
        int l = valid ? lab[t] : -1;
        const bool ok = valid && l >= 0 && l < G;
        if (!ok) l = -1 - lane;  // unique sentinel: never matches a real label
        const unsigned peers = __match_any_sync(0xffffffffu, l);
        int pos = -1;
        if (ok) {
            const int rank = __popc(peers & lt_mask);
            pos = running[l] + rank;
        }
        __syncwarp();
        if (ok && (__ffs(peers) - 1) == lane) running[l] += __popc(peers);
        __syncwarp();
        if (ok) {
            members[pos] = t;
            positions[t] = pos;
        }
        // the cache row of this lane's token (contiguous or paged)
        const long long src = valid ? (long long)cache_row(geo, bh, t) * ROW_BYTES : 0;
        // cooperative 16-byte row copies for the 32 tokens of this step
        for (int i = lane; i < 32 * CPR; i += 32) {
            const int r = i / CPR, c = i - r * CPR;
            const int pr = __shfl_sync(0xffffffffu, pos, r);
            const long long sr = __shfl_sync(0xffffffffu, src, r);
            if (pr >= 0) {
                const int4 kv = *(const int4 *)(key_cache + sr + c * 16);
                const int4 vv = *(const int4 *)(value_cache + sr + c * 16);
                *(int4 *)(kdst + (int64_t)pr * ROW_BYTES + c * 16) = kv;
                *(int4 *)(vdst + (int64_t)pr * ROW_BYTES + c * 16) = vv;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 4. centroids: sequential fp32 sums in ascending token order, then divide
// ---------------------------------------------------------------------------
template <typename T>
__global__ void summary_centroid_kernel(int N, int G, int D, SummaryWs ws, SantaSummary out) {
    const int g = blockIdx.x, bh = blockIdx.y;
    const int idx = ws.active_idx[(int64_t)bh * G + g];
    if (idx < 0) return;
    const int n = ws.counts[(int64_t)bh * G + g];
    const int start = ws.full_start[(int64_t)bh * G + g];
    const T *rows = (const T *)out.sorted_key + ((int64_t)bh * N + start) * D;
    const float nf = (float)n;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.0f;
        for (int r = 0; r < n; ++r) acc = __fadd_rn(acc, to_f32<T>(rows[(int64_t)r * D + d]));
        out.centroids[((int64_t)bh * out.max_groups + idx) * D + d] = __fdiv_rn(acc, nf);
    }
}

}  // namespace santa

using namespace santa;

static int check_geo(const SantaGeometry *geo) {
    if (!geo) return SANTA_ERR_INVALID_ARGUMENT;
    if (geo->batch <= 0 || geo->num_kv_heads <= 0 || geo->group <= 0 ||
        geo->group > SANTA_MAX_GROUP)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (geo->head_dim != 64 && geo->head_dim != 128) return SANTA_ERR_UNSUPPORTED;
    if (geo->kv_dtype != SANTA_DTYPE_F32 && geo->kv_dtype != SANTA_DTYPE_BF16)
        return SANTA_ERR_UNSUPPORTED;
    if (geo->n_total <= 0 || geo->capacity < geo->n_total) return SANTA_ERR_INVALID_ARGUMENT;
    if (geo->sample_end <= 0 || geo->sample_end > geo->n_total) return SANTA_ERR_INVALID_ARGUMENT;
    if (geo->block_table) {
        // paged: page_size a power of two, capacity = max_pages * page_size
        if (geo->page_size <= 0 || (geo->page_size & (geo->page_size - 1)) ||
            geo->max_pages <= 0 || geo->num_pages <= 0 ||
            (int64_t)geo->max_pages * geo->page_size != geo->capacity)
            return SANTA_ERR_INVALID_ARGUMENT;
    }
    // recent rows travel as negative 32-bit row codes in the gather kernel
    if (cache_rows(*geo) >= (int64_t)INT32_MAX - 1) return SANTA_ERR_UNSUPPORTED;
    return SANTA_OK;
}

extern "C" int santa_check_geometry(const SantaGeometry *geo) { return check_geo(geo); }

extern "C" int santa_build_summary_workspace_bytes(const SantaGeometry *geo, int32_t n_clusters,
                                                   size_t *bytes) {
    int st = check_geo(geo);
    if (st) return st;
    if (!bytes || n_clusters <= 0 || n_clusters > SANTA_MAX_CLUSTERS)
        return SANTA_ERR_INVALID_ARGUMENT;
    const int BH = geo->batch * geo->num_kv_heads;
    const int nchunks = ceil_div(geo->sample_end, kChunk);
    *bytes = summary_ws_layout(BH, n_clusters, nchunks, nullptr, nullptr);
    return SANTA_OK;
}

extern "C" int santa_build_summary(const SantaGeometry *geo, const void *key_cache,
                                   const void *value_cache, const int32_t *labels,
                                   int32_t n_clusters, const SantaSummary *out,
                                   void *workspace, size_t workspace_bytes,
                                   cudaStream_t stream) {
    int st = check_geo(geo);
    if (st) return st;
    if (!key_cache || !value_cache || !labels || !out || n_clusters <= 0 ||
        n_clusters > SANTA_MAX_CLUSTERS || out->max_groups < n_clusters)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (!out->members || !out->positions || !out->starts || !out->lengths || !out->log_n ||
        !out->centroids || !out->n_groups || !out->sorted_key || !out->sorted_value)
        return SANTA_ERR_INVALID_ARGUMENT;
    const int BH = geo->batch * geo->num_kv_heads;
    const int N = geo->sample_end, G = n_clusters, D = geo->head_dim;
    const int nchunks = ceil_div(N, kChunk);
    size_t need = summary_ws_layout(BH, G, nchunks, nullptr, nullptr);
    if (!workspace || workspace_bytes < need) return SANTA_ERR_WORKSPACE;
    SummaryWs ws;
    summary_ws_layout(BH, G, nchunks, (char *)workspace, &ws);
    SANTA_CUDA_CHECK(cudaMemsetAsync(ws.flag, 0, 16, stream));

    const int esize = geo->kv_dtype == SANTA_DTYPE_BF16 ? 2 : 4;
    const int row_bytes = D * esize;
    dim3 grid_c(ceil_div(nchunks, kWarpsPerCta), BH);
    const size_t smem_c = (size_t)kWarpsPerCta * G * sizeof(int32_t);
    summary_count_kernel<<<grid_c, 32 * kWarpsPerCta, smem_c, stream>>>(labels, N, G, nchunks, ws);
    SANTA_LAUNCH_CHECK();
    summary_scan_kernel<<<BH, 1024, 0, stream>>>(G, nchunks, ws, *out);
    SANTA_LAUNCH_CHECK();
    switch (row_bytes) {
        case 128:
            summary_scatter_kernel<128><<<grid_c, 32 * kWarpsPerCta, smem_c, stream>>>(
                labels, (const char *)key_cache, (const char *)value_cache, N, G, nchunks,
                *geo, ws, *out);
            break;
        case 256:
            summary_scatter_kernel<256><<<grid_c, 32 * kWarpsPerCta, smem_c, stream>>>(
                labels, (const char *)key_cache, (const char *)value_cache, N, G, nchunks,
                *geo, ws, *out);
            break;
        case 512:
            summary_scatter_kernel<512><<<grid_c, 32 * kWarpsPerCta, smem_c, stream>>>(
                labels, (const char *)key_cache, (const char *)value_cache, N, G, nchunks,
                *geo, ws, *out);
            break;
        default:
            return SANTA_ERR_UNSUPPORTED;
    }
    SANTA_LAUNCH_CHECK();
    dim3 grid_m(G, BH);
    if (geo->kv_dtype == SANTA_DTYPE_BF16)
        summary_centroid_kernel<__nv_bfloat16><<<grid_m, D, 0, stream>>>(N, G, D, ws, *out);
    else
        summary_centroid_kernel<float><<<grid_m, D, 0, stream>>>(N, G, D, ws, *out);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}
