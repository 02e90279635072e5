// KV cache maintenance of the attention layer (santapp_ruler/attention/
// santapp.py:66-77 LayerCache, :234-283 _append_cache / _trim_cache, and the
// RoPE of _attention_forward :308-313), fused into one launch per layer call:
//
//   q_rot = q * cos + rotate_half(q) * sin        (bf16 tensors, as torch
//   k_rot = k * cos + rotate_half(k) * sin         computes them: each product
//                                                  and the sum rounded to bf16)
//   cache_k[b, kv, start + t] = k_rot[b, kv, t];  cache_v[...] = v[b, kv, t]
//
// rotate_half(x) = cat(-x[D/2:], x[:D/2]).  Inputs are the projections'
// natural layout [B, T, H, D] (no transpose copy); the rotated queries are
// written [B, Hq, T, D] in bf16 (prefill) and/or fp32 (decode).  Trimming
// the cache is a length change on the host (no kernel).  The cache is either
// contiguous [B, Hkv, capacity, D] or a paged pool [num_pages, Hkv,
// page_size, D] addressed through a block table (cache_row); in a paged pool
// a token whose page id is outside [0, num_pages) is not written.
#include "common.cuh"

namespace santa {

__device__ __forceinline__ __nv_bfloat16 rope1(__nv_bfloat16 x, __nv_bfloat16 xr, __nv_bfloat16 c,
                                               __nv_bfloat16 s) {
    const __nv_bfloat16 a = __float2bfloat16_rn(__bfloat162float(x) * __bfloat162float(c));
    const __nv_bfloat16 b = __float2bfloat16_rn(__bfloat162float(xr) * __bfloat162float(s));
    return __float2bfloat16_rn(__bfloat162float(a) + __bfloat162float(b));
}

// one thread per (b, t, head, d) with head over the Hq query heads followed
// by the Hkv key/value heads
__global__ void rope_append_kernel(int B, int T, int Hq, int Hkv, int D,
                                   const __nv_bfloat16 *q, const __nv_bfloat16 *k,
                                   const __nv_bfloat16 *v, const __nv_bfloat16 *cos,
                                   const __nv_bfloat16 *sin, __nv_bfloat16 *kc, __nv_bfloat16 *vc,
                                   SantaGeometry geo, int start, __nv_bfloat16 *q_bf16,
                                   float *q_f32) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int H = Hq + Hkv;
    const int64_t total = (int64_t)B * T * H * D;
    if (i >= total) return;
    const int d = (int)(i % D);
    const int hh = (int)((i / D) % H);
    const int t = (int)((i / ((int64_t)D * H)) % T);
    const int b = (int)(i / ((int64_t)D * H * T));
    const int half = D / 2;
    const int dr = d < half ? d + half : d - half;
    const __nv_bfloat16 c = cos[((int64_t)b * T + t) * D + d];
    const __nv_bfloat16 s = sin[((int64_t)b * T + t) * D + d];
    if (hh < Hq) {
        const __nv_bfloat16 *row = q + (((int64_t)b * T + t) * Hq + hh) * D;
        const __nv_bfloat16 xr = d < half ? __hneg(row[dr]) : row[dr];
        const __nv_bfloat16 o = rope1(row[d], xr, c, s);
        const int64_t oi = (((int64_t)b * Hq + hh) * T + t) * D + d;
        if (q_bf16) q_bf16[oi] = o;
        if (q_f32) q_f32[oi] = __bfloat162float(o);
    } else {
        const int kv = hh - Hq;
        const __nv_bfloat16 *row = k + (((int64_t)b * T + t) * Hkv + kv) * D;
        const __nv_bfloat16 xr = d < half ? __hneg(row[dr]) : row[dr];
        const int p = start + t;
        if (geo.block_table) {
            const int page = geo.block_table[(int64_t)b * geo.max_pages + p / geo.page_size];
            if ((unsigned)page >= (unsigned)geo.num_pages) return;
        }
        const int64_t ci = cache_row(geo, b * Hkv + kv, p) * D + d;
        kc[ci] = rope1(row[d], xr, c, s);
        vc[ci] = v[(((int64_t)b * T + t) * Hkv + kv) * D + d];
    }
}

}  // namespace santa

using namespace santa;

static int rope_append(int32_t batch, int32_t tokens, int32_t num_query_heads,
                       int32_t num_kv_heads, int32_t head_dim, const void *q, const void *k,
                       const void *v, const void *cos, const void *sin, void *key_cache,
                       void *value_cache, const SantaGeometry &geo, int32_t start,
                       void *q_rot_bf16, float *q_rot_f32, cudaStream_t stream) {
    if (batch <= 0 || tokens <= 0 || num_query_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
        (head_dim & 1))
        return SANTA_ERR_INVALID_ARGUMENT;
    if (!q || !k || !v || !cos || !sin || !key_cache || !value_cache)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (start < 0 || (int64_t)start + tokens > geo.capacity) return SANTA_ERR_INVALID_ARGUMENT;
    const int64_t total = (int64_t)batch * tokens * (num_query_heads + num_kv_heads) * head_dim;
    rope_append_kernel<<<(unsigned)ceil_div64(total, 256), 256, 0, stream>>>(
        batch, tokens, num_query_heads, num_kv_heads, head_dim, (const __nv_bfloat16 *)q,
        (const __nv_bfloat16 *)k, (const __nv_bfloat16 *)v, (const __nv_bfloat16 *)cos,
        (const __nv_bfloat16 *)sin, (__nv_bfloat16 *)key_cache, (__nv_bfloat16 *)value_cache,
        geo, start, (__nv_bfloat16 *)q_rot_bf16, q_rot_f32);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

extern "C" int santa_rope_append(int32_t batch, int32_t tokens, int32_t num_query_heads,
                                 int32_t num_kv_heads, int32_t head_dim, const void *q,
                                 const void *k, const void *v, const void *cos, const void *sin,
                                 void *key_cache, void *value_cache, int32_t capacity,
                                 int32_t start, void *q_rot_bf16, float *q_rot_f32,
                                 cudaStream_t stream) {
    SantaGeometry geo = {};
    geo.batch = batch;
    geo.num_kv_heads = num_kv_heads;
    geo.capacity = capacity;
    return rope_append(batch, tokens, num_query_heads, num_kv_heads, head_dim, q, k, v, cos, sin,
                       key_cache, value_cache, geo, start, q_rot_bf16, q_rot_f32, stream);
}

extern "C" int santa_rope_append_paged(int32_t batch, int32_t tokens, int32_t num_query_heads,
                                       int32_t num_kv_heads, int32_t head_dim, const void *q,
                                       const void *k, const void *v, const void *cos,
                                       const void *sin, void *key_pool, void *value_pool,
                                       const int32_t *block_table, int32_t page_size,
                                       int32_t max_pages, int32_t num_pages, int32_t start,
                                       void *q_rot_bf16, float *q_rot_f32, cudaStream_t stream) {
    if (!block_table || page_size <= 0 || (page_size & (page_size - 1)) || max_pages <= 0 ||
        num_pages <= 0 || (int64_t)max_pages * page_size > INT32_MAX)
        return SANTA_ERR_INVALID_ARGUMENT;
    SantaGeometry geo = {};
    geo.batch = batch;
    geo.num_kv_heads = num_kv_heads;
    geo.capacity = max_pages * page_size;
    geo.block_table = block_table;
    geo.page_size = page_size;
    geo.max_pages = max_pages;
    geo.num_pages = num_pages;
    return rope_append(batch, tokens, num_query_heads, num_kv_heads, head_dim, q, k, v, cos, sin,
                       key_pool, value_pool, geo, start, q_rot_bf16, q_rot_f32, stream);
}
