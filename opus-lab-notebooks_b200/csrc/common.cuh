// Shared device helpers for the SANTA++ sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "santa_b200.h"

#define SANTA_MAX_GROUP 8      // query heads per KV head handled by one CTA
#define SANTA_MAX_CLUSTERS 1024
#define SANTA_MAX_SAMPLES 1024

namespace santa {

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

// Philox4x32-10 (Salmon et al., SC'11): counter (c0..c3), key (k0,k1).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c.x;
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x);
        const uint32_t lo1 = 0xCD9E8D57u * c.z;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

__device__ __forceinline__ uint32_t uint4_word(const uint4& v, int j) {
    return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// Total order on floats as unsigned keys (larger float -> larger key);
// -0.0 is folded onto +0.0 first so equal values get equal keys.
__device__ __forceinline__ uint32_t float_order_key(float f) {
    f = __fadd_rn(f, 0.0f);
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Row of token p of (batch, KV head) bh in the key / value cache, in rows of
// head_dim elements from the cache base.  Contiguous caches [B, Hkv, cap, D]:
// bh * capacity + p.  Paged pools [num_pages, Hkv, page_size, D] (page_size a
// power of two, checked on the host): the page comes from the sequence's
// block-table row; a page id outside [0, num_pages) reads page 0 so that a
// corrupt table cannot address memory outside the pool.
__device__ __forceinline__ int64_t cache_row(const SantaGeometry &g, int bh, int p) {
    if (!g.block_table) return (int64_t)bh * g.capacity + p;
    const int b = bh / g.num_kv_heads, kv = bh - b * g.num_kv_heads;
    const int sh = __ffs(g.page_size) - 1;
    int page = __ldg(g.block_table + (int64_t)b * g.max_pages + (p >> sh));
    page = (unsigned)page < (unsigned)g.num_pages ? page : 0;
    return (((int64_t)page * g.num_kv_heads + kv) << sh) + (p & (g.page_size - 1));
}

// Rows in the cache a geometry addresses (the bound of cache_row).
__host__ __device__ inline int64_t cache_rows(const SantaGeometry &g) {
    return g.block_table ? (int64_t)g.num_pages * g.num_kv_heads * g.page_size
                         : (int64_t)g.batch * g.num_kv_heads * g.capacity;
}

}  // namespace santa

// Status helpers for the C ABI.
#define SANTA_CUDA_CHECK(expr)                                  \
    do {                                                        \
        cudaError_t _e = (expr);                                \
        if (_e != cudaSuccess) {                                \
            santa_set_cuda_error(_e);                           \
            return SANTA_ERR_CUDA;                              \
        }                                                       \
    } while (0)

#define SANTA_LAUNCH_CHECK()                                    \
    do {                                                        \
        cudaError_t _e = cudaGetLastError();                    \
        if (_e != cudaSuccess) {                                \
            santa_set_cuda_error(_e);                           \
            return SANTA_ERR_CUDA;                              \
        }                                                       \
    } while (0)

void santa_set_cuda_error(cudaError_t e);

namespace santa {
// Per-device launch set-up, safe from several host threads and for one
// process that drives several GPUs (santa_lib.cu).
// Raises fn's dynamic shared memory limit on the current device to at least
// `bytes` (cudaFuncSetAttribute is a per-device setting).
int ensure_dyn_smem(const void *fn, size_t bytes);
// Multiprocessor count of the current device.
int num_sms();
// A device attribute of the current device (0 if it cannot be read).
int device_attr(cudaDeviceAttr attr);
}  // namespace santa
