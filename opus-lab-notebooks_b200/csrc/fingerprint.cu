// Key fingerprints for clustering (santapp_ruler/attention/santapp.py:598-690).
//
// For one (layer, KV head) the reference builds, over the clustered prefix's
// keys K [N, D] (the cache upcast to fp32) and the rotated queries of the
// group's query heads at P probe positions,
//   F[:, h*P + p] = K @ q_h[probe_p] / sqrt(D)              (:672-683)
//   F = (F - mean_rows(F)) / (std_rows(F, population) + 1e-6) (:684-691)
// and clusters the rows of F.  Defined arithmetic (the oracle's
// or_fingerprints / or_zscore restate it):
//   dot     sequential fmaf chain over D
//   F       fl32(dot / divisor), divisor = fl32(sqrt(D)), IEEE division
//   mean    exact signed Q64.64 sum of the column, fl32(fl64(sum) / N)
//   var     exact Q64.64 sum of fl32(fl32(x - mean)^2), fl32(fl64(sum) / N)
//   z       fl32(fl32(x - mean) / fl32(sqrt_rn(var) + 1e-6))
// so the fingerprints, and the k-means labels computed from them, do not
// depend on the reduction order.
//
// Kernels: fp_dots_kernel (32 rows x 64 columns per CTA, 2 x 4 fmaf chains a
// thread, operands staged in shared memory), fp_colsum_kernel (exact column
// sums with 128-bit atomics), fp_colsq_kernel (exact sums of squared
// deviations), fp_normalize_kernel.
#include "common.cuh"

#include <math.h>

namespace santa {

typedef unsigned __int128 u128f;

__device__ __forceinline__ u128f fp_fx_mag(float v) {  // |v| truncated to Q64.64
    const uint32_t bits = __float_as_uint(v) & 0x7fffffffu;
    const uint32_t ex = bits >> 23;
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
        return ((u128f)mant) << sh;
    }
    if (sh <= -32) return 0;
    return (u128f)(mant >> (-sh));
}
// two's complement Q64.64 of v (sums wrap modulo 2^128 and stay exact)
__device__ __forceinline__ u128f fp_fx_signed(float v) {
    const u128f m = fp_fx_mag(v);
    return (__float_as_uint(v) & 0x80000000u) ? (u128f)0 - m : m;
}
__device__ __forceinline__ double fp_fx_to_double(u128f s, bool is_signed) {
    bool neg = false;
    if (is_signed && (s >> 127)) {
        s = (u128f)0 - s;
        neg = true;
    }
    const unsigned long long hi = (unsigned long long)(s >> 64), lo = (unsigned long long)s;
    const double d = __dadd_rn(__ull2double_rn(hi), __dmul_rn(__ull2double_rn(lo), 0x1p-64));
    return neg ? -d : d;
}
__device__ __forceinline__ void fp_atomic_add_u128(unsigned long long *p, u128f v) {
    const unsigned long long lo = (unsigned long long)v;
    unsigned long long hi = (unsigned long long)(v >> 64);
    if (lo) {
        const unsigned long long old = atomicAdd(p, lo);
        if (old + lo < old) hi += 1ull;
    }
    if (hi) atomicAdd(p + 1, hi);
}

template <typename T>
__device__ __forceinline__ float fp_ld(const T *p);
template <> __device__ __forceinline__ float fp_ld<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float fp_ld<__nv_bfloat16>(const __nv_bfloat16 *p) {
    return __bfloat162float(*p);
}

constexpr int kFpRows = 32, kFpCols = 64, kFpThreads = 256;

// F[n][c] for c = h*P + p: keys rows x probe-query columns
template <typename T>
__global__ void __launch_bounds__(kFpThreads) fp_dots_kernel(
    const T *keys, int64_t n, int d, const float *q, int64_t q_head_stride, int P,
    const int64_t *probes, int cols, float divisor, float *out) {
    extern __shared__ __align__(16) float fp_smem[];
    const int pitch = d + 1;
    float *ks = fp_smem;                 // [kFpRows][d+1]
    float *qs = ks + kFpRows * pitch;    // [kFpCols][d+1]
    const int tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
    const int64_t r0 = (int64_t)blockIdx.x * kFpRows;
    const int c0 = blockIdx.y * kFpCols;
    for (int i = tid; i < kFpRows * d; i += kFpThreads) {
        const int r = i / d, t = i - r * d;
        ks[r * pitch + t] = r0 + r < n ? fp_ld<T>(keys + (r0 + r) * d + t) : 0.f;
    }
    for (int i = tid; i < kFpCols * d; i += kFpThreads) {
        const int c = i / d, t = i - c * d;
        float v = 0.f;
        if (c0 + c < cols) {
            const int h = (c0 + c) / P, p = (c0 + c) - h * P;
            v = q[(int64_t)h * q_head_stride + probes[p] * d + t];
        }
        qs[c * pitch + t] = v;
    }
    __syncthreads();
    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.f;
    const float *ka = ks + rg * pitch, *kb = ks + (rg + 16) * pitch;
    for (int t = 0; t < d; ++t) {
        const float a = ka[t], b = kb[t];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const float c = qs[(cg + 16 * jj) * pitch + t];
            acc[0][jj] = fmaf(a, c, acc[0][jj]);
            acc[1][jj] = fmaf(b, c, acc[1][jj]);
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int64_t r = r0 + rg + 16 * i;
        if (r >= n) continue;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int c = c0 + cg + 16 * jj;
            if (c < cols) out[r * cols + c] = __fdiv_rn(acc[i][jj], divisor);
        }
    }
}

constexpr int kFpRowChunk = 1024;

// exact column sums (signed) or sums of squared deviations from mean[c]
template <bool SQ>
__global__ void fp_colsum_kernel(const float *f, int64_t n, int cols, const float *mean,
                                 unsigned long long *acc) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const int64_t r0 = (int64_t)blockIdx.y * kFpRowChunk;
    const int64_t r1 = min(n, r0 + kFpRowChunk);
    u128f s = 0;
    const float m = SQ ? mean[c] : 0.f;
    for (int64_t r = r0; r < r1; ++r) {
        const float x = f[r * cols + c];
        if (SQ) {
            const float dv = __fsub_rn(x, m);
            s += fp_fx_mag(__fmul_rn(dv, dv));
        } else {
            s += fp_fx_signed(x);
        }
    }
    fp_atomic_add_u128(acc + 2 * c, s);
}

__global__ void fp_mean_kernel(const unsigned long long *acc, int cols, int64_t n, float *mean) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const u128f s = ((u128f)acc[2 * c + 1] << 64) | acc[2 * c];
    mean[c] = __double2float_rn(__ddiv_rn(fp_fx_to_double(s, true), (double)n));
}

__global__ void fp_denominator_kernel(const unsigned long long *acc, int cols, int64_t n,
                                      float *den) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    const u128f s = ((u128f)acc[2 * c + 1] << 64) | acc[2 * c];
    const float var = __double2float_rn(__ddiv_rn(fp_fx_to_double(s, false), (double)n));
    den[c] = __fadd_rn(__fsqrt_rn(var), 1e-6f);
}

__global__ void fp_normalize_kernel(float *f, int64_t n, int cols, const float *mean,
                                    const float *den) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * cols) return;
    const int c = (int)(i % cols);
    f[i] = __fdiv_rn(__fsub_rn(f[i], mean[c]), den[c]);
}

}  // namespace santa

using namespace santa;

extern "C" int santa_fingerprints_workspace_bytes(int32_t cols, size_t *bytes) {
    if (!bytes || cols <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    *bytes = (size_t)cols * (16 + 16 + 4 + 4) + 256;
    return SANTA_OK;
}

extern "C" int santa_fingerprints(const void *keys, int32_t key_dtype, int64_t n, int32_t d,
                                  const float *queries, int64_t q_head_stride,
                                  int32_t group, const int64_t *probes, int32_t n_probes,
                                  float divisor, int32_t normalize, float *out, void *workspace,
                                  size_t workspace_bytes, cudaStream_t stream) {
    if (!keys || !queries || !probes || !out || n <= 0 || d <= 0 || group <= 0 || n_probes <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (key_dtype != SANTA_DTYPE_F32 && key_dtype != SANTA_DTYPE_BF16) return SANTA_ERR_UNSUPPORTED;
    if (d > 512 || !(divisor > 0.f)) return SANTA_ERR_UNSUPPORTED;
    const int cols = group * n_probes;
    size_t need = 0;
    santa_fingerprints_workspace_bytes(cols, &need);
    if (normalize && (!workspace || workspace_bytes < need)) return SANTA_ERR_WORKSPACE;
    const size_t smem = (size_t)(kFpRows + kFpCols) * (d + 1) * 4;
    dim3 grid((unsigned)ceil_div64(n, kFpRows), (unsigned)ceil_div(cols, kFpCols));
    if (key_dtype == SANTA_DTYPE_BF16) {
        if (smem > 48 * 1024)
            SANTA_CUDA_CHECK(cudaFuncSetAttribute(fp_dots_kernel<__nv_bfloat16>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)smem));
        fp_dots_kernel<__nv_bfloat16><<<grid, kFpThreads, smem, stream>>>(
            (const __nv_bfloat16 *)keys, n, d, queries, q_head_stride, n_probes, probes, cols,
            divisor, out);
    } else {
        if (smem > 48 * 1024)
            SANTA_CUDA_CHECK(cudaFuncSetAttribute(fp_dots_kernel<float>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)smem));
        fp_dots_kernel<float><<<grid, kFpThreads, smem, stream>>>(
            (const float *)keys, n, d, queries, q_head_stride, n_probes, probes, cols, divisor,
            out);
    }
    SANTA_LAUNCH_CHECK();
    if (!normalize) return SANTA_OK;
    char *w = (char *)workspace;
    unsigned long long *sum = (unsigned long long *)w;
    unsigned long long *sq = sum + 2 * (size_t)cols;
    float *mean = (float *)(sq + 2 * (size_t)cols);
    float *den = mean + cols;
    SANTA_CUDA_CHECK(cudaMemsetAsync(w, 0, (size_t)cols * 32, stream));
    dim3 cg((unsigned)ceil_div(cols, 128), (unsigned)ceil_div64(n, kFpRowChunk));
    fp_colsum_kernel<false><<<cg, 128, 0, stream>>>(out, n, cols, nullptr, sum);
    SANTA_LAUNCH_CHECK();
    fp_mean_kernel<<<ceil_div(cols, 128), 128, 0, stream>>>(sum, cols, n, mean);
    SANTA_LAUNCH_CHECK();
    fp_colsum_kernel<true><<<cg, 128, 0, stream>>>(out, n, cols, mean, sq);
    SANTA_LAUNCH_CHECK();
    fp_denominator_kernel<<<ceil_div(cols, 128), 128, 0, stream>>>(sq, cols, n, den);
    SANTA_LAUNCH_CHECK();
    fp_normalize_kernel<<<(unsigned)ceil_div64(n * cols, 256), 256, 0, stream>>>(out, n, cols,
                                                                               mean, den);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}
