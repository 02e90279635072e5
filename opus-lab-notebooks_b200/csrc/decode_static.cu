// santa_decode for callers that cannot allocate device memory.
//
// Some callers of this library are not allowed to call cudaMalloc: a serving
// stack whose memory manager has already reserved all device memory for its
// KV-cache pool, a host application that loads this library as a plugin and
// forbids device allocations after start-up, or a decode loop that must not
// pay for cudaMalloc's implicit device synchronisation.  For them this file
// provides santa_decode_static_scratch: the same decode step as santa_decode,
// with its scratch workspace in a fixed array that lives in the library's own
// device memory instead of a buffer the caller allocates.
#include <mutex>

#include "common.cuh"

// The scratch every call on a device shares.  Each GPU that loads the
// library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_decode_scratch[SANTA_DECODE_STATIC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void *g_scratch_ptr[kMaxDevices] = {};  // device address of g_decode_scratch per device
}  // namespace

// Device address of the scratch array on the current device.  Host code must
// not use the name g_decode_scratch as a pointer: on the host it is only a
// stand-in, so its address is looked up once per device, with that device
// current, and cached for the life of the process.  The address belongs to
// the device's primary context; after cudaDeviceReset destroys that context
// the cached address is stale, so a process that resets a device must not
// call this entry point on it again (the header says so).
static int scratch_address(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        santa_set_cuda_error(e);
        return SANTA_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return SANTA_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess || !p) {
            santa_set_cuda_error(e);
            return SANTA_ERR_CUDA;
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return SANTA_OK;
}

extern "C" int santa_decode_static_scratch(const SantaGeometry *geo, const SantaDecodeParams *p,
                                           const float *q, const void *key_cache,
                                           const void *value_cache, const SantaSummary *summary,
                                           const int32_t *sample_a, const int32_t *sample_b,
                                           float *out, float *lse, int32_t *n_exact, float *ess,
                                           cudaStream_t stream) {
    if (!summary) return SANTA_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    int st = santa_decode_workspace_bytes(geo, p, summary->max_groups, &need);
    if (st) return st;
    // geometries whose workspace does not fit the fixed array are refused
    if (need > (size_t)SANTA_DECODE_STATIC_SCRATCH_BYTES) return SANTA_ERR_WORKSPACE;
    void *scratch = nullptr;
    st = scratch_address(&scratch);
    if (st) return st;
    // santa_decode clears the parts of the workspace that must start at zero
    return santa_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b, out, lse,
                        n_exact, ess, scratch, (size_t)SANTA_DECODE_STATIC_SCRATCH_BYTES, stream);
}
