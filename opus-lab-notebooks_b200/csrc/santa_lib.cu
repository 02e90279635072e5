// Library-wide C ABI helpers: status strings, last CUDA error, version.
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

static thread_local int g_last_cuda_error = 0;

void santa_set_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }

extern "C" const char *santa_status_string(int status) {
    switch (status) {
        case SANTA_OK: return "ok";
        case SANTA_ERR_INVALID_ARGUMENT: return "invalid argument (shape, stride, index or budget)";
        case SANTA_ERR_UNSUPPORTED: return "unsupported configuration (dtype or head_dim)";
        case SANTA_ERR_CUDA: return "CUDA runtime error";
        case SANTA_ERR_WORKSPACE: return "workspace missing or too small";
        default: return "unknown status";
    }
}

extern "C" int santa_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" const char *santa_version(void) { return "santa_b200 0.1 (sm_100a)"; }

namespace santa {
namespace {
std::mutex g_launch_mutex;
// (device, kernel) -> dynamic shared memory limit already set
std::map<std::pair<int, const void *>, size_t> g_smem_set;
// (device, attribute) -> value
std::map<std::pair<int, int>, int> g_dev_attr;

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return dev;
}
}  // namespace

int ensure_dyn_smem(const void *fn, size_t bytes) {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_launch_mutex);
    size_t &done = g_smem_set[std::make_pair(dev, fn)];
    if (done >= bytes) return SANTA_OK;
    SANTA_CUDA_CHECK(
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    done = bytes;
    return SANTA_OK;
}

int device_attr(cudaDeviceAttr attr) {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_launch_mutex);
    auto key = std::make_pair(dev, (int)attr);
    auto it = g_dev_attr.find(key);
    if (it != g_dev_attr.end()) return it->second;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, attr, dev) != cudaSuccess) {
        cudaGetLastError();
        v = 0;
    }
    g_dev_attr[key] = v;
    return v;
}

int num_sms() {
    const int n = device_attr(cudaDevAttrMultiProcessorCount);
    return n > 0 ? n : 148;
}
}  // namespace santa
