// Library-wide C ABI helpers: status strings, last CUDA error, version.
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
