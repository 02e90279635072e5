// SANTA++ decode over sequence shards: the LSE merge of the per-shard
// partials gathered by exchange 2.
//
// Shard r's partial of one (sequence, query head) holds m_r (log2 units),
// l_r = sum_j 2^(lw_j - m_r) and o_r = sum_j 2^(lw_j - m_r) v_j over the rows
// the shard attended (its selected clusters, its samples with their
// stratified weights, the recent window on the shard that holds it).  The
// estimator over all shards is
//   out = sum_r 2^(m_r - M) o_r / sum_r 2^(m_r - M) l_r,   M = max_r m_r,
// the same self-normalised combine as santapp.py:472-506 over the union of
// the shards' rows.  The ESS sums (santapp.py:481-485) merge the same way.
// (The peer-memory exchange merges inside the attention kernel instead.)
//
// Also the exchange buffer's host side: allocation, IPC handles, mapping.
#include "decode_common.cuh"

#include <math.h>
#include <string.h>

namespace santa {

template <int D>
__global__ void __launch_bounds__(D) merge_shards_kernel(int rows, int num_shards,
                                                         const float *partials, float *out,
                                                         float *lse, float *ess) {
    constexpr int PS = D + 8;
    const int row = blockIdx.x, d = threadIdx.x;
    auto part = [&](int r, int j) { return partials[((int64_t)r * rows + row) * PS + j]; };
    const ShardMerged s = shard_merge_header(num_shards, part);
    float acc = 0.f;
    for (int r = 0; r < num_shards; ++r)
        if (part(r, 1) > 0.f) acc = fmaf(part(r, 8 + d), exp2f(part(r, 0) - s.M), acc);
    out[(int64_t)row * D + d] = acc * shard_out_scale(s);
    if (d == 0) {
        if (lse) lse[row] = shard_lse(s);
        if (ess) ess[row] = shard_ess(s);
    }
}

int launch_merge_shards(int rows, int head_dim, int num_shards, const float *partials,
                        float *out, float *lse, float *ess, cudaStream_t stream) {
    if (head_dim == 64)
        merge_shards_kernel<64><<<rows, 64, 0, stream>>>(rows, num_shards, partials, out, lse, ess);
    else
        merge_shards_kernel<128>
            <<<rows, 128, 0, stream>>>(rows, num_shards, partials, out, lse, ess);
    SANTA_LAUNCH_CHECK();
    return SANTA_OK;
}

}  // namespace santa

using namespace santa;

extern "C" int santa_p2p_buffer_bytes(int32_t num_shards, int32_t rows, int32_t keys_per_row,
                                      int32_t head_dim, size_t *bytes) {
    if (!bytes || num_shards < 1 || num_shards > SANTA_MAX_SHARDS || rows <= 0 ||
        keys_per_row <= 0 || head_dim <= 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    *bytes = p2p_buffer_bytes(num_shards, rows, keys_per_row, head_dim + 8);
    return SANTA_OK;
}

extern "C" int santa_p2p_alloc(size_t bytes, void **buffer) {
    if (!buffer || bytes == 0) return SANTA_ERR_INVALID_ARGUMENT;
    SANTA_CUDA_CHECK(cudaMalloc(buffer, bytes));
    SANTA_CUDA_CHECK(cudaMemset(*buffer, 0, bytes));
    return SANTA_OK;
}

extern "C" int santa_p2p_free(void *buffer) {
    if (buffer) SANTA_CUDA_CHECK(cudaFree(buffer));
    return SANTA_OK;
}

extern "C" int santa_p2p_ipc_handle(void *buffer, void *handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == SANTA_IPC_HANDLE_BYTES, "IPC handle size");
    if (!buffer || !handle) return SANTA_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    SANTA_CUDA_CHECK(cudaIpcGetMemHandle(&h, buffer));
    memcpy(handle, &h, sizeof(h));
    return SANTA_OK;
}

extern "C" int santa_p2p_ipc_open(const void *handle, void **mapped) {
    if (!handle || !mapped) return SANTA_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    SANTA_CUDA_CHECK(cudaIpcOpenMemHandle(mapped, h, cudaIpcMemLazyEnablePeerAccess));
    return SANTA_OK;
}

extern "C" int santa_p2p_ipc_close(void *mapped) {
    if (mapped) SANTA_CUDA_CHECK(cudaIpcCloseMemHandle(mapped));
    return SANTA_OK;
}

extern "C" int santa_p2p_peek(const void *address, uint64_t *value) {
    if (!address || !value) return SANTA_ERR_INVALID_ARGUMENT;
    SANTA_CUDA_CHECK(cudaMemcpy(value, address, 8, cudaMemcpyDeviceToHost));
    return SANTA_OK;
}

extern "C" int santa_p2p_poke(void *address, uint64_t value) {
    if (!address) return SANTA_ERR_INVALID_ARGUMENT;
    SANTA_CUDA_CHECK(cudaMemcpy(address, &value, 8, cudaMemcpyHostToDevice));
    return SANTA_OK;
}
