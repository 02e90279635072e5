// C ABI of the SANTA++ sparse decode (include/santa_b200.h).
//
// santa_decode replaces SantaPlusEngine._approximate_attention
// (santapp_ruler/attention/santapp.py:365-506) for every (batch, query head)
// of a decode step; santa_decode_plan / santa_decode_execute are its two
// stream-ordered halves, santa_decode_select reads the selection out.
#include "decode_common.cuh"

#include <stdlib.h>
#include <string.h>

using namespace santa;

extern "C" int santa_check_geometry(const SantaGeometry *geo);

static int pick_splits(const SantaGeometry *geo, const SantaDecodeParams *p) {
    if (p->num_splits > 0) return p->num_splits;
    const int BH = geo->batch * geo->num_kv_heads;
    int s = (2 * num_sms()) / BH;
    if (s < 1) s = 1;
    if (s > 64) s = 64;
    return s;
}

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
    {
        // the attention kernel balances rows on a 32-bit cost scale
        // (at most 3 per row: union + recent + sampled rows of every segment)
        const int64_t rows = (int64_t)geo->n_total + (int64_t)geo->group * p->samples;
        // (kCostSample per row at most, plus the start charge per segment)
        if ((int64_t)geo->batch * geo->num_kv_heads * (rows * kCostSample + kCostSegment) >=
            ((int64_t)1 << 31))
            return SANTA_ERR_UNSUPPORTED;
    }
    if (!(p->scale > 0.f)) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->num_splits < 0 || p->num_splits > 256) return SANTA_ERR_INVALID_ARGUMENT;
    return SANTA_OK;
}

static size_t workspace_bytes(const SantaGeometry *geo, const SantaDecodeParams *p,
                              int max_groups, int nsplit) {
    const int BH = geo->batch * geo->num_kv_heads;
    return decode_ws_layout(BH, max_groups, geo->group, p->samples,
                            attend_partial_slots(geo, nsplit), geo->head_dim, geo->sample_end,
                            nullptr, nullptr);
}

extern "C" int santa_decode_workspace_bytes(const SantaGeometry *geo, const SantaDecodeParams *p,
                                            int32_t max_groups, size_t *bytes) {
    int st = check_decode(geo, p, max_groups);
    if (st) return st;
    if (!bytes) return SANTA_ERR_INVALID_ARGUMENT;
    *bytes = workspace_bytes(geo, p, max_groups, pick_splits(geo, p));
    return SANTA_OK;
}

static int prepare_decode(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                          const void *key_cache, const void *value_cache,
                          const SantaSummary *summary, const int32_t *sample_a,
                          const int32_t *sample_b, bool need_draws, void *workspace,
                          size_t ws_bytes, DecodeArgs *a) {
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
    if (needs_summary && ((uintptr_t)summary->centroids & 15))  // 16-byte centroid copies
        return SANTA_ERR_UNSUPPORTED;
    if ((p->mode == SANTA_MODE_UNIFORM || p->mode == SANTA_MODE_SANTA) && !summary->positions)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (need_draws && p->sample_source == SANTA_SAMPLES_INJECTED && p->mode != SANTA_MODE_TOPK) {
        if (!sample_a) return SANTA_ERR_INVALID_ARGUMENT;
        if (p->mode == SANTA_MODE_GUIDED && !sample_b) return SANTA_ERR_INVALID_ARGUMENT;
    }
    const int BH = geo->batch * geo->num_kv_heads;
    const int nsplit = pick_splits(geo, p);
    if (!workspace || ws_bytes < workspace_bytes(geo, p, summary->max_groups, nsplit))
        return SANTA_ERR_WORKSPACE;
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
    a->cluster_base = 0;
    a->num_shards = 1;
    a->shard_index = 0;
    a->cand_out = nullptr;
    a->shard_cands = nullptr;
    a->part_out = nullptr;
    memset(&a->p2p, 0, sizeof(a->p2p));
    a->tma = 0;  // set by the attention launcher
    decode_ws_layout(BH, summary->max_groups, geo->group, p->samples,
                     attend_partial_slots(geo, nsplit), geo->head_dim, geo->sample_end,
                     (char *)workspace, &a->ws);
    return SANTA_OK;
}

extern "C" int santa_decode_plan(const SantaGeometry *geo, const SantaDecodeParams *p,
                                 const float *q, const void *key_cache, const void *value_cache,
                                 const SantaSummary *summary, const int32_t *sample_a,
                                 const int32_t *sample_b, int32_t *n_exact, void *workspace,
                                 size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b, true,
                            workspace, workspace_bytes, &a);
    if (st) return st;
    a.n_exact = n_exact;
    return launch_plan(a, stream);
}

extern "C" int santa_decode_bad_draws(const SantaGeometry *geo, const void *workspace,
                                      size_t workspace_bytes, int32_t *segments,
                                      cudaStream_t stream) {
    if (!geo || !workspace || !segments) return SANTA_ERR_INVALID_ARGUMENT;
    const int64_t BH = (int64_t)geo->batch * geo->num_kv_heads;
    if (geo->batch <= 0 || geo->num_kv_heads <= 0) return SANTA_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < (size_t)BH * 4) return SANTA_ERR_WORKSPACE;
    int32_t *h = (int32_t *)malloc((size_t)BH * 4);
    if (!h) return SANTA_ERR_INVALID_ARGUMENT;
    cudaError_t e = cudaMemcpyAsync(h, workspace, (size_t)BH * 4, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        free(h);
        santa_set_cuda_error(e);
        return SANTA_ERR_CUDA;
    }
    int32_t n = 0;
    for (int64_t i = 0; i < BH; ++i) n += h[i] != 0 ? 1 : 0;
    free(h);
    *segments = n;
    return SANTA_OK;
}

extern "C" int santa_decode_execute(const SantaGeometry *geo, const SantaDecodeParams *p,
                                    const float *q, const void *key_cache,
                                    const void *value_cache, const SantaSummary *summary,
                                    float *out, float *lse, float *ess, void *workspace,
                                    size_t workspace_bytes, cudaStream_t stream) {
    if (!out) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, nullptr, nullptr, false,
                            workspace, workspace_bytes, &a);
    if (st) return st;
    a.out = out;
    a.lse = lse;
    a.ess = ess;
    return launch_execute(a, stream);
}

extern "C" int santa_decode(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                            const void *key_cache, const void *value_cache,
                            const SantaSummary *summary, const int32_t *sample_a,
                            const int32_t *sample_b, float *out, float *lse, int32_t *n_exact,
                            float *ess, void *workspace, size_t workspace_bytes,
                            cudaStream_t stream) {
    if (!out) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b, true,
                            workspace, workspace_bytes, &a);
    if (st) return st;
    a.out = out;
    a.lse = lse;
    a.n_exact = n_exact;
    a.ess = ess;
    st = launch_plan(a, stream);
    if (st) return st;
    return launch_execute(a, stream);
}

extern "C" int santa_decode_select(const SantaGeometry *geo, const SantaDecodeParams *p,
                                   const float *q, const void *key_cache, const void *value_cache,
                                   const SantaSummary *summary, const int32_t *sample_a,
                                   const int32_t *sample_b, uint8_t *selected,
                                   int32_t *sample_rows, int32_t *n_exact, void *workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, sample_b, true,
                            workspace, workspace_bytes, &a);
    if (st) return st;
    a.n_exact = n_exact;
    st = launch_plan(a, stream);
    if (st) return st;
    return launch_expand(a, selected, sample_rows, stream);
}

// ---------------------------------------------------------------------------
// sequence shards (HYBRID, bf16 caches)
// ---------------------------------------------------------------------------
static int bind_p2p(const SantaGeometry *geo, const SantaDecodeParams *p,
                    const SantaShard *shard, DecodeArgs *a) {
    memset(&a->p2p, 0, sizeof(a->p2p));
    const SantaP2P *c = shard->p2p;
    if (!c) return SANTA_OK;
    if (!c->peer_buffers || !c->local_buffer || !c->error_flag || c->epoch == 0 ||
        c->wait_limit_us < 0)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (c->rows != geo->batch * geo->num_kv_heads * geo->group ||
        c->keys_per_row != p->topk_clusters || c->partial_floats != geo->head_dim + 8)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)c->local_buffer & 255) != 0) return SANTA_ERR_INVALID_ARGUMENT;
    a->p2p.peers = c->peer_buffers;
    a->p2p.local = (unsigned char *)c->local_buffer;
    a->p2p.epoch = c->epoch;
    a->p2p.wait_ns = (unsigned long long)(c->wait_limit_us > 0 ? c->wait_limit_us : 2000000) * 1000ull;
    a->p2p.err = c->error_flag;
    a->p2p.rank = shard->shard_index;
    a->p2p.n = shard->num_shards;
    a->p2p.rows = c->rows;
    a->p2p.kk = c->keys_per_row;
    a->p2p.pf = c->partial_floats;
    return SANTA_OK;
}

static int check_shard(const SantaGeometry *geo, const SantaDecodeParams *p,
                       const SantaShard *shard, bool need_candidates) {
    if (!geo || !p || !shard) return SANTA_ERR_INVALID_ARGUMENT;
    // a shard owns a contiguous slice of every sequence: paged shards are not built
    if (p->mode != SANTA_MODE_HYBRID || geo->kv_dtype != SANTA_DTYPE_BF16 || geo->block_table)
        return SANTA_ERR_UNSUPPORTED;
    if (shard->num_shards < 1 || shard->num_shards > SANTA_MAX_SHARDS) return SANTA_ERR_INVALID_ARGUMENT;
    if (shard->shard_index < 0 || shard->shard_index >= shard->num_shards)
        return SANTA_ERR_INVALID_ARGUMENT;
    if (shard->cluster_base < 0) return SANTA_ERR_INVALID_ARGUMENT;
    if (p->topk_clusters < 1 || (int64_t)p->topk_clusters * shard->num_shards > SANTA_SHARD_MAX_KEYS)
        return SANTA_ERR_UNSUPPORTED;
    if (need_candidates && !shard->candidates && !shard->p2p) return SANTA_ERR_INVALID_ARGUMENT;
    return SANTA_OK;
}

static int prepare_shard(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                         const void *key_cache, const void *value_cache,
                         const SantaSummary *summary, const SantaShard *shard,
                         const int32_t *sample_a, bool need_candidates, bool need_draws,
                         void *workspace, size_t ws_bytes, DecodeArgs *a) {
    int st = check_shard(geo, p, shard, need_candidates);
    if (st) return st;
    st = prepare_decode(geo, p, q, key_cache, value_cache, summary, sample_a, nullptr, need_draws,
                        workspace, ws_bytes, a);
    if (st) return st;
    if ((int64_t)shard->cluster_base + summary->max_groups >= 0xFFFFFFFFll)
        return SANTA_ERR_INVALID_ARGUMENT;
    a->cluster_base = shard->cluster_base;
    a->num_shards = shard->num_shards;
    a->shard_index = shard->shard_index;
    a->shard_cands = need_candidates ? shard->candidates : nullptr;
    if (need_candidates && shard->p2p) {
        // the selection launch runs the candidates pass and the key exchange
        // itself (peer memory, low-latency words whose keys carry 24-bit ids)
        st = bind_p2p(geo, p, shard, a);
        if (st) return st;
        if ((int64_t)shard->cluster_base + summary->max_groups >= 0xFFFFFFll)
            return SANTA_ERR_UNSUPPORTED;
        if (shard->p2p->partial_floats != geo->head_dim + 8) return SANTA_ERR_INVALID_ARGUMENT;
        a->shard_cands = nullptr;
        if (!select_group_supported(*a)) return SANTA_ERR_UNSUPPORTED;
    }
    return SANTA_OK;
}

extern "C" int santa_shard_candidates(const SantaGeometry *geo, const SantaDecodeParams *p,
                                      const float *q, const void *key_cache,
                                      const void *value_cache, const SantaSummary *summary,
                                      const SantaShard *shard, uint64_t *keys, void *workspace,
                                      size_t workspace_bytes, cudaStream_t stream) {
    if (!keys) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    int st = prepare_shard(geo, p, q, key_cache, value_cache, summary, shard, nullptr, false,
                           false, workspace, workspace_bytes, &a);
    if (st) return st;
    a.cand_out = keys;
    return launch_plan(a, stream);
}

extern "C" int santa_shard_plan(const SantaGeometry *geo, const SantaDecodeParams *p,
                                const float *q, const void *key_cache, const void *value_cache,
                                const SantaSummary *summary, const SantaShard *shard,
                                const int32_t *sample_a, int32_t *n_exact, void *workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_shard(geo, p, q, key_cache, value_cache, summary, shard, sample_a, true, true,
                           workspace, workspace_bytes, &a);
    if (st) return st;
    a.n_exact = n_exact;
    return launch_plan(a, stream);
}

extern "C" int santa_shard_execute(const SantaGeometry *geo, const SantaDecodeParams *p,
                                   const float *q, const void *key_cache,
                                   const void *value_cache, const SantaSummary *summary,
                                   const SantaShard *shard, float *partial, void *workspace,
                                   size_t workspace_bytes, cudaStream_t stream) {
    if (!partial || !shard) return SANTA_ERR_INVALID_ARGUMENT;
    int st = check_shard(geo, p, shard, false);
    if (st) return st;
    DecodeArgs a;
    if (shard->p2p) return SANTA_ERR_INVALID_ARGUMENT;  // santa_shard_attend merges in place
    st = prepare_decode(geo, p, q, key_cache, value_cache, summary, nullptr, nullptr, false,
                        workspace, workspace_bytes, &a);
    if (st) return st;
    a.part_out = partial;
    return launch_execute(a, stream);
}

extern "C" int santa_shard_attend(const SantaGeometry *geo, const SantaDecodeParams *p,
                                  const float *q, const void *key_cache, const void *value_cache,
                                  const SantaSummary *summary, const SantaShard *shard, float *out,
                                  float *lse, float *ess, void *workspace, size_t workspace_bytes,
                                  cudaStream_t stream) {
    if (!out || !shard || !shard->p2p) return SANTA_ERR_INVALID_ARGUMENT;
    int st = check_shard(geo, p, shard, false);
    if (st) return st;
    // the merged rows are written with one vector store per lane
    if (((uintptr_t)out & (geo->head_dim == 128 ? 15 : 7)) != 0) return SANTA_ERR_INVALID_ARGUMENT;
    DecodeArgs a;
    st = prepare_decode(geo, p, q, key_cache, value_cache, summary, nullptr, nullptr, false,
                        workspace, workspace_bytes, &a);
    if (st) return st;
    st = bind_p2p(geo, p, shard, &a);
    if (st) return st;
    a.out = out;
    a.lse = lse;
    a.ess = ess;
    a.part_out = (float *)(a.p2p.local + p2p_stage_offset(a.p2p.n, a.p2p.rows, a.p2p.kk, a.p2p.pf));
    return launch_execute(a, stream);
}

extern "C" int santa_shard_select(const SantaGeometry *geo, const SantaDecodeParams *p,
                                  const float *q, const void *key_cache, const void *value_cache,
                                  const SantaSummary *summary, const SantaShard *shard,
                                  const int32_t *sample_a, uint8_t *selected,
                                  int32_t *sample_rows, int32_t *n_exact, void *workspace,
                                  size_t workspace_bytes, cudaStream_t stream) {
    DecodeArgs a;
    int st = prepare_shard(geo, p, q, key_cache, value_cache, summary, shard, sample_a, true, true,
                           workspace, workspace_bytes, &a);
    if (st) return st;
    a.n_exact = n_exact;
    st = launch_plan(a, stream);
    if (st) return st;
    return launch_expand(a, selected, sample_rows, stream);
}

extern "C" int santa_merge_shards(int32_t rows, int32_t head_dim, int32_t num_shards,
                                  const float *partials, float *out, float *lse, float *ess,
                                  cudaStream_t stream) {
    if (rows <= 0 || num_shards < 1 || num_shards > SANTA_MAX_SHARDS) return SANTA_ERR_INVALID_ARGUMENT;
    if (head_dim != 64 && head_dim != 128) return SANTA_ERR_UNSUPPORTED;
    if (!partials || !out) return SANTA_ERR_INVALID_ARGUMENT;
    return launch_merge_shards(rows, head_dim, num_shards, partials, out, lse, ess, stream);
}
