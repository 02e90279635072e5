/*
 * santa_b200.h -- C ABI of the B200 (sm_100a) SANTA++ attention library.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t,
 * is stream-ordered (no host synchronisation unless stated), allocates no
 * device memory and returns SANTA_OK (0) or a negative status code.  Callers
 * own all buffers; scratch space is passed in as a workspace whose size the
 * matching *_workspace_bytes query reports.
 *
 * Reference interfaces replaced (paths inside santapp-ruler-bench/src):
 *   santa_build_summary        santapp_ruler/attention/santapp.py:508-540
 *                              (SantaPlusEngine._build_summary)
 *   santa_decode               santapp_ruler/attention/santapp.py:365-506
 *                              (SantaPlusEngine._approximate_attention), batched
 *                              over (batch, query head) as the decode branch of
 *                              _attention_forward does per head at :347-358
 *   santa_prefill              santapp_ruler/attention/santapp.py:320-346
 *                              (prefill branch -> sdpa_attention_forward)
 *   santa_prefill_paged        the same over the paged LayerCache
 *   santa_rope_append          santapp_ruler/attention/santapp.py:234-274, 308-313
 *                              (_append_cache and the RoPE of _attention_forward)
 *   santa_rope_append_paged    the same into the paged form of the LayerCache of :66-77
 *   santa_fingerprints         santapp_ruler/attention/santapp.py:598-691
 *   santa_kmeans_*             santapp_ruler/attention/minibatch_kmeans.py:58-267
 *                              (_squared_distances, _assign, _greedy_kmeans_plus_plus,
 *                              the mini-batch update and reassignment of fit_predict)
 *   santa_shard_*, santa_merge_shards
 *                              no counterpart (the reference is single-GPU):
 *                              santa_decode over sequence shards
 */
#ifndef SANTA_B200_H
#define SANTA_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define SANTA_OK 0
#define SANTA_ERR_INVALID_ARGUMENT -1 /* bad shape, stride, index or budget */
#define SANTA_ERR_UNSUPPORTED -2      /* valid but not built (dtype, head_dim) */
#define SANTA_ERR_CUDA -3             /* a CUDA runtime call failed */
#define SANTA_ERR_WORKSPACE -4        /* workspace missing or too small */

/* ---- enums ----------------------------------------------------------- */
#define SANTA_DTYPE_F32 0
#define SANTA_DTYPE_BF16 1

/* decode modes: the four reference modes (santapp.py:395-468) plus the
 * exact-top-k-plus-uniform-samples estimator. */
#define SANTA_MODE_TOPK 0    /* budget walk over ranked clusters, plain softmax */
#define SANTA_MODE_GUIDED 1  /* cluster-guided importance sampling */
#define SANTA_MODE_UNIFORM 2 /* uniform importance sampling over the prefix */
#define SANTA_MODE_SANTA 3   /* exact-softmax proposal (reads every old key) */
#define SANTA_MODE_HYBRID 4  /* exact top-k clusters + uniform samples of the rest */

#define SANTA_SAMPLES_DEVICE 0   /* draw samples on the device (Philox4x32-10) */
#define SANTA_SAMPLES_INJECTED 1 /* caller passes the draws (parity runs) */

/* ---- shapes ---------------------------------------------------------- */

/* Geometry of one attention layer's KV cache.
 * Contiguous (block_table NULL): key/value caches are [batch, num_kv_heads,
 * capacity, head_dim], row-major.
 * Paged (block_table set, the LayerCache of santapp.py:66-77 split into
 * fixed-size pages): key/value are page pools [num_pages, num_kv_heads,
 * page_size, head_dim]; token p of sequence b lives in page
 * block_table[b * max_pages + p / page_size], slot p % page_size (capacity =
 * max_pages * page_size; page_size a power of two).  Page ids outside
 * [0, num_pages) read page 0.  The summary build and every single-GPU decode
 * entry point accept both layouts; the santa_shard_* entry points take
 * contiguous caches only (SANTA_ERR_UNSUPPORTED).  Cache rows (batch x
 * num_kv_heads x capacity, or num_pages x num_kv_heads x page_size) must be
 * below 2^31 - 2 (SANTA_ERR_UNSUPPORTED).
 * Tokens [0, n_total) are valid; [0, sample_end) is the clustered old prefix
 * (santapp.py:374-379), [sample_end, n_total) is attended exactly. */
typedef struct SantaGeometry {
    int32_t batch;
    int32_t num_kv_heads;
    int32_t group;        /* query heads per KV head (GQA), <= 8 */
    int32_t head_dim;     /* 64 or 128 */
    int32_t capacity;     /* tokens per sequence (contiguous: row stride of the cache) */
    int32_t n_total;      /* valid tokens */
    int32_t sample_end;   /* end of the clustered prefix, 0 < sample_end <= n_total */
    int32_t kv_dtype;     /* SANTA_DTYPE_F32 or SANTA_DTYPE_BF16 */
    const int32_t *block_table; /* paged: device [batch][max_pages] page ids; NULL: contiguous */
    int32_t page_size;    /* paged: tokens per page, a power of two */
    int32_t max_pages;    /* paged: pages per sequence (block_table row length) */
    int32_t num_pages;    /* paged: pages in each pool */
    int32_t reserved;
} SantaGeometry;

/* Cluster summary of every (batch, KV head): the ClusterSummary fields of
 * santapp.py:53-63 in fixed-stride arrays, plus a copy of the old prefix of
 * K and V physically reordered so that each cluster is a contiguous run.
 * Per (b, kv): rows [0, n_groups) of starts/lengths/log_n/centroids are the
 * non-empty clusters in ascending cluster id (santapp.py:513-524). */
typedef struct SantaSummary {
    int32_t *members;      /* [B, Hkv, sample_end] token ids, sorted by (cluster, token) */
    int32_t *positions;    /* [B, Hkv, sample_end] inverse permutation of members */
    int32_t *starts;       /* [B, Hkv, max_groups] start of each cluster in members */
    int32_t *lengths;      /* [B, Hkv, max_groups] */
    float *log_n;          /* [B, Hkv, max_groups] fl32(log(fl64(length))) */
    float *centroids;      /* [B, Hkv, max_groups, head_dim] mean key, fp32 */
    int32_t *n_groups;     /* [B, Hkv] number of non-empty clusters */
    void *sorted_key;      /* [B, Hkv, sample_end, head_dim] cache dtype */
    void *sorted_value;    /* [B, Hkv, sample_end, head_dim] cache dtype */
    int32_t max_groups;    /* cluster id bound (n_clusters), <= 1024 */
} SantaSummary;

typedef struct SantaDecodeParams {
    int32_t mode;          /* SANTA_MODE_* */
    int32_t topk_clusters; /* HYBRID: exact clusters per query head */
    int32_t token_budget;  /* TOPK: samples_per_head of the reference (santapp.py:391, 409) */
    int32_t samples;       /* GUIDED/UNIFORM/SANTA/HYBRID: draws per query head, <= 1024 */
    float scale;           /* softmax scale, 1/sqrt(head_dim) in the reference */
    int32_t sample_source; /* SANTA_SAMPLES_DEVICE or SANTA_SAMPLES_INJECTED */
    uint64_t seed;         /* Philox key for device sampling */
    uint64_t step;         /* Philox counter word (decode step) */
    int32_t num_splits;    /* CTAs per (batch, KV head); 0 = pick automatically */
    const uint64_t *step_dev; /* optional device word read by the kernels in place of
                                 step (a decode step captured once in a CUDA graph and
                                 replayed with a new step each time); NULL: step */
} SantaDecodeParams;

/* ---- library --------------------------------------------------------- */
const char *santa_status_string(int status);
/* Last CUDA error recorded by an entry point that returned SANTA_ERR_CUDA. */
int santa_last_cuda_error(void);
const char *santa_version(void);

/* ---- cluster summary -------------------------------------------------- */

/* Workspace for santa_build_summary. */
int santa_build_summary_workspace_bytes(const SantaGeometry *geo, int32_t n_clusters,
                                        size_t *bytes);

/* Build the cluster summary from per-token cluster labels.
 * key_cache/value_cache: the layer's cache (geometry above).
 * labels: [B, Hkv, sample_end] int32 in [0, n_clusters).
 * Replaces SantaPlusEngine._build_summary (santapp.py:508-540): counts by
 * bincount, members by a stable sort on the label, starts by exclusive
 * cumsum, centroids as sequential fp32 sums in ascending token order (the
 * order CPU index_add_ uses) divided by the count.  Also writes the
 * cluster-sorted K/V copy that santa_decode streams from. */
int santa_build_summary(const SantaGeometry *geo, const void *key_cache,
                        const void *value_cache, const int32_t *labels,
                        int32_t n_clusters, const SantaSummary *out,
                        void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- sparse decode ---------------------------------------------------- */

int santa_decode_workspace_bytes(const SantaGeometry *geo, const SantaDecodeParams *p,
                                 int32_t max_groups, size_t *bytes);

/* One decode step for every (batch, query head).
 * q:        [B, Hkv*group, head_dim] fp32 query (RoPE already applied).
 * sample_a / sample_b: [B, Hq, samples] int32 draws when
 *           sample_source == SANTA_SAMPLES_INJECTED, else NULL:
 *             HYBRID  a = rank in [0, n_rest) among non-selected prefix tokens
 *             GUIDED  a = cluster row in [0, n_groups), b = offset inside it
 *             UNIFORM a = token id in [0, sample_end)
 *             SANTA   a = token id in [0, sample_end)
 * out:      [B, Hq, head_dim] fp32 attention output.
 * lse:      [B, Hq] fp32 log of the estimator's softmax denominator (natural
 *           log), for merging partial results across sequence shards.
 * n_exact:  [B, Hq] int32 exact old-prefix tokens (TOPK/HYBRID), or NULL.
 * ess:      [B, Hq] fp32 effective sample size / samples (santapp.py:481-485)
 *           for sampling modes, or NULL. */
int santa_decode(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                 const void *key_cache, const void *value_cache,
                 const SantaSummary *summary, const int32_t *sample_a,
                 const int32_t *sample_b, float *out, float *lse, int32_t *n_exact,
                 float *ess, void *workspace, size_t workspace_bytes,
                 cudaStream_t stream);

/* santa_decode in two stream-ordered halves sharing one workspace:
 *   santa_decode_plan     centroid scoring, ranking, selection and draws
 *                         (santapp.py:395-468); writes the per-(b, kv) work
 *                         list into the workspace and n_exact if non-NULL;
 *   santa_decode_execute  the gather attention and the LSE merge over that
 *                         work list (santapp.py:472-506).
 * Both must be called with the same geometry, params, q and summary. */
int santa_decode_plan(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                      const void *key_cache, const void *value_cache,
                      const SantaSummary *summary, const int32_t *sample_a,
                      const int32_t *sample_b, int32_t *n_exact, void *workspace,
                      size_t workspace_bytes, cudaStream_t stream);
int santa_decode_execute(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                         const void *key_cache, const void *value_cache,
                         const SantaSummary *summary, float *out, float *lse, float *ess,
                         void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* Size of the fixed scratch array behind santa_decode_static_scratch. */
#define SANTA_DECODE_STATIC_SCRATCH_BYTES (16u << 20) /* 16 MiB */

/* santa_decode for callers that cannot allocate device memory.  It has no
 * counterpart in the reference.  Some callers may not call cudaMalloc: a
 * serving stack whose memory manager has reserved all device memory for its
 * own pools, a host application that loads this library as a plugin and bans
 * device allocations after start-up, or a decode loop that cannot afford
 * cudaMalloc's implicit device synchronisation.  This entry point takes the
 * same inputs and outputs as santa_decode but no workspace: the scratch lives
 * in a fixed SANTA_DECODE_STATIC_SCRATCH_BYTES array inside the library, held
 * by every GPU that loads the library until the process exits.  It allocates
 * nothing.
 *   - Geometries whose santa_decode_workspace_bytes exceeds the array are
 *     refused with SANTA_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address (once
 *     per device, with that device current) and keeps it for the life of the
 *     process; make that first call before any stream capture.  The address
 *     belongs to the device's primary context: a process that destroys that
 *     context (cudaDeviceReset) must not call this entry point on that device
 *     again, since the kept address would be stale.
 *   - All calls on a device share the one array and it keeps the previous
 *     call's contents; each call clears what must start at zero, but calls
 *     whose work overlaps on the GPU (other streams, other host threads) race
 *     on it and must be serialised by the caller. */
int santa_decode_static_scratch(const SantaGeometry *geo, const SantaDecodeParams *p,
                                const float *q, const void *key_cache, const void *value_cache,
                                const SantaSummary *summary, const int32_t *sample_a,
                                const int32_t *sample_b, float *out, float *lse,
                                int32_t *n_exact, float *ess, cudaStream_t stream);

/* Selection step of santa_decode alone, read out per query head: which
 * clusters are attended exactly and which sorted rows were sampled.  Same
 * arguments and workspace as santa_decode.  Replaces the ranking and draw
 * part of _approximate_attention (santapp.py:397-411, 429-468) for tests and
 * for the distinct-row traffic accounting.
 * selected:    [B, Hq, max_groups] uint8, 1 = cluster row attended exactly, or NULL.
 * sample_rows: [B, Hq, samples] int32 row in the cluster-sorted copy, -1 = none, or NULL.
 * n_exact:     [B, Hq] int32, or NULL. */
int santa_decode_select(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                        const void *key_cache, const void *value_cache,
                        const SantaSummary *summary, const int32_t *sample_a,
                        const int32_t *sample_b, uint8_t *selected, int32_t *sample_rows,
                        int32_t *n_exact, void *workspace, size_t workspace_bytes,
                        cudaStream_t stream);

/* Injected draws out of range: *segments = the number of (batch, KV head)
 * segments whose last selection in this workspace (santa_decode, _plan,
 * _select or a shard entry point with SANTA_SAMPLES_INJECTED) met a draw
 * outside the range documented at santa_decode; such a draw is clamped into
 * range.  The selection kernel clears and sets one flag per segment at the
 * start of the workspace; this call synchronises the stream and reads them
 * (host-blocking, for parity runs). */
int santa_decode_bad_draws(const SantaGeometry *geo, const void *workspace,
                           size_t workspace_bytes, int32_t *segments, cudaStream_t stream);

/* ---- KV cache (attention/santapp.py:66-77, 234-283, 308-313) ---------- */

/* RoPE of the new tokens' queries and keys (x*cos + rotate_half(x)*sin with
 * every product and the sum rounded to bf16, as torch evaluates the
 * reference's bf16 expression) and their append to the layer cache at
 * [start, start + tokens) (LayerCache append, santapp.py:234-274).
 * q [B, tokens, Hq, D], k and v [B, tokens, Hkv, D], cos and sin [B, tokens, D]
 * (bf16, the projections' natural layout); caches [B, Hkv, capacity, D] bf16.
 * Rotated queries out as [B, Hq, tokens, D] bf16 and/or fp32 (either may be
 * NULL).  Trimming (santapp.py:276-283) is a host-side length change. */
int santa_rope_append(int32_t batch, int32_t tokens, int32_t num_query_heads,
                      int32_t num_kv_heads, int32_t head_dim, const void *q, const void *k,
                      const void *v, const void *cos, const void *sin, void *key_cache,
                      void *value_cache, int32_t capacity, int32_t start, void *q_rot_bf16,
                      float *q_rot_f32, cudaStream_t stream);

/* The same into paged pools [num_pages, Hkv, page_size, head_dim] (the
 * paged SantaGeometry layout): token start + t of sequence b goes to page
 * block_table[b * max_pages + (start + t) / page_size], slot (start + t) %
 * page_size.  page_size a power of two; start + tokens <= max_pages *
 * page_size.  Tokens whose page id is outside [0, num_pages) are not written
 * (the caller maps the pages before the append). */
int santa_rope_append_paged(int32_t batch, int32_t tokens, int32_t num_query_heads,
                            int32_t num_kv_heads, int32_t head_dim, const void *q, const void *k,
                            const void *v, const void *cos, const void *sin, void *key_pool,
                            void *value_pool, const int32_t *block_table, int32_t page_size,
                            int32_t max_pages, int32_t num_pages, int32_t start,
                            void *q_rot_bf16, float *q_rot_f32, cudaStream_t stream);

/* ---- dense prefill (attention/santapp.py:320-346) ---------------------- */

typedef struct SantaPrefillShape {
    int32_t batch;
    int32_t num_query_heads;  /* multiple of num_kv_heads (GQA) */
    int32_t num_kv_heads;
    int32_t seq_len;          /* T */
    int32_t head_dim;         /* 128 */
    float scale;              /* softmax scale, 1/sqrt(head_dim) in the reference */
    int32_t causal;           /* 1: key s attends only to queries t >= s */
    int32_t kv_capacity;      /* tokens between the (batch, KV head) blocks of k
                                 and v (a KV cache's capacity), >= seq_len;
                                 0 = seq_len */
} SantaPrefillShape;

/* Workspace: the 32 KB shared-memory images of every 128-token tile of K and
 * of V^T (2 * B * Hkv * ceil(T / 128) * 32768 bytes). */
int santa_prefill_workspace_bytes(const SantaPrefillShape *shape, size_t *bytes);

/* Attention of every query position over the prompt, as the reference's
 * prefill (sdpa_attention_forward -> torch scaled_dot_product_attention,
 * is_causal=True, GQA by head // group).  q [B, Hq, T, D], k and v
 * [B, Hkv, kv_capacity, D] (tokens [0, T) used), out [B, Hq, T, D], all bf16
 * and 16-byte aligned; lse
 * [B, Hq, T] fp32 natural-log softmax denominators (or NULL).  tcgen05 MMAs
 * with fp32 accumulation; P is rounded to bf16 before the P.V product.
 * error_flag (device int32, zeroed by the caller) is set to 1 if a bounded
 * wait inside the kernel gave up; the output is then undefined. */
int santa_prefill(const SantaPrefillShape *shape, const void *q, const void *k, const void *v,
                  void *out, float *lse, int32_t *error_flag, void *workspace,
                  size_t workspace_bytes, cudaStream_t stream);

/* The same with K and V in paged pools [num_pages, Hkv, page_size, D] (the
 * paged SantaGeometry layout; tokens [0, seq_len) through block_table
 * [batch][max_pages]; page ids outside [0, num_pages) read page 0).
 * shape->kv_capacity is ignored; max_pages * page_size >= seq_len. */
int santa_prefill_paged(const SantaPrefillShape *shape, const void *q, const void *key_pool,
                        const void *value_pool, const int32_t *block_table, int32_t page_size,
                        int32_t max_pages, int32_t num_pages, void *out, float *lse,
                        int32_t *error_flag, void *workspace, size_t workspace_bytes,
                        cudaStream_t stream);

/* ---- key fingerprints (attention/santapp.py:598-690) -------------------- */

int santa_fingerprints_workspace_bytes(int32_t cols, size_t *bytes);

/* Fingerprints of one (layer, KV head): out[n][h*P + p] =
 * fl32(dot(key_n, q_h[probes[p]]) / divisor) for the group's `group` query
 * heads (santapp.py:672-683), then, if normalize, the per-column population
 * z-score (x - mean) / (std + 1e-6) (:684-691).  keys [n, d] (SANTA_DTYPE_F32
 * or _BF16, upcast exactly); queries: rotated fp32 queries, head h of the group
 * at queries + h * q_head_stride, [T, d] per head; probes [P] int64 positions;
 * divisor = fl32(sqrt(d)).  Defined arithmetic: fmaf-chain dots, IEEE divide,
 * column mean and variance as exact Q64.64 sums divided in fp64 then rounded
 * to fp32, sqrt correctly rounded: results do not depend on reduction order. */
int santa_fingerprints(const void *keys, int32_t key_dtype, int64_t n, int32_t d,
                       const float *queries, int64_t q_head_stride, int32_t group,
                       const int64_t *probes, int32_t n_probes, float divisor,
                       int32_t normalize, float *out, void *workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* ---- MiniBatchKMeans (attention/minibatch_kmeans.py) -------------------- */

/* The data-dependent arithmetic of SklearnLikeTorchMiniBatchKMeans.fit_predict
 * (minibatch_kmeans.py:128-334); the caller keeps the reference's control flow
 * and its numpy RandomState draws.  x is [n_rows, d] fp32 row-major; `rows`
 * (int64, may be NULL) selects the rows an operation sees (x[rows[i]]), as
 * the reference's x[batch_ids] / x[init_ids] / x[validation_ids].
 * Defined arithmetic: dots are sequential fmaf chains over d; dist2 =
 * max(0, fl32(fl32(|x|^2 + |c|^2) - 2 dot)); inertia and potentials are exact
 * Q64.64 fixed-point sums, accumulated into two uint64 words (lo, hi) that the
 * caller zeroes. d % 4 == 0 and d <= 512 for assign; k <= 4096. */

/* out[i] = |x_i|^2 for n rows (_squared_distances' x^2 term, :58-66). */
int santa_kmeans_sqnorm(const float *x, int64_t n, int32_t d, float *out, cudaStream_t stream);

/* Nearest centre of every selected row, lowest index on ties (_assign, :68-71).
 * xx: |x|^2 indexed like x; cc: |c|^2 of the k centres.  labels [n] int32,
 * min_dist [n] (or NULL), inertia_fx [2] uint64 += fixed-point sum (or NULL). */
int santa_kmeans_assign(const float *x, const int64_t *rows, const float *xx, int64_t n,
                        int32_t d, const float *centers, const float *cc, int32_t k,
                        int32_t *labels, float *min_dist, unsigned long long *inertia_fx,
                        cudaStream_t stream);

int santa_kmeans_update_workspace_bytes(int64_t nb, int32_t k, size_t *bytes);

/* Mini-batch centre update (:226-239): batch counts, per-cluster sums in
 * ascending batch order, new = (c * n + sum) / (n + bc) for clusters in the
 * batch; counts updated in place, centers_new written, batch_counts [k] (or
 * NULL).  Labels outside [0, k) are ignored. */
int santa_kmeans_update(const float *x, const int64_t *rows, int64_t nb, int32_t d,
                        const int32_t *labels, int32_t k, const float *centers, float *counts,
                        float *centers_new, float *batch_counts, void *workspace,
                        size_t workspace_bytes, cudaStream_t stream);

/* Low-count reassignment (:241-267): centre clusters[i] <- selected row
 * batch_rows[i], its count <- new_count. */
int santa_kmeans_reassign(const float *x, const int64_t *rows, const int32_t *batch_rows,
                          const int32_t *clusters, int32_t n_reassign, int32_t d,
                          float *centers, float *counts, float new_count, cudaStream_t stream);

int santa_kmeans_plusplus_workspace_bytes(int64_t n, int32_t trials, size_t *bytes);

/* Greedy k-means++ over the n selected rows (_greedy_kmeans_plus_plus,
 * :73-126): centre 0 = row first_id; centre c picks, among `trials`
 * candidates found by searchsorted (fp64) of uniforms[(c-1)*trials + t] x
 * potential in the fixed-point prefix sums of the closest distances, the one
 * with the lowest potential (first on ties).  uniforms: device fp64
 * [(k-1)*trials] in the reference's draw order.  centers [k, d]; chosen_ids
 * [k] indices into the selected rows (or NULL). trials <= 16. */
int santa_kmeans_plusplus(const float *x, const int64_t *rows, const float *xx, int64_t n,
                          int32_t d, int32_t k, int32_t trials, int64_t first_id,
                          const double *uniforms, float *centers, int64_t *chosen_ids,
                          void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- sequence-sharded decode ------------------------------------------ */

/* The reference decodes on one GPU (README.md:355): these entry points have
 * no one-to-one counterpart there.  They split santa_decode in HYBRID mode
 * (santapp.py:365-506 with the exact top-k clusters plus uniform samples of
 * the rest) over contiguous shards of every sequence's clustered prefix, one
 * shard per rank, around two small exchanges that the caller runs (NCCL
 * all-gathers):
 *
 *   1. santa_shard_candidates: this shard's top-k cluster keys per
 *      (sequence, query head).  Exchange 1 gathers them from every shard.
 *   2. santa_shard_plan: every rank takes the same global top-k from the
 *      gathered keys and selects the local clusters among them; samples
 *      are drawn from this shard's non-selected tokens (the caller splits
 *      the sample budget across shards in proportion to their token counts,
 *      and each sample carries the weight n_rest_shard / samples_shard of
 *      stratified sampling).
 *   3. santa_shard_execute: the gather attention over the shard's rows,
 *      written as an unnormalised partial per (sequence, query head).
 *      Exchange 2 gathers the partials.
 *   4. santa_merge_shards: LSE merge of the gathered partials into out, lse
 *      and ess, identical on every rank.
 *
 * A cluster's global id is cluster_base + its row in this shard's summary;
 * shards list their clusters in increasing global id, so the ranking (guess
 * descending, lowest global id first on ties) is the one santa_decode applies
 * to the concatenated summary.  The recent window [sample_end, n_total) lives
 * on one shard (the caller gives the others n_total == sample_end).  bf16
 * caches only; geometry, params, summary and workspace as for santa_decode
 * (santa_decode_workspace_bytes). */
#define SANTA_MAX_SHARDS 32
#define SANTA_SHARD_MAX_KEYS 512 /* num_shards * topk_clusters */
#define SANTA_PARTIAL_FLOATS(head_dim) ((head_dim) + 8)

/* Peer-memory exchange (optional): every rank allocates one exchange buffer
 * (santa_p2p_alloc, santa_p2p_buffer_bytes), shares its IPC handle, maps the
 * others' (santa_p2p_ipc_open) and passes the table of all ranks' buffers as
 * mapped in this process.  A step is then two launches and no collective:
 *   santa_shard_plan   scores this shard's clusters, stores its top-k keys
 *                      straight into every rank's buffer, waits for every
 *                      rank's keys of the same (sequence, query head), and
 *                      selects and draws as with gathered keys;
 *   santa_shard_attend the gather attention, then stores this shard's
 *                      partials into every rank's buffer, waits for every
 *                      rank's and merges them into out / lse / ess.
 * Every 8-byte word a kernel stores into a peer's buffer carries the step's
 * epoch beside its data (no flags, no fences).  Waits are bounded by
 * wait_limit_us (0: 2 s); a wait that runs out sets *error_flag to 1, and the
 * outputs of that step (and of later steps until the flag is cleared) are
 * NaN.  epoch = the step number + 1, increasing by one per step, the same
 * for the plan and attend calls of one step on every rank; all ranks make the
 * same calls in the same order.  The plan launch needs all of its thread-block
 * clusters resident at once (SANTA_ERR_UNSUPPORTED otherwise) and k <= 32;
 * global cluster ids must stay below 2^24 - 1. */
typedef struct SantaP2P {
    void *const *peer_buffers;   /* device array [num_shards] of buffers (own at shard_index) */
    void *local_buffer;          /* this rank's buffer (256-byte aligned) */
    uint64_t epoch;
    int32_t *error_flag;         /* device int32 */
    int32_t rows;                /* B * Hq */
    int32_t keys_per_row;        /* topk_clusters */
    int32_t partial_floats;      /* SANTA_PARTIAL_FLOATS(head_dim) */
    int32_t wait_limit_us;       /* bound of every wait; 0 = 2 s */
} SantaP2P;

#define SANTA_IPC_HANDLE_BYTES 64

int santa_p2p_buffer_bytes(int32_t num_shards, int32_t rows, int32_t keys_per_row,
                           int32_t head_dim, size_t *bytes);
/* cudaMalloc'd exchange buffer, zeroed (no word carries an epoch tag). */
int santa_p2p_alloc(size_t bytes, void **buffer);
int santa_p2p_free(void *buffer);
int santa_p2p_ipc_handle(void *buffer, void *handle);
int santa_p2p_ipc_open(const void *handle, void **mapped);
int santa_p2p_ipc_close(void *mapped);
/* 8 bytes at a device address (own or mapped peer buffer), for set-up checks. */
int santa_p2p_peek(const void *address, uint64_t *value);
int santa_p2p_poke(void *address, uint64_t value);

typedef struct SantaShard {
    int32_t shard_index;         /* this rank's shard, < num_shards */
    int32_t num_shards;          /* <= SANTA_MAX_SHARDS */
    int32_t cluster_base;        /* global id of row 0 of this shard's summary */
    int32_t reserved;
    const uint64_t *candidates;  /* plan: [num_shards][B*Hq][topk_clusters] gathered keys
                                    (ignored with p2p: the plan launch exchanges them) */
    const SantaP2P *p2p;         /* NULL: the caller exchanges keys and partials */
} SantaShard;

/* Candidate keys: [B*Hq][topk_clusters] uint64, per row descending, key =
 * (order-preserving bits of the fp32 guess) << 32 | (0xFFFFFFFF - global id),
 * 0 where the shard has fewer clusters. */
int santa_shard_candidates(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                           const void *key_cache, const void *value_cache,
                           const SantaSummary *summary, const SantaShard *shard, uint64_t *keys,
                           void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* Selection and draws of this shard under the global top-k of
 * shard->candidates; sample_a as for santa_decode (ranks in [0, n_rest) of
 * this shard) when sample_source is SANTA_SAMPLES_INJECTED. */
int santa_shard_plan(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                     const void *key_cache, const void *value_cache, const SantaSummary *summary,
                     const SantaShard *shard, const int32_t *sample_a, int32_t *n_exact,
                     void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* partial: [B*Hq][SANTA_PARTIAL_FLOATS(head_dim)] fp32: m (log2 units), l,
 * ms, e1, e2, samples, 0, 0, then o[head_dim] = sum 2^(lw - m) v; l = sum
 * 2^(lw - m); ms, e1, e2 the same sums over the sample weights alone. */
int santa_shard_execute(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                        const void *key_cache, const void *value_cache,
                        const SantaSummary *summary, const SantaShard *shard, float *partial,
                        void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* Selection readout of santa_shard_plan (arguments of santa_decode_select);
 * with shard->p2p it takes part in the key exchange like santa_shard_plan. */
int santa_shard_select(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                       const void *key_cache, const void *value_cache,
                       const SantaSummary *summary, const SantaShard *shard,
                       const int32_t *sample_a, uint8_t *selected, int32_t *sample_rows,
                       int32_t *n_exact, void *workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* Peer-memory form of santa_shard_execute + exchange 2 + santa_merge_shards
 * in one launch (shard->p2p required): out [B*Hq][head_dim] (16-byte aligned
 * for head_dim 128, 8-byte for 64), lse and ess as santa_decode writes them,
 * identical on every rank and bit-identical to the NCCL-exchange path. */
int santa_shard_attend(const SantaGeometry *geo, const SantaDecodeParams *p, const float *q,
                       const void *key_cache, const void *value_cache,
                       const SantaSummary *summary, const SantaShard *shard, float *out,
                       float *lse, float *ess, void *workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* partials: [num_shards][rows][SANTA_PARTIAL_FLOATS(head_dim)]; rows = B*Hq.
 * out [rows][head_dim], lse [rows] (natural log) and ess [rows] (may be
 * NULL) as santa_decode writes them. */
int santa_merge_shards(int32_t rows, int32_t head_dim, int32_t num_shards, const float *partials,
                       float *out, float *lse, float *ess, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SANTA_B200_H */
