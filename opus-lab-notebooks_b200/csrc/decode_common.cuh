// Shared definitions of the SANTA++ decode kernels (selection + attention).
//
// A decode step is two launches:
//   select  per (batch, KV head) = segment bh: centroid guesses for the GQA
//           group, ranking, top-k / budget walk, the union of the group's
//           selections and the importance samples; one CTA per segment, or
//           (hybrid, k <= 32) a cluster of one CTA per query head
//           (decode_select_group.cu).  It writes a work list for the segment
//           into the workspace.
//   attend  streams the rows of every segment's work list (selected clusters
//           of the cluster-sorted copy, the exact recent window of the cache,
//           sampled rows) with an online softmax per query head, and merges
//           partial results with an LSE merge.
//
// Every segment's work list is a virtual row space [0, U + R + NS):
//   [0, U)          rows of the union of selected clusters (ascending cluster)
//   [U, U + R)      the exact recent window [sample_end, n_total) of the cache
//   [U + R, ...)    the sampled rows, head-major
#pragma once

#include "common.cuh"

namespace santa {

constexpr int kSelThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// packed sample word: bits 0-23 sorted row, 24-26 local head, 27 = absolute
// log weight (santa mode: lw does not depend on the row's score)
constexpr uint32_t kPosMask = 0xFFFFFFu;
constexpr int kHeadShift = 24;
constexpr uint32_t kAbsBit = 1u << 27;

// row mask bits: 0-7 local heads the row contributes to, 8 = sampled row,
// 9 = absolute log weight
constexpr int kMaskSample = 256;
constexpr int kMaskAbs = 512;


struct DecodeWs {
    int32_t *counters;   // [BH] CTAs finished per segment (last one merges)
    int32_t *flag;       // [BH] 1 = an injected draw of the segment was out of range
                         // (clamped); cleared by the segment's selection kernel
    int32_t *meta;       // [BH][8]: 0 n_union, 1 U, 2 R, 3 n_samples, 4 total rows
    int32_t *head_meta;  // [BH][8][2]: n_exact, n_samples
    int32_t *u_start;    // [BH][G] sorted-row start of each union entry
    int32_t *u_mask;     // [BH][G] heads that selected it
    int32_t *u_cid;      // [BH][G] cluster row of each union entry
    int32_t *u_off;      // [BH][G+1] prefix of union rows
    int32_t *s_pos;      // [BH][g*S] packed sample words
    float *s_off;        // [BH][g*S] log2-units offset (or absolute log2 weight)
    float *lse_old;      // [BH][8] santa mode: log2-sum-exp2 of old scores
    float *partial;      // [n_slots][g][D + 8] split partials
    int32_t *w_row;      // [BH][sample_end] union rows expanded: row | (head mask << 24)
};

__host__ __device__ inline int partial_stride(int D) { return D + 8; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline size_t decode_ws_layout(int BH, int G, int g, int S, int n_slots, int D, int N, char *base,
                               DecodeWs *ws) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off = align_up(off + bytes, 256);
        return o;
    };
    const int gs = g * (S > 0 ? S : 1);
    size_t o_flag = take((size_t)BH * 4);  // first: santa_decode_bad_draws reads it
    size_t o_cnt = take((size_t)BH * 4);
    size_t o_meta = take((size_t)BH * 8 * 4);
    size_t o_hm = take((size_t)BH * 16 * 4);
    size_t o_us = take((size_t)BH * G * 4);
    size_t o_um = take((size_t)BH * G * 4);
    size_t o_uc = take((size_t)BH * G * 4);
    size_t o_uo = take((size_t)BH * (G + 1) * 4);
    size_t o_sp = take((size_t)BH * gs * 4);
    size_t o_so = take((size_t)BH * gs * 4);
    size_t o_lo = take((size_t)BH * 8 * 4);
    size_t o_pa = take((size_t)n_slots * g * partial_stride(D) * 4);
    size_t o_wr = take((size_t)BH * N * 4);
    if (base && ws) {
        ws->w_row = (int32_t *)(base + o_wr);
        ws->counters = (int32_t *)(base + o_cnt);
        ws->flag = (int32_t *)(base + o_flag);
        ws->meta = (int32_t *)(base + o_meta);
        ws->head_meta = (int32_t *)(base + o_hm);
        ws->u_start = (int32_t *)(base + o_us);
        ws->u_mask = (int32_t *)(base + o_um);
        ws->u_cid = (int32_t *)(base + o_uc);
        ws->u_off = (int32_t *)(base + o_uo);
        ws->s_pos = (int32_t *)(base + o_sp);
        ws->s_off = (float *)(base + o_so);
        ws->lse_old = (float *)(base + o_lo);
        ws->partial = (float *)(base + o_pa);
    }
    return off;
}

// ---------------------------------------------------------------------------
// peer-memory exchange between sequence shards (one buffer per rank, mapped
// into every other rank's address space through CUDA IPC).  Low-latency
// protocol: every 8-byte word a producer stores into a peer's buffer carries
// the step's epoch tag next to its data, so a consumer polls its own (local)
// buffer until each word it needs shows the current tag.  No flags and no
// memory fences: an aligned 8-byte store is single-copy atomic, so a word
// with the right tag also holds the right data.
//   [0, 1024)     set-up marker (at 768)
//   keys   u64   [2 parities][n ranks][rows][kk]  candidate keys, tag in
//                bits 24-31 (see ll_key_encode)
//   parts  u64x2 [2 parities][n ranks][rows][pf / 2] partials: one 16-byte
//                line holds two floats, each word = tag << 32 | float bits
//   stage  f32   [rows][pf]  this rank's partials before they are sent
//                (local use only)
// Epoch e (> 0, increasing by one per step) uses parity e & 1: a rank cannot
// run two steps ahead of a peer, because each step's selection waits for
// every peer's keys of that step, which a peer only sends after it finished
// reading the previous step's partials (the kernels of one rank run in
// stream order).
// ---------------------------------------------------------------------------
struct P2PArgs {
    void *const *peers;      // device array [n]: every rank's buffer as mapped here
    unsigned char *local;    // this rank's buffer
    unsigned long long epoch;
    unsigned long long wait_ns;  // bound of every wait (globaltimer ns)
    int32_t *err;            // set to 1 when a wait for a peer gave up
    int rank, n, rows, kk, pf;
};
constexpr size_t kP2PKeys = 1024;
__host__ __device__ inline size_t p2p_parts_offset(int n, int rows, int kk) {
    return (kP2PKeys + (size_t)2 * n * rows * kk * 8 + 255) / 256 * 256;
}
__host__ __device__ inline size_t p2p_stage_offset(int n, int rows, int kk, int pf) {
    return p2p_parts_offset(n, rows, kk) + (size_t)2 * n * rows * pf * 8;
}
__host__ __device__ inline size_t p2p_buffer_bytes(int n, int rows, int kk, int pf) {
    return p2p_stage_offset(n, rows, kk, pf) + (size_t)rows * pf * 4;
}
struct DecodeArgs {
    SantaGeometry geo;
    SantaDecodeParams p;
    SantaSummary sum;
    const float *q;
    const char *key_cache;
    const char *value_cache;
    const int32_t *sample_a;
    const int32_t *sample_b;
    float *out;
    float *lse;
    int32_t *n_exact;
    float *ess;
    int nsplit;   // SIMT attend: CTAs per segment
    DecodeWs ws;
    // sequence shards (HYBRID): global cluster id = cluster_base + cluster row
    int cluster_base;
    int num_shards;
    int shard_index;              // this rank's shard (threshold selection reads its own keys)
    uint64_t *cand_out;           // select: write the local top-k keys and stop
    const uint64_t *shard_cands;  // select: [num_shards][B*Hq][k] keys -> global top-k
    float *part_out;              // attend: unnormalised partial per (b, query head)
    P2PArgs p2p;                  // peers == nullptr: the caller exchanges
    int tma;                      // attend: the sorted copies' tensor maps are valid
};

// rank r's key list region (this step's parity) in the buffer at base
__device__ __forceinline__ uint64_t *p2p_key_slot(const P2PArgs &c, void *base, int r) {
    return (uint64_t *)((unsigned char *)base + kP2PKeys) +
           ((size_t)((c.epoch & 1) * c.n + r) * c.rows * c.kk);
}
// rank r's partial lines (this step's parity) in the buffer at base
__device__ __forceinline__ ulonglong2 *p2p_part_slot(const P2PArgs &c, void *base, int r) {
    return (ulonglong2 *)((unsigned char *)base + p2p_parts_offset(c.n, c.rows, c.kk)) +
           ((size_t)((c.epoch & 1) * c.n + r) * c.rows * (c.pf / 2));
}
__device__ __forceinline__ float *p2p_stage(const P2PArgs &c) {
    return (float *)(c.local + p2p_stage_offset(c.n, c.rows, c.kk, c.pf));
}

// tags: 8 bits (never 0) inside a key, 32 bits (never 0 in practice) beside
// a float; a zeroed buffer and the previous use of a parity (epoch - 2) never
// match the current epoch
__device__ __forceinline__ uint32_t ll_key_tag(unsigned long long epoch) {
    return (uint32_t)(epoch % 255ull) + 1u;
}
// key = order bits << 32 | (0xFFFFFFFF - global id) with global id < 2^24 - 1
// (the top byte of the low word is 0xFF and carries the tag instead); key 0
// (no key) is sent as the tag alone
__device__ __forceinline__ uint64_t ll_key_encode(uint64_t key, uint32_t tag) {
    return (key & 0xFFFFFFFF00FFFFFFull) | ((uint64_t)tag << 24);
}
__device__ __forceinline__ uint64_t ll_key_decode(uint64_t w) {
    const uint64_t lo = w & 0xFFFFFFull;
    return ((w >> 32) == 0ull && lo == 0ull) ? 0ull : ((w & 0xFFFFFFFF00000000ull) | 0xFF000000ull | lo);
}
__device__ __forceinline__ void st_relaxed_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_v2(ulonglong2 *p, uint64_t x, uint64_t y) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};\n" ::"l"(p), "l"(x), "l"(y)
                 : "memory");
}
__device__ __forceinline__ ulonglong2 ld_relaxed_sys_v2(const ulonglong2 *p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];\n"
                 : "=l"(v.x), "=l"(v.y)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint64_t p2p_now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Poll one key word of the local buffer until it carries `tag` (bounded by
// c.wait_ns from t0; on time-out the error flag is set and the word is
// returned as "no key").  ok is cleared on time-out and skips later waits.
__device__ __forceinline__ uint64_t ll_key_wait(const P2PArgs &c, const uint64_t *p, uint32_t tag,
                                                uint64_t t0, bool &ok) {
    for (uint32_t i = 0;; ++i) {
        const uint64_t w = ld_relaxed_sys(p);
        if ((uint32_t)((w >> 24) & 0xFFu) == tag) return ll_key_decode(w);
        if (!ok) return 0ull;
        if ((i & 31u) == 31u && p2p_now_ns() - t0 > c.wait_ns) {
            atomicExch(c.err, 1);
            ok = false;
            return 0ull;
        }
    }
}
// Poll one partial line of the local buffer until both words carry `tag`;
// the two floats, or NaN on time-out (error flag set, ok cleared).
__device__ __forceinline__ float2 ll_part_wait(const P2PArgs &c, const ulonglong2 *p,
                                               uint32_t tag, uint64_t t0, bool &ok) {
    for (uint32_t i = 0;; ++i) {
        const ulonglong2 v = ld_relaxed_sys_v2(p);
        if ((uint32_t)(v.x >> 32) == tag && (uint32_t)(v.y >> 32) == tag)
            return make_float2(__uint_as_float((uint32_t)v.x), __uint_as_float((uint32_t)v.y));
        if (!ok) return make_float2(__int_as_float(0x7FC00000), __int_as_float(0x7FC00000));
        if ((i & 31u) == 31u && p2p_now_ns() - t0 > c.wait_ns) {
            atomicExch(c.err, 1);
            ok = false;
            return make_float2(__int_as_float(0x7FC00000), __int_as_float(0x7FC00000));
        }
    }
}

// LSE merge of one (sequence, query head) row over the shards' partials
// (header m, l, ms, e1, e2, samples; values o[d]) in ascending shard order;
// part(r, j) returns float j of shard r's partial.  The single-launch merge
// kernel and the attention kernel's fused merge both use it, so the two
// exchange paths give the same bits.  One shard gives acc = o, L = l.
struct ShardMerged {
    float M, L, MS, E1, E2, ns;
};
template <typename Part>
__device__ __forceinline__ ShardMerged shard_merge_header(int num_shards, Part part) {
    ShardMerged s;
    s.M = -INFINITY;
    s.MS = -INFINITY;
    for (int r = 0; r < num_shards; ++r) {
        if (part(r, 1) > 0.f) s.M = fmaxf(s.M, part(r, 0));
        if (part(r, 3) > 0.f) s.MS = fmaxf(s.MS, part(r, 2));
    }
    s.L = 0.f;
    s.E1 = 0.f;
    s.E2 = 0.f;
    s.ns = 0.f;
    for (int r = 0; r < num_shards; ++r) {
        if (part(r, 1) > 0.f) s.L = fmaf(part(r, 1), exp2f(part(r, 0) - s.M), s.L);
        if (part(r, 3) > 0.f) {
            const float fe = exp2f(part(r, 2) - s.MS);
            s.E1 = fmaf(part(r, 3), fe, s.E1);
            s.E2 = fmaf(part(r, 4), fe * fe, s.E2);
        }
        s.ns += part(r, 5);
    }
    return s;
}
// (times 1/L, as the single-GPU merge does: one shard gives the same bits)
__device__ __forceinline__ float shard_out_scale(const ShardMerged &s) {
    return s.L > 0.f ? 1.f / s.L : 0.f;
}
__device__ __forceinline__ float shard_lse(const ShardMerged &s) {
    return s.L > 0.f ? (s.M + log2f(s.L)) * kLn2 : -INFINITY;
}
__device__ __forceinline__ float shard_ess(const ShardMerged &s) {
    return (s.ns > 0.f && s.E2 > 0.f) ? (s.E1 * s.E1 / s.E2) / s.ns : 0.f;
}

// ---------------------------------------------------------------------------
// row resolution: virtual row v of segment bh -> K/V row addresses + weights
// ---------------------------------------------------------------------------
struct RowInfo {
    const char *k;
    const char *v;
    float off;  // log2-units additive offset (or absolute weight when kMaskAbs)
    int mask;   // see kMask*
};

// sp / so: optional copy of the segment's first scap sample words and
// offsets in shared memory (rows beyond it are read from the workspace).
__device__ __forceinline__ RowInfo resolve_row(const DecodeArgs &a, int bh, int v, int U, int R,
                                               int total, int n_union, const int *u_off,
                                               const int *u_start, const int *u_mask,
                                               int row_bytes, const int32_t *sp = nullptr,
                                               const float *so = nullptr, int scap = 0) {
    RowInfo ri;
    const int g = a.geo.group;
    const int sample_end = a.geo.sample_end;
    const char *sk = (const char *)a.sum.sorted_key + (int64_t)bh * sample_end * row_bytes;
    const char *sv = (const char *)a.sum.sorted_value + (int64_t)bh * sample_end * row_bytes;
    if (v >= total) {
        ri.k = sk;
        ri.v = sv;
        ri.off = 0.f;
        ri.mask = 0;
    } else if (v < U) {
        int lo = 0, hi = n_union - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (u_off[mid] <= v) lo = mid;
            else hi = mid - 1;
        }
        const int row = u_start[lo] + (v - u_off[lo]);
        ri.k = sk + (int64_t)row * row_bytes;
        ri.v = sv + (int64_t)row * row_bytes;
        ri.off = 0.f;
        ri.mask = u_mask[lo];
    } else if (v < U + R) {
        const int64_t row = cache_row(a.geo, bh, sample_end + (v - U));
        ri.k = a.key_cache + row * row_bytes;
        ri.v = a.value_cache + row * row_bytes;
        ri.off = 0.f;
        ri.mask = (1 << g) - 1;
    } else {
        const int j = v - U - R;
        const uint32_t pk = j < scap ? (uint32_t)sp[j]
                                     : (uint32_t)a.ws.s_pos[(int64_t)bh * g * a.p.samples + j];
        const int row = (int)(pk & kPosMask);
        const int h = (int)((pk >> kHeadShift) & 7u);
        ri.k = sk + (int64_t)row * row_bytes;
        ri.v = sv + (int64_t)row * row_bytes;
        ri.off = j < scap ? so[j] : a.ws.s_off[(int64_t)bh * g * a.p.samples + j];
        ri.mask = (1 << h) | kMaskSample | ((pk & kAbsBit) ? kMaskAbs : 0);
    }
    return ri;
}

// Per-warp online-softmax state for a warp merge in shared memory.
template <int D>
struct WarpState {
    float m[SANTA_MAX_GROUP], l[SANTA_MAX_GROUP];
    float ms[SANTA_MAX_GROUP], e1[SANTA_MAX_GROUP], e2[SANTA_MAX_GROUP];
    float o[SANTA_MAX_GROUP][D];
};

// Merge NW warp states into one partial (m, l, ms, e1, e2, pad, o[D]) per
// head at dst (stride PSTR); threads [0, nthreads) participate.
template <int D>
__device__ void merge_warp_states(const WarpState<D> *ws, int NW, int g, float *dst, int tid,
                                  int nthreads) {
    const int PSTR = partial_stride(D);
    if (tid < g) {
        const int h = tid;
        float M = -INFINITY, MS = -INFINITY;
        for (int w = 0; w < NW; ++w) {
            M = fmaxf(M, ws[w].m[h]);
            MS = fmaxf(MS, ws[w].ms[h]);
        }
        float L = 0.f, E1 = 0.f, E2 = 0.f;
        for (int w = 0; w < NW; ++w) {
            if (ws[w].l[h] > 0.f) L += ws[w].l[h] * exp2f(ws[w].m[h] - M);
            if (ws[w].e1[h] > 0.f) {
                E1 += ws[w].e1[h] * exp2f(ws[w].ms[h] - MS);
                E2 += ws[w].e2[h] * exp2f(2.f * (ws[w].ms[h] - MS));
            }
        }
        dst[h * PSTR + 0] = M;
        dst[h * PSTR + 1] = L;
        dst[h * PSTR + 2] = MS;
        dst[h * PSTR + 3] = E1;
        dst[h * PSTR + 4] = E2;
    }
    for (int i = tid; i < g * D; i += nthreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, ws[w].m[h]);
        float acc = 0.f;
        for (int w = 0; w < NW; ++w)
            if (ws[w].l[h] > 0.f) acc += ws[w].o[h][d] * exp2f(ws[w].m[h] - M);
        dst[h * PSTR + 8 + d] = acc;
    }
}

// Merge partial slots first..first+count-1 (stride slot_step slots) of
// segment bh into out / lse / ess.
template <int D>
__device__ void merge_partials_to_output(const DecodeArgs &a, int bh, const float *pall,
                                         int count, int tid, int nthreads) {
    const int g = a.geo.group;
    const int PSTR = partial_stride(D);
    const int b = bh / a.geo.num_kv_heads, kv = bh - b * a.geo.num_kv_heads;
    for (int i = tid; i < g * D; i += nthreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
        for (int s = 0; s < count; ++s) M = fmaxf(M, pall[(s * g + h) * PSTR + 0]);
        float L = 0.f, acc = 0.f;
        for (int s = 0; s < count; ++s) {
            const float *ps = pall + (s * g + h) * PSTR;
            if (ps[1] > 0.f) {
                const float f = exp2f(ps[0] - M);
                L += ps[1] * f;
                acc += ps[8 + d] * f;
            }
        }
        const int64_t oh = (int64_t)b * a.geo.num_kv_heads * g + (int64_t)kv * g + h;
        a.out[oh * D + d] = L > 0.f ? acc / L : 0.f;
        if (d == 0) {
            if (a.lse) a.lse[oh] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
            if (a.ess) {
                float MS = -INFINITY;
                for (int s = 0; s < count; ++s) MS = fmaxf(MS, pall[(s * g + h) * PSTR + 2]);
                float E1 = 0.f, E2 = 0.f;
                for (int s = 0; s < count; ++s) {
                    const float *ps = pall + (s * g + h) * PSTR;
                    if (ps[3] > 0.f) {
                        E1 += ps[3] * exp2f(ps[2] - MS);
                        E2 += ps[4] * exp2f(2.f * (ps[2] - MS));
                    }
                }
                const int ns = a.ws.head_meta[((int64_t)bh * 8 + h) * 2 + 1];
                a.ess[oh] = (ns > 0 && E2 > 0.f) ? (E1 * E1 / E2) / (float)ns : 0.f;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                            uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                                  uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *(const uint32_t *)&v;
}

// mbarrier + bulk-copy (TMA engine, non-tensor form) helpers
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Bounded wait: gives up after ~2 s of wall time and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0u && global_timer_ns() - t0 > 2000000000ull) return false;
    }
}
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory");
}
// 16-byte asynchronous global->shared copy (L1 bypass)
__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst_smem)), "l"(src)
                 : "memory");
}
// The mbarrier receives one arrival once every cp.async this thread issued
// so far has landed (the barrier's expected count includes these arrivals).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------------------
// launchers (host, defined in decode_select.cu / decode_attend.cu)
// ---------------------------------------------------------------------------
int launch_plan(DecodeArgs &a, cudaStream_t stream);
int launch_execute(DecodeArgs &a, cudaStream_t stream);
int launch_expand(DecodeArgs &a, uint8_t *selected, int32_t *sample_rows, cudaStream_t stream);
// hybrid selection on a thread-block cluster (decode_select_group.cu)
bool select_group_supported(const DecodeArgs &a);
int launch_select_group(DecodeArgs &a, cudaStream_t stream);
int num_sms();
int attend_partial_slots(const SantaGeometry *geo, int nsplit);

// The Philox counter word of this decode step: the device word when the
// caller supplied one (a captured step replayed with a new counter), else
// the parameter.
__device__ __forceinline__ uint64_t decode_step_word(const SantaDecodeParams &p) {
    return p.step_dev ? *p.step_dev : p.step;
}

// Row costs on which the gather attention kernel splits the step's rows into
// equal CTA shares (a 32-bit scale: the API rejects geometries whose total
// could overflow it).
constexpr int kCostRow = 2;     // balancing cost of a union or recent-window row
constexpr int kCostSample = 3;  // balancing cost of a sampled (scattered) row
// balancing cost of starting a segment (ring drain, CTA fold, the next
// segment's q fragments, row entries and first copies: ~4-5 us, measured with
// per-CTA timers; 768 / 1024 / 1280 / 1536 / 2048 / 3072 swept on the 32K and
// 128K decode workloads and on one rank's share of the 8-shard 128K job,
// 1024-1536 within 1 us of each other, 1280 kept); charged before the
// segment's first row, so the CTA whose share covers a segment boundary
// takes fewer rows
constexpr int kCostSegment = 1280;
int launch_merge_shards(int rows, int head_dim, int num_shards, const float *partials,
                        float *out, float *lse, float *ess, cudaStream_t stream);

}  // namespace santa
