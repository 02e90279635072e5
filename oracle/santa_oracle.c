/*
 * CPU restatement of the SANTA++ hot path's integer and fp32 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: only tests, the smoke check and the CPU-baseline leg of bench.py
 * load it.  Nothing in the product path links or calls it.
 *
 * It restates, in plain C with an explicitly defined evaluation order, the
 * pieces of the reference whose results must match bit for bit:
 *
 *   - squared distances and nearest-centre assignment
 *       santapp_ruler/attention/minibatch_kmeans.py:58-71
 *   - greedy k-means++ initialisation
 *       santapp_ruler/attention/minibatch_kmeans.py:73-126
 *   - the mini-batch centre update (bincount / index_add_ / online means)
 *       santapp_ruler/attention/minibatch_kmeans.py:226-239
 *   - cluster-summary key centroids (index_add_ then divide)
 *       santapp_ruler/attention/santapp.py:526-533
 *   - centroid guess  log(n_g) + c_g . q * scale
 *       santapp_ruler/attention/santapp.py:397-400, 431-434
 *
 * Defined arithmetic (the CUDA kernels follow exactly the same rules):
 *
 *   dot(a, b)      acc = 0; for i in 0..d-1: acc = fmaf(a[i], b[i], acc)
 *   sqnorm(a)      dot(a, a)
 *   dist2(x, c)    max(0, fl32(fl32(|x|^2 + |c|^2) - 2 * dot(x, c)))
 *   sums of non-negative fp32 values (potentials, inertia, prefix sums):
 *                  every term is truncated to unsigned fixed point with 64
 *                  fractional bits and added exactly in 128-bit integers, so
 *                  the result does not depend on summation order; the total
 *                  is converted back as fl32(fl64(hi) + fl64(lo) * 2^-64).
 *   cluster sums   sequential fp32 additions in ascending row order, which
 *                  is exactly what CPU index_add_ does.
 *
 * The reference evaluates the same formulas through MKL sgemm and torch's
 * vectorised CPU reductions, whose summation order is not specified and
 * differs between CPUs; the restatement therefore agrees with the reference
 * to the last ulp or so, and the golden-vector tests measure how often that
 * changes a label or a selection.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no -ffast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

/* ------------------------------------------------------------------ */
/* defined arithmetic                                                  */
/* ------------------------------------------------------------------ */

static inline float dot_fma(const float *a, const float *b, int d) {
    float acc = 0.0f;
    for (int i = 0; i < d; ++i) acc = fmaf(a[i], b[i], acc);
    return acc;
}

/* Truncate a non-negative float to Q64.64 fixed point. */
static inline u128 fx_of(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if (bits & 0x80000000u) return 0; /* negative or -0: treated as 0 */
    uint32_t ex = (bits >> 23) & 0xffu;
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
        if (sh > 103) sh = 103; /* saturate absurdly large inputs */
        return ((u128)mant) << sh;
    }
    if (sh <= -32) return 0;
    return (u128)(mant >> (-sh));
}

static inline float fx_to_float(u128 s) {
    uint64_t hi = (uint64_t)(s >> 64);
    uint64_t lo = (uint64_t)s;
    double d = (double)hi + ((double)lo) * 0x1p-64;
    return (float)d;
}

static inline double fx_to_double(u128 s) {
    uint64_t hi = (uint64_t)(s >> 64);
    uint64_t lo = (uint64_t)s;
    return (double)hi + ((double)lo) * 0x1p-64;
}

/* ------------------------------------------------------------------ */
/* exported helpers                                                    */
/* ------------------------------------------------------------------ */

float or_fx_sum(const float *v, int64_t n) {
    u128 s = 0;
    for (int64_t i = 0; i < n; ++i) s += fx_of(v[i]);
    return fx_to_float(s);
}

/* Inclusive prefix sums under the fixed-point rule, returned as fp32. */
void or_fx_cumsum(const float *v, int64_t n, float *out) {
    u128 s = 0;
    for (int64_t i = 0; i < n; ++i) {
        s += fx_of(v[i]);
        out[i] = fx_to_float(s);
    }
}

void or_sqnorm(const float *x, int64_t n, int d, float *out) {
    for (int64_t i = 0; i < n; ++i) out[i] = dot_fma(x + i * d, x + i * d, d);
}

static inline float dist2_def(float xx, float cc, float dt) {
    float s = xx + cc;
    float r = s - 2.0f * dt; /* 2*dt is exact; one rounding */
    return r > 0.0f ? r : 0.0f;
}

/* C[i][j] = dot(A_i, B_j) for A[na,d] and B given transposed, BT[d][nb].
 * Each dot is the sequential fmaf chain over d; the loop over j is SIMD. */
static void dots_bt(const float *A, int64_t na, const float *BT, int64_t nb, int d,
                    float *C) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < na; ++i) {
        float *ci = C + i * nb;
        const float *ai = A + i * d;
        for (int64_t j = 0; j < nb; ++j) ci[j] = 0.0f;
        for (int t = 0; t < d; ++t) {
            const float a = ai[t];
            const float *bt = BT + (int64_t)t * nb;
            for (int64_t j = 0; j < nb; ++j) ci[j] = fmaf(a, bt[j], ci[j]);
        }
    }
}

static float *transpose(const float *x, int64_t n, int d) {
    float *t = (float *)malloc(sizeof(float) * (size_t)n * d);
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < d; ++j) t[(int64_t)j * n + i] = x[i * d + j];
    return t;
}

/* Nearest centre for each row; ties resolve to the lowest centre index.
 * minimum distances in mind[n]; returns the fixed-point inertia as fp32. */
float or_assign(const float *x, const float *xx, int64_t n, const float *c,
                const float *cc, int k, int d, int32_t *labels, float *mind) {
    float *cT = transpose(c, k, d);
    float *md = mind ? mind : (float *)malloc(sizeof(float) * n);
    const int64_t CH = 256;
#pragma omp parallel for schedule(dynamic)
    for (int64_t i0 = 0; i0 < n; i0 += CH) {
        int64_t m = (n - i0) < CH ? (n - i0) : CH;
        float *dots = (float *)malloc(sizeof(float) * (size_t)m * k);
        for (int64_t i = 0; i < m; ++i) {
            const float *ai = x + (i0 + i) * d;
            float *ci = dots + i * k;
            for (int j = 0; j < k; ++j) ci[j] = 0.0f;
            for (int t = 0; t < d; ++t) {
                const float a = ai[t];
                const float *bt = cT + (int64_t)t * k;
                for (int j = 0; j < k; ++j) ci[j] = fmaf(a, bt[j], ci[j]);
            }
            float best = INFINITY;
            int bl = 0;
            for (int j = 0; j < k; ++j) {
                float v = dist2_def(xx[i0 + i], cc[j], ci[j]);
                if (v < best) {
                    best = v;
                    bl = j;
                }
            }
            labels[i0 + i] = bl;
            md[i0 + i] = best;
        }
        free(dots);
    }
    u128 s = 0;
    for (int64_t i = 0; i < n; ++i) s += fx_of(md[i]);
    if (!mind) free(md);
    free(cT);
    return fx_to_float(s);
}

/* Greedy k-means++ (minibatch_kmeans.py:73-126).  The random draws do not
 * depend on the data, so the caller passes them in: first_id and
 * uniforms[(k-1)*trials] in the order the reference draws them. */
void or_kmeans_pp(const float *x, int64_t n, int d, int k, int trials,
                  int64_t first_id, const double *uniforms, float *centers,
                  int64_t *chosen_ids) {
    float *xx = (float *)malloc(sizeof(float) * n);
    float *closest = (float *)malloc(sizeof(float) * n);
    float *cum = (float *)malloc(sizeof(float) * n);
    float *cand = (float *)malloc(sizeof(float) * (size_t)trials * n);
    int64_t *cid = (int64_t *)malloc(sizeof(int64_t) * trials);
    float *pot = (float *)malloc(sizeof(float) * trials);
    or_sqnorm(x, n, d, xx);

    memcpy(centers, x + first_id * d, sizeof(float) * d);
    if (chosen_ids) chosen_ids[0] = first_id;
    float c0 = xx[first_id];
    u128 s = 0;
    for (int64_t i = 0; i < n; ++i) {
        closest[i] = dist2_def(xx[i], c0, dot_fma(x + i * d, centers, d));
        s += fx_of(closest[i]);
    }
    float potential = fx_to_float(s);

    float *xT = transpose(x, n, d);
    float *cp = (float *)malloc(sizeof(float) * (size_t)trials * d);
    for (int ci = 1; ci < k; ++ci) {
        or_fx_cumsum(closest, n, cum);
        for (int t = 0; t < trials; ++t) {
            double val = uniforms[(int64_t)(ci - 1) * trials + t] * (double)potential;
            /* searchsorted(side="left") compares in fp64 */
            int64_t lo = 0, hi = n;
            while (lo < hi) {
                int64_t mid = lo + (hi - lo) / 2;
                if ((double)cum[mid] < val) lo = mid + 1;
                else hi = mid;
            }
            if (lo > n - 1) lo = n - 1;
            cid[t] = lo;
            memcpy(cp + (int64_t)t * d, x + lo * d, sizeof(float) * d);
        }
        dots_bt(cp, trials, xT, n, d, cand);
        for (int t = 0; t < trials; ++t) {
            float cc = xx[cid[t]];
            float *row = cand + (int64_t)t * n;
            u128 ps = 0;
            for (int64_t i = 0; i < n; ++i) {
                float v = dist2_def(cc, xx[i], row[i]);
                if (closest[i] < v) v = closest[i];
                row[i] = v;
                ps += fx_of(v);
            }
            pot[t] = fx_to_float(ps);
        }
        int best = 0;
        for (int t = 1; t < trials; ++t)
            if (pot[t] < pot[best]) best = t;
        memcpy(centers + (int64_t)ci * d, x + cid[best] * d, sizeof(float) * d);
        if (chosen_ids) chosen_ids[ci] = cid[best];
        memcpy(closest, cand + (int64_t)best * n, sizeof(float) * n);
        potential = pot[best];
    }
    free(xT); free(cp);
    free(xx); free(closest); free(cum); free(cand); free(cid); free(pot);
}

/* Mini-batch centre update (minibatch_kmeans.py:226-239): batch counts,
 * index_add_ sums in batch order, then
 *   new = (c * n + sum) / (n + bc)   for clusters present in the batch.
 * counts is updated in place; centers_new receives the new centres. */
void or_minibatch_update(const float *xb, const int32_t *labels, int64_t nb,
                         int d, int k, const float *centers, float *counts,
                         float *centers_new, float *batch_counts_out) {
    float *bsum = (float *)calloc((size_t)k * d, sizeof(float));
    float *bc = (float *)calloc((size_t)k, sizeof(float));
    for (int64_t i = 0; i < nb; ++i) {
        int g = labels[i];
        bc[g] += 1.0f;
        float *dst = bsum + (int64_t)g * d;
        const float *src = xb + i * d;
        for (int j = 0; j < d; ++j) dst[j] = dst[j] + src[j];
    }
    for (int g = 0; g < k; ++g) {
        float nc = counts[g] + bc[g];
        const float *cg = centers + (int64_t)g * d;
        float *og = centers_new + (int64_t)g * d;
        if (bc[g] > 0.0f) {
            for (int j = 0; j < d; ++j) {
                float a = cg[j] * counts[g];
                float b = a + bsum[(int64_t)g * d + j];
                og[j] = b / nc;
            }
        } else {
            memcpy(og, cg, sizeof(float) * d);
        }
        counts[g] = nc;
        if (batch_counts_out) batch_counts_out[g] = bc[g];
    }
    free(bsum);
    free(bc);
}

/* Cluster-summary centroids (santapp.py:526-533): sequential fp32 sums of
 * member rows in ascending row order, divided by the member count.
 * keys[n,d] fp32, labels[n] in [0,k); out[k,d] (rows of empty clusters are 0). */
void or_cluster_means(const float *keys, const int32_t *labels, int64_t n, int d,
                      int k, float *out, int64_t *counts) {
    memset(out, 0, sizeof(float) * (size_t)k * d);
    memset(counts, 0, sizeof(int64_t) * (size_t)k);
    for (int64_t i = 0; i < n; ++i) {
        int g = labels[i];
        counts[g] += 1;
        float *dst = out + (int64_t)g * d;
        const float *src = keys + i * d;
        for (int j = 0; j < d; ++j) dst[j] = dst[j] + src[j];
    }
    for (int g = 0; g < k; ++g) {
        if (!counts[g]) continue;
        float nf = (float)counts[g];
        for (int j = 0; j < d; ++j) out[(int64_t)g * d + j] = out[(int64_t)g * d + j] / nf;
    }
}

/* Key fingerprints (santapp.py:672-683): out[i][h*P + p] =
 * fl32(dot(keys_i, q_h[probes[p]]) / divisor), q_h at q + h * q_stride. */
void or_fingerprints(const float *keys, int64_t n, int d, const float *q, int64_t q_stride,
                     int g, const int64_t *probes, int P, float divisor, float *out) {
    const int cols = g * P;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        for (int c = 0; c < cols; ++c) {
            const int h = c / P, p = c % P;
            const float dt = dot_fma(keys + i * d, q + (int64_t)h * q_stride + probes[p] * d, d);
            out[i * cols + c] = dt / divisor;
        }
}

/* Column z-score (santapp.py:684-691) with exact sums: mean = fl32(fl64(S)/n)
 * of the exact signed fixed-point column sum S; var likewise over
 * fl32(fl32(x - mean)^2); z = fl32(fl32(x - mean) / fl32(sqrt(var) + 1e-6)). */
void or_zscore(float *f, int64_t n, int cols) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < cols; ++c) {
        u128 s = 0;
        for (int64_t i = 0; i < n; ++i) {
            const float x = f[i * cols + c];
            const u128 m = fx_of(fabsf(x));
            s += (x < 0.0f) ? (u128)0 - m : m;
        }
        int neg = (int)(s >> 127);
        u128 mag = neg ? (u128)0 - s : s;
        double sd = fx_to_double(mag);
        if (neg) sd = -sd;
        const float mean = (float)(sd / (double)n);
        u128 q = 0;
        for (int64_t i = 0; i < n; ++i) {
            const float dv = f[i * cols + c] - mean;
            q += fx_of(dv * dv);
        }
        const float var = (float)(fx_to_double(q) / (double)n);
        const float den = sqrtf(var) + 1e-6f;
        for (int64_t i = 0; i < n; ++i) f[i * cols + c] = (f[i * cols + c] - mean) / den;
    }
}

/* guess_g = fl32(log_n[g] + fl32(dot(c_g, q) * scale)) for G centroids. */
void or_centroid_guess(const float *cent, const float *log_n, int G, int d,
                       const float *q, float scale, float *out) {
    for (int g = 0; g < G; ++g) {
        float dt = dot_fma(cent + (int64_t)g * d, q, d);
        float sc = dt * scale;
        out[g] = log_n[g] + sc;
    }
}

/* Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw,
 * "Parallel random numbers: as easy as 1, 2, 3", SC'11).  One call maps a
 * 128-bit counter and 64-bit key to four 32-bit words. */
void or_philox4x32(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}
