/*
 * gat_oracle.c -- CPU restatement of the reference GAT forward (checker only).
 *
 * TEST INFRASTRUCTURE: loaded by tests/, __graft_entry__.smoke() and the
 * CPU legs of bench.py only. Never linked into libgat_b200.so.
 *
 * Parity with the reference is pinned by tests/test_oracle_golden.py against
 * vectors produced by the reference's own sources (tests/golden/make_golden.py).
 * Build: see oracle/Makefile (-O2 -ffp-contract=off -fopenmp). Parallel loops
 * only split independent destination rows, so results do not depend on the
 * thread count.
 */
#include "gat_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float leak(float v) { return v >= 0.f ? v : 0.2f * v; } /* gat.hpp:52 */
static inline float elu(float v) { return v >= 0.f ? v : expm1f(v); }  /* gat.hpp:53 */

uint16_t oracle_rne(float x) { /* common.cpp:80-83 */
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x7fffffu)) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float oracle_expand(uint16_t b) { /* common.cpp:84 */
    uint32_t u = (uint32_t)b << 16;
    float x;
    memcpy(&x, &u, 4);
    return x;
}

void oracle_quantize(const float* in, float* out, uint64_t count) { /* common.cpp:94-96 */
    for (uint64_t i = 0; i < count; ++i) out[i] = oracle_expand(oracle_rne(in[i]));
}

static int cmp_u64(const void* a, const void* b) {
    uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? -1 : x > y ? 1 : 0;
}

uint64_t oracle_degree_schedule(uint64_t n, const uint64_t* row, uint32_t* perm) {
    /* common.cpp:121-123: comparator (degree, row id) ascending == sort of the
     * packed key degree<<32 | row (degrees and ids are < 2^32 here). */
    uint64_t* key = (uint64_t*)malloc(n * sizeof(uint64_t));
    for (uint64_t i = 0; i < n; ++i) key[i] = ((row[i + 1] - row[i]) << 32) | i;
    qsort(key, n, sizeof(uint64_t), cmp_u64);
    for (uint64_t i = 0; i < n; ++i) perm[i] = (uint32_t)(key[i] & 0xffffffffu);
    free(key);
    uint64_t steps = 0;
    for (uint64_t base = 0; base < n; base += 16) {
        uint64_t last = base + 16 < n ? base + 16 : n;
        uint32_t r = perm[last - 1];
        steps += row[r + 1] - row[r];
    }
    return steps;
}

/* Z = X W with FP32 accumulation in ascending k (stands in for cblas_sgemm,
 * ref_fp32.cpp:5 / baseline_standard.cpp:4-5). */
static void project(uint64_t n, int in, int width, const float* x, const float* w, float* z) {
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        float* zr = z + (size_t)i * width;
        for (int c = 0; c < width; ++c) zr[c] = 0.f;
        for (int k = 0; k < in; ++k) {
            float xv = x[(size_t)i * in + k];
            const float* wr = w + (size_t)k * width;
            for (int c = 0; c < width; ++c) zr[c] += xv * wr[c];
        }
    }
}

/* baseline_standard.cpp:7-20 with scalar=true */
static void lr_scalar(uint64_t n, int heads, int dim, const float* z, const float* al,
                      const float* ar, float* left, float* right) {
    int width = heads * dim;
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (int h = 0; h < heads; ++h) {
            const float* zr = z + (size_t)i * width + h * dim;
            float l = 0.f, r = 0.f;
            for (int d = 0; d < dim; ++d) {
                l += zr[d] * al[h * dim + d];
                r += zr[d] * ar[h * dim + d];
            }
            left[(size_t)i * heads + h] = l;
            right[(size_t)i * heads + h] = r;
        }
}

void oracle_ref_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                      int in, int heads, int dim, const float* x, const float* w,
                      const float* al, const float* ar, int hidden,
                      float* z_out, float* left_out, float* right_out, float* max_out,
                      float* den_out, float* p_edge, float* out) {
    const int width = heads * dim;
    float* z = z_out ? z_out : (float*)malloc((size_t)n * width * sizeof(float));
    float* left = left_out ? left_out : (float*)malloc((size_t)n * heads * sizeof(float));
    float* right = right_out ? right_out : (float*)malloc((size_t)n * heads * sizeof(float));
    project(n, in, width, x, w, z);                 /* ref_fp32.cpp:5 */
    lr_scalar(n, heads, dim, z, al, ar, left, right); /* ref_fp32.cpp:6 */
    #pragma omp parallel
    {
        size_t cap = 0;
        float* score = NULL;
        float* alpha = NULL;
        #pragma omp for schedule(dynamic, 64)
        for (long long i = 0; i < (long long)n; ++i) {
            uint64_t b = row[i], e = row[i + 1], deg = e - b;
            if (deg > cap) {
                free(score); free(alpha);
                cap = deg;
                score = (float*)malloc(cap * sizeof(float));
                alpha = (float*)malloc(cap * sizeof(float));
            }
            float* o = out + (size_t)i * width;
            for (int c = 0; c < width; ++c) o[c] = 0.f; /* ref_fp32.cpp:18 */
            for (int h = 0; h < heads; ++h) {       /* ref_fp32.cpp:8-17 */
                float m = -INFINITY;
                float li = left[(size_t)i * heads + h];
                for (uint64_t k = 0; k < deg; ++k) {
                    float s = leak(li + right[(size_t)col[b + k] * heads + h]);
                    score[k] = s;
                    m = s > m ? s : m;
                }
                if (max_out) max_out[(size_t)i * heads + h] = deg == 0 ? 0.f : m;
                float den = 0.f;
                for (uint64_t k = 0; k < deg; ++k) {
                    float v = expf(score[k] - m);
                    if (p_edge) p_edge[(b + k) * heads + h] = v;
                    score[k] = v;
                    den += v;
                }
                if (den_out) den_out[(size_t)i * heads + h] = den;
                for (uint64_t k = 0; k < deg; ++k) alpha[k] = score[k] / den;
                /* ref_fp32.cpp:19-22 iterate edge-major; per output element the
                 * accumulation runs over edges in CSR order, as here. */
                for (uint64_t k = 0; k < deg; ++k) {
                    const float* zr = z + (size_t)col[b + k] * width + h * dim;
                    float a = alpha[k];
                    for (int d = 0; d < dim; ++d) o[h * dim + d] += a * zr[d];
                }
            }
            if (hidden)
                for (int c = 0; c < width; ++c) o[c] = elu(o[c]); /* ref_fp32.cpp:24 */
        }
        free(score); free(alpha);
    }
    if (!z_out) free(z);
    if (!left_out) free(left);
    if (!right_out) free(right);
}

void oracle_fp64_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                       int in, int heads, int dim, const float* x, const float* w,
                       const float* al, const float* ar, float* out) {
    /* boundaries.cpp:15-21 */
    const int width = heads * dim;
    double* z = (double*)calloc((size_t)n * width, sizeof(double));
    double* l = (double*)calloc((size_t)n * heads, sizeof(double));
    double* r = (double*)calloc((size_t)n * heads, sizeof(double));
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (int h = 0; h < heads; ++h)
            for (int d = 0; d < dim; ++d) {
                double v = 0;
                for (int k = 0; k < in; ++k) v += (double)x[(size_t)i * in + k] * w[(size_t)k * width + h * dim + d];
                z[(size_t)i * width + h * dim + d] = v;
                l[(size_t)i * heads + h] += v * al[h * dim + d];
                r[(size_t)i * heads + h] += v * ar[h * dim + d];
            }
    #pragma omp parallel
    {
        size_t cap = 0;
        double* sc = NULL;
        #pragma omp for schedule(dynamic, 16)
        for (long long i = 0; i < (long long)n; ++i) {
            uint64_t b = row[i], e = row[i + 1], deg = e - b;
            if (deg > cap) { free(sc); cap = deg; sc = (double*)malloc(cap * sizeof(double)); }
            for (int h = 0; h < heads; ++h) {
                double m = -INFINITY, den = 0;
                for (uint64_t k = 0; k < deg; ++k) {
                    double v = l[(size_t)i * heads + h] + r[(size_t)col[b + k] * heads + h];
                    v = v >= 0 ? v : .2 * v;
                    sc[k] = v;
                    m = v > m ? v : m;
                }
                for (uint64_t k = 0; k < deg; ++k) { sc[k] = exp(sc[k] - m); den += sc[k]; }
                for (int d = 0; d < dim; ++d) {
                    double sum = 0;
                    for (uint64_t k = 0; k < deg; ++k) sum += sc[k] * z[(size_t)col[b + k] * width + h * dim + d];
                    out[(size_t)i * width + h * dim + d] = den > 0 ? (float)(sum / den) : 0.f;
                }
            }
        }
        free(sc);
    }
    free(z); free(l); free(r);
}

void oracle_online_counters(uint64_t n, const uint64_t* row, const uint32_t* col, const uint32_t* perm,
                            int heads, const float* left, const float* right, int block,
                            uint64_t* row_blocks, uint64_t* row_updates, uint64_t* row_rescales,
                            uint64_t* totals) {
    uint64_t t_blocks = 0, t_updates = 0, t_rescales = 0, t_events = 0, t_steps = 0;
    for (int h = 0; h < heads; ++h)
        for (uint64_t base = 0; base < n; base += 16) {
            const int batch = (int)(n - base < 16 ? n - base : 16);
            uint32_t rows[16];
            uint64_t deg[16], maxdeg = 0;
            float run[16];
            int seen[16];
            for (int k = 0; k < batch; ++k) {
                rows[k] = perm[base + k];
                deg[k] = row[rows[k] + 1] - row[rows[k]];
                maxdeg = deg[k] > maxdeg ? deg[k] : maxdeg;
                run[k] = -INFINITY;
                seen[k] = 0;
                const size_t idx = (size_t)rows[k] * heads + h;
                if (row_blocks) row_blocks[idx] = 0;
                if (row_updates) row_updates[idx] = 0;
                if (row_rescales) row_rescales[idx] = 0;
            }
            t_steps += maxdeg;
            for (uint64_t begin = 0; begin < maxdeg; begin += (uint64_t)block) {
                int changed = 0;
                for (int k = 0; k < batch; ++k) {
                    if (begin >= deg[k]) continue;
                    const size_t idx = (size_t)rows[k] * heads + h;
                    const float l = left[idx];
                    uint64_t end = begin + (uint64_t)block;
                    end = end < deg[k] ? end : deg[k];
                    float bm = -INFINITY;
                    for (uint64_t s = begin; s < end; ++s) {
                        const float sc = leak(l + right[(size_t)col[row[rows[k]] + s] * heads + h]);
                        bm = sc > bm ? sc : bm;
                    }
                    const float prev = run[k];
                    run[k] = bm > run[k] ? bm : run[k];
                    const int update = run[k] > prev;
                    const int rescale = update && seen[k];  /* den > 0 once a block was taken */
                    seen[k] = 1;
                    ++t_blocks;
                    t_updates += (uint64_t)update;
                    t_rescales += (uint64_t)rescale;
                    changed |= rescale;
                    if (row_blocks) ++row_blocks[idx];
                    if (row_updates) row_updates[idx] += (uint64_t)update;
                    if (row_rescales) row_rescales[idx] += (uint64_t)rescale;
                }
                t_events += (uint64_t)changed;
            }
        }
    totals[0] = t_blocks;
    totals[1] = t_updates;
    totals[2] = t_rescales;
    totals[3] = t_events;
    totals[4] = t_steps;  /* summed over heads, as the reference counts them */
}

void oracle_max_prescan(uint64_t n, const uint64_t* row, const uint32_t* col, int heads,
                        const float* left, const float* right, float* max) {
    /* baseline_standard.cpp:44-51: m = leaky(L + max_j R_j); 0 for empty rows. */
    #pragma omp parallel for schedule(dynamic, 64)
    for (long long i = 0; i < (long long)n; ++i)
        for (int h = 0; h < heads; ++h) {
            float mr = -INFINITY;
            for (uint64_t e = row[i]; e < row[i + 1]; ++e) {
                float v = right[(size_t)col[e] * heads + h];
                mr = v > mr ? v : mr;
            }
            max[(size_t)i * heads + h] = row[i] == row[i + 1] ? 0.f : leak(mr + left[(size_t)i * heads + h]);
        }
}

void oracle_standard_aggregate(uint64_t n, const uint64_t* row, const uint32_t* col,
                               int heads, int dim, const float* z, const float* left,
                               const float* right, const float* max,
                               const float* fixed_p, const float* fixed_den,
                               float* out, float* den_out) {
    /* baseline_standard.cpp:52-84 */
    const int width = heads * dim;
    #pragma omp parallel for schedule(dynamic, 64)
    for (long long i = 0; i < (long long)n; ++i) {
        float acc[8 * 64];
        float den[8];
        for (int c = 0; c < width; ++c) acc[c] = 0.f;
        for (int h = 0; h < heads; ++h) den[h] = 0.f;
        for (uint64_t e = row[i]; e < row[i + 1]; ++e) {
            const float* zr = z + (size_t)col[e] * width;
            for (int h = 0; h < heads; ++h) {
                float wgt = fixed_p ? fixed_p[e * heads + h]
                                    : expf(leak(left[(size_t)i * heads + h] + right[(size_t)col[e] * heads + h]) -
                                           max[(size_t)i * heads + h]);
                den[h] += wgt;
                for (int d = 0; d < dim; ++d) acc[h * dim + d] += wgt * zr[h * dim + d];
            }
        }
        for (int h = 0; h < heads; ++h) den_out[(size_t)i * heads + h] = fixed_den ? fixed_den[(size_t)i * heads + h] : den[h];
        for (int c = 0; c < width; ++c) out[(size_t)i * width + c] = acc[c];
    }
}

/* V[c] += sum_k a[k] * wq[k][h*dim+c] for one neighbour step (or one block):
 * sequential FP32 over k, the accumulation order of AMX tdpbf16ps; the
 * products of two BF16 values are exact in FP32. */
static void tfs_accumulate(int in, int width, int h, int dim, const float* a, const float* wq, float* v) {
    for (int c = 0; c < dim; ++c) {
        float acc = v[c];
        for (int k = 0; k < in; ++k) acc = acc + a[k] * wq[(size_t)k * width + h * dim + c];
        v[c] = acc;
    }
}

void oracle_tfs_aggregate(uint64_t n, const uint64_t* row, const uint32_t* col, int in, int heads, int dim,
                          const float* xq, const float* wq, const float* left, const float* right,
                          const float* max_in, const float* fixed_p, const float* fixed_den, int rounding,
                          int block, int threshold, float* out, float* den_out, float* max_out) {
    const int width = heads * dim;
    #pragma omp parallel for schedule(dynamic, 16)
    for (long long i = 0; i < (long long)n; ++i) {
        const uint64_t beg = row[i], deg = row[i + 1] - row[i];
        const uint64_t B = block > 0 ? (uint64_t)block : (deg ? deg : 1);
        float* hb = (float*)malloc((size_t)in * sizeof(float));
        float* u = (float*)malloc((size_t)in * sizeof(float));
        float* p = (float*)malloc((size_t)B * sizeof(float));
        for (int h = 0; h < heads; ++h) {
            const float L = left ? left[(size_t)i * heads + h] : 0.f;
            float v[64];
            for (int c = 0; c < dim; ++c) v[c] = 0.f;
            float den = 0.f, m = -INFINITY;
            for (uint64_t b0 = 0; b0 < deg; b0 += B) {
                const uint64_t cnt = deg - b0 < B ? deg - b0 : B;
                /* weights of the block */
                if (fixed_p) {
                    for (uint64_t b = 0; b < cnt; ++b) p[b] = fixed_p[(beg + b0 + b) * heads + h];
                } else if (max_in) { /* baseline_tfs.cpp:55-57: exp(leaky(L+R) - prescan max) */
                    const float mx = max_in[(size_t)i * heads + h];
                    for (uint64_t b = 0; b < cnt; ++b)
                        p[b] = expf(leak(L + right[(size_t)col[beg + b0 + b] * heads + h]) - mx);
                    m = mx;
                } else { /* icpp_online.cpp:75-135: block max, running max, rescale */
                    float bm = -INFINITY;
                    for (uint64_t b = 0; b < cnt; ++b) {
                        p[b] = leak(L + right[(size_t)col[beg + b0 + b] * heads + h]);
                        bm = p[b] > bm ? p[b] : bm;
                    }
                    const float prev = m;
                    m = bm > m ? bm : m;
                    const int changed = m > prev && den > 0.f;
                    const float r = expf(changed ? prev - m : 0.f);
                    den = den * r;
                    for (uint64_t b = 0; b < cnt; ++b) p[b] = expf(p[b] - m);
                    if (changed)
                        for (int c = 0; c < dim; ++c) v[c] = v[c] * r;
                }
                for (uint64_t b = 0; b < cnt; ++b) den = den + p[b];
                if (rounding == 0) { /* baseline_tfs.cpp:60-84: V += RNE(p*x) . W per neighbour */
                    for (uint64_t b = 0; b < cnt; ++b) {
                        const float* xr = xq + (size_t)col[beg + b0 + b] * in;
                        for (int k = 0; k < in; ++k) hb[k] = oracle_expand(oracle_rne(xr[k] * p[b]));
                        tfs_accumulate(in, width, h, dim, hb, wq, v);
                    }
                } else {
                    for (int k = 0; k < in; ++k) u[k] = 0.f;
                    if (rounding == 1 || (int64_t)cnt < (int64_t)threshold) {
                        /* icpp_block.cpp:151-178: FP32 FMA chain over the block */
                        for (int k = 0; k < in; ++k) {
                            float acc = 0.f;
                            for (uint64_t b = 0; b < cnt; ++b)
                                acc = fmaf(p[b], xq[(size_t)col[beg + b0 + b] * in + k], acc);
                            u[k] = acc;
                        }
                    } else {
                        /* icpp_heads_hybrid.cpp:186-214: p = hi + lo (two BF16), hi pass then lo pass */
                        for (int k = 0; k < in; ++k) {
                            float acc = 0.f;
                            for (uint64_t b = 0; b < cnt; ++b) {
                                const float hi = oracle_expand(oracle_rne(p[b]));
                                acc = acc + hi * xq[(size_t)col[beg + b0 + b] * in + k];
                            }
                            for (uint64_t b = 0; b < cnt; ++b) {
                                const float hi = oracle_expand(oracle_rne(p[b]));
                                const float lo = oracle_expand(oracle_rne(p[b] - hi));
                                acc = acc + lo * xq[(size_t)col[beg + b0 + b] * in + k];
                            }
                            u[k] = acc;
                        }
                    }
                    for (int k = 0; k < in; ++k) hb[k] = oracle_expand(oracle_rne(u[k])); /* icpp_block.cpp:185-188 */
                    tfs_accumulate(in, width, h, dim, hb, wq, v);
                }
            }
            for (int c = 0; c < dim; ++c) out[(size_t)i * width + h * dim + c] = v[c];
            den_out[(size_t)i * heads + h] = fixed_den ? fixed_den[(size_t)i * heads + h] : den;
            if (max_out) max_out[(size_t)i * heads + h] = m;
        }
        free(hb); free(u); free(p);
    }
}

void oracle_prepare_blr(int in, int heads, int dim, const float* w, const float* al, const float* ar,
                        float* blr) {
    /* common.cpp:100-106 */
    const int width = heads * dim;
    for (int k = 0; k < in; ++k)
        for (int h = 0; h < heads; ++h) {
            float l = 0.f, r = 0.f;
            for (int d = 0; d < dim; ++d) {
                const float wv = w[(size_t)k * width + h * dim + d];
                l = fmaf(wv, al[h * dim + d], l);
                r = fmaf(wv, ar[h * dim + d], r);
            }
            blr[(size_t)k * 2 * heads + h] = l;
            blr[(size_t)k * 2 * heads + heads + h] = r;
        }
}

void oracle_lr_reordered(uint64_t n, int in, int heads, const float* x, const float* xq, const float* blr,
                         int policy, float* left, float* right) {
    /* baseline_standard.cpp:29-43 */
    const int cols = 2 * heads;
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (int c = 0; c < cols; ++c) {
            float acc = 0.f;
            for (int k = 0; k < in; ++k) {
                const float b = blr[(size_t)k * cols + c];
                acc = policy == 0 ? fmaf(xq[(size_t)i * in + k], oracle_expand(oracle_rne(b)), acc)
                                  : fmaf(x[(size_t)i * in + k], b, acc);
            }
            if (c < heads) left[(size_t)i * heads + c] = acc;
            else right[(size_t)i * heads + c - heads] = acc;
        }
}

void oracle_finish(uint64_t n, int heads, int dim, const float* den, int hidden, float* out) {
    /* baseline_standard.cpp:85-97; activation() (gat.hpp:57-62) is exp(x)-1 for x<0. */
    const int width = heads * dim;
    #pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (int h = 0; h < heads; ++h) {
            float d = den[(size_t)i * heads + h];
            float scale = d > 0 ? 1.f / d : 0.f;
            for (int c = 0; c < dim; ++c) {
                float v = out[(size_t)i * width + h * dim + c] * scale;
                if (hidden && v < 0) v = expf(v) - 1.f;
                out[(size_t)i * width + h * dim + c] = v;
            }
        }
}

void oracle_b0_layer(uint64_t n, const uint64_t* row, const uint32_t* col,
                     int in, int heads, int dim, const float* x, const float* w,
                     const float* al, const float* ar, int hidden, int bf16, int round_z,
                     float* z_out, float* left_out, float* right_out, float* max_out,
                     float* den_out, float* out) {
    const int width = heads * dim;
    float* z = z_out ? z_out : (float*)malloc((size_t)n * width * sizeof(float));
    float* left = left_out ? left_out : (float*)malloc((size_t)n * heads * sizeof(float));
    float* right = right_out ? right_out : (float*)malloc((size_t)n * heads * sizeof(float));
    float* max = max_out ? max_out : (float*)malloc((size_t)n * heads * sizeof(float));
    float* den = den_out ? den_out : (float*)malloc((size_t)n * heads * sizeof(float));
    if (bf16) { /* convert (common.cpp:85-93) of X and prepare()'s BF16 W (common.cpp:99) */
        float* xq = (float*)malloc((size_t)n * in * sizeof(float));
        float* wq = (float*)malloc((size_t)in * width * sizeof(float));
        oracle_quantize(x, xq, (uint64_t)n * in);
        oracle_quantize(w, wq, (uint64_t)in * width);
        project(n, in, width, xq, wq, z);
        free(xq); free(wq);
    } else {
        project(n, in, width, x, w, z);
    }
    lr_scalar(n, heads, dim, z, al, ar, left, right);
    if (round_z) oracle_quantize(z, z, (uint64_t)n * width);
    oracle_max_prescan(n, row, col, heads, left, right, max);
    oracle_standard_aggregate(n, row, col, heads, dim, z, left, right, max, NULL, NULL, out, den);
    oracle_finish(n, heads, dim, den, hidden, out);
    if (!z_out) free(z);
    if (!left_out) free(left);
    if (!right_out) free(right);
    if (!max_out) free(max);
    if (!den_out) free(den);
}
