/*
 * moe_oracle.c -- CPU restatement of the reference MoE feed-forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product package links, loads or
 * calls this file: it is the checker that tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg compare the CUDA library against.  It is pinned
 * against golden vectors produced by the reference's own PyTorch path
 * (tests/golden/make_golden.py), so parity is "pinned", not "unpinned".
 *
 * Each function cites the reference code it restates, by path inside the
 * reference project (src/moe_dispatch/...).  Rounding points follow the
 * reference's PyTorch path (implementation="torch"):
 *   - router logits in fp32 (layer.py:123), bias added in fp32 (layer.py:136),
 *     top-k with ties to the lower expert index (csrc/dispatch.cu:327-336),
 *     softmax over the selected scores only (layer.py:137-138);
 *   - dispatch: counts, padded exclusive offsets, stable expert order of the
 *     flattened assignment p = t*K + k (reference.py:42-65 with a stable sort);
 *   - grouped GEMM accumulates in fp32 and rounds once to bf16
 *     (experts.py:21-35, _triton_gemm.py:52-70);
 *   - SwiGLU: bf16(silu(f32 gate) * f32 up) (experts.py:38-41);
 *   - combine: fp32 product w*f32(eo) rounded, then a sequential fp32 sum over
 *     k = 0..K-1, then one cast (reference.py:67-76; torch's CPU reduction
 *     over that axis is sequential).
 *
 * Router logits use a defined fp32 summation order (see oracle_router_logits)
 * which the CUDA router reproduces, so logits (and hence top-k ids) are
 * bit-exact between the two.
 *
 * Build: oracle/Makefile (gcc -O3 -mavx2 -mfma -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_BF16 = 2 };
enum { OR_OK = 0, OR_EINVAL = 1, OR_ENOMEM = 2 };

/* ---- scalar conversions (IEEE round-to-nearest-even, as torch does) ---- */

static inline float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u); /* quiet NaN */
    uint32_t rounding = ((bits >> 16) & 1u) + 0x7fffu;
    return (uint16_t)((bits + rounding) >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

static inline uint16_t f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline float load_elem(const void* base, int dtype, int64_t i) {
    if (dtype == OR_F32) return ((const float*)base)[i];
    if (dtype == OR_F16) return f16_to_f32(((const uint16_t*)base)[i]);
    return bf16_to_f32(((const uint16_t*)base)[i]);
}

static inline void store_elem(void* base, int dtype, int64_t i, float v) {
    if (dtype == OR_F32) ((float*)base)[i] = v;
    else if (dtype == OR_F16) ((uint16_t*)base)[i] = f32_to_f16(v);
    else ((uint16_t*)base)[i] = f32_to_bf16(v);
}

static inline int elem_bytes(int dtype) { return dtype == OR_F32 ? 4 : 2; }

/* Exported so tests can check the conversion helpers against torch. */
uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
uint16_t oracle_f32_to_f16(float f) { return f32_to_f16(f); }

/* ---- router: layer.py:123 (F.linear(x.float(), router_weight)) ----
 *
 * The fp32 summation order is part of the definition, so that the CUDA router
 * reproduces every logit bit for bit:
 *   experts <= 32: slice l (l = 0..31) holds the elements h with
 *     (h / 8) mod 32 == l -- runs of 8 consecutive elements, 256 apart; each
 *     slice is a sequential fmaf chain in increasing h from +0.0f; the 32
 *     partial sums are combined by a xor butterfly: for off = 16, 8, 4, 2, 1:
 *     p[l] = p[l] + p[l ^ off]; the logit is p[0] (every l ends equal).
 *   experts > 32: one sequential fmaf chain over h = 0..H-1 from +0.0f. */

#define OR_ROUTER_SLICED_MAX_EXPERTS 32

static float dot_sliced(const uint16_t* xr, const float* wr, int hidden) {
    float p[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int h0 = 8 * l; h0 < hidden; h0 += 256) {
            const int h1 = h0 + 8 < hidden ? h0 + 8 : hidden;
            for (int h = h0; h < h1; ++h) acc = fmaf(bf16_to_f32(xr[h]), wr[h], acc);
        }
        p[l] = acc;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float q[32];
        for (int l = 0; l < 32; ++l) q[l] = p[l] + p[l ^ off];
        memcpy(p, q, sizeof(p));
    }
    return p[0];
}

int oracle_router_logits(const uint16_t* x_bf16, const float* w, int64_t tokens, int hidden,
                         int experts, float* logits) {
    if (tokens < 0 || hidden < 1 || experts < 1) return OR_EINVAL;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
        const uint16_t* xr = x_bf16 + t * (int64_t)hidden;
        for (int e = 0; e < experts; ++e) {
            const float* wr = w + (int64_t)e * hidden;
            float acc = 0.0f;
            if (experts <= OR_ROUTER_SLICED_MAX_EXPERTS) {
                acc = dot_sliced(xr, wr, hidden);
            } else {
                for (int h = 0; h < hidden; ++h) acc = fmaf(bf16_to_f32(xr[h]), wr[h], acc);
            }
            logits[t * experts + e] = acc;
        }
    }
    return OR_OK;
}

/* ---- top-k + softmax: dispatch.cu:327-376 (ties -> lower index),
 *      layer.py:136-139 (bias added before selection; softmax of selected) ---- */

int oracle_topk_softmax(const float* logits, const float* bias, int64_t tokens, int experts,
                        int topk, int32_t* ids32, int64_t* ids64, float* weights) {
    if (tokens < 0 || experts < 1 || topk < 1 || topk > experts || experts > 1024) return OR_EINVAL;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
        float values[1024];
        unsigned char taken[1024];
        float chosen[64];
        for (int e = 0; e < experts; ++e) {
            values[e] = logits[t * experts + e] + (bias ? bias[e] : 0.0f);
            taken[e] = 0;
        }
        for (int k = 0; k < topk; ++k) {
            int best = -1;
            for (int e = 0; e < experts; ++e) {
                if (taken[e]) continue;
                if (best < 0 || values[e] > values[best]) best = e; /* strict '>' keeps the lower index on ties */
            }
            chosen[k] = values[best];
            ids32[t * topk + k] = best;
            if (ids64) ids64[t * topk + k] = best;
            taken[best] = 1;
        }
        /* softmax over the K selected values; chosen[0] is their maximum */
        float ex[64];
        float total = 0.0f;
        for (int k = 0; k < topk; ++k) {
            ex[k] = expf(chosen[k] - chosen[0]);
            total += ex[k];
        }
        float inv = 1.0f / total;
        for (int k = 0; k < topk; ++k) weights[t * topk + k] = ex[k] * inv;
    }
    return OR_OK;
}

/* ---- dispatch index: reference.py:42-65 (counts by scatter_add, cumsum of
 *      aligned counts, expert sort of p = t*K+k) and dispatch.cu:13-34,194-205.
 *      The sort is stable: within an expert, assignments keep their p order. ---- */

int oracle_dispatch_index(const int32_t* ids, int64_t tokens, int topk, int experts, int alignment,
                          int32_t* counts, int32_t* offsets, int32_t* slots, int32_t* inverse) {
    if (tokens < 0 || topk < 1 || experts < 1 || alignment < 1) return OR_EINVAL;
    int64_t n = tokens * topk;
    for (int e = 0; e < experts; ++e) counts[e] = 0;
    for (int64_t p = 0; p < n; ++p) {
        int e = ids[p];
        if (e >= 0 && e < experts) slots[p] = counts[e]++;
        else slots[p] = -1;
    }
    offsets[0] = 0;
    for (int e = 0; e < experts; ++e) {
        int32_t span = alignment == 1 ? counts[e] : (counts[e] + alignment - 1) / alignment * alignment;
        offsets[e + 1] = offsets[e] + span;
    }
    for (int64_t p = 0; p < n; ++p) {
        int e = ids[p];
        inverse[p] = (e >= 0 && e < experts) ? offsets[e] + slots[p] : -1;
    }
    return OR_OK;
}

/* ---- pack: dispatch.cu:36-74 (row copy) and dispatch.cu:207-216 (zeroed padding) ---- */

int oracle_pack(const void* x, int dtype, const int32_t* inverse, const int32_t* counts,
                const int32_t* offsets, int64_t tokens, int topk, int experts, int64_t hidden,
                int64_t packed_rows, void* packed) {
    if (tokens < 0 || topk < 1 || hidden < 1) return OR_EINVAL;
    size_t row_bytes = (size_t)hidden * elem_bytes(dtype);
    int64_t n = tokens * topk;
    for (int64_t p = 0; p < n; ++p) {
        int32_t dest = inverse[p];
        if (dest < 0 || dest >= packed_rows) continue;
        memcpy((char*)packed + (size_t)dest * row_bytes, (const char*)x + (size_t)(p / topk) * row_bytes,
               row_bytes);
    }
    for (int e = 0; e < experts; ++e) {
        int64_t start = (int64_t)offsets[e] + counts[e], end = offsets[e + 1];
        for (int64_t r = start; r < end && r < packed_rows; ++r)
            memset((char*)packed + (size_t)r * row_bytes, 0, row_bytes);
    }
    return OR_OK;
}

/* ---- combine: reference.py:67-76 (index_select, fp32 mul, sum over k, one cast) ---- */

int oracle_combine(const void* expert_output, int dtype, const int32_t* inverse, const float* weights,
                   int64_t tokens, int topk, int64_t hidden, int64_t packed_rows, void* output) {
    if (tokens < 0 || topk < 1 || hidden < 1) return OR_EINVAL;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; ++t) {
        for (int64_t c = 0; c < hidden; ++c) {
            float acc = 0.0f;
            for (int k = 0; k < topk; ++k) {
                int64_t p = t * topk + k;
                int32_t row = inverse[p];
                if (row < 0 || row >= packed_rows) continue;
                float product = weights[p] * load_elem(expert_output, dtype, (int64_t)row * hidden + c);
                acc = acc + product;
            }
            store_elem(output, dtype, t * hidden + c, acc);
        }
    }
    return OR_OK;
}

/* ---- SwiGLU: experts.py:38-41 and dispatch.cu:277-292 (rows >= valid_rows are zero) ---- */

static inline float silu_f32(float g) { return g / (1.0f + expf(-g)); }

int oracle_swiglu(const void* projection, int dtype, int64_t rows, int64_t width, int64_t valid_rows,
                  void* output) {
    if (rows < 0 || width < 1) return OR_EINVAL;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < width; ++c) {
            float v = 0.0f;
            if (r < valid_rows) {
                float g = load_elem(projection, dtype, r * 2 * width + c);
                float u = load_elem(projection, dtype, r * 2 * width + width + c);
                v = silu_f32(g) * u;
            }
            store_elem(output, dtype, r * width + c, v);
        }
    }
    return OR_OK;
}

/* ---- grouped GEMM: experts.py:21-35 / _triton_gemm.py:37-70.
 *      For each expert e and packed row r in [offsets[e], offsets[e+1]):
 *        out[r, n] = bf16( sum_k a[r, k] * w[e, n, k] )   (fp32 accumulation)
 *      w is [E, N, K] (K contiguous), as the reference stores gate_up/down. ---- */

#define OR_NB 16

static float dot_f32(const float* a, const float* b, int64_t k) {
    float acc[16] = {0};
    int64_t i = 0;
    for (; i + 16 <= k; i += 16)
        for (int j = 0; j < 16; ++j) acc[j] = fmaf(a[i + j], b[i + j], acc[j]);
    for (; i < k; ++i) acc[i & 15] = fmaf(a[i], b[i], acc[i & 15]);
    float s = 0.0f;
    for (int j = 0; j < 16; ++j) s += acc[j];
    return s;
}

int oracle_grouped_gemm_bf16(const uint16_t* a, const uint16_t* w, const int32_t* offsets, int experts,
                             int64_t n_cols, int64_t k_dim, int64_t rows, uint16_t* out) {
    if (experts < 1 || n_cols < 1 || k_dim < 1) return OR_EINVAL;
    for (int e = 0; e < experts; ++e) {
        int64_t r0 = offsets[e], r1 = offsets[e + 1];
        if (r1 > rows) r1 = rows;
        if (r1 <= r0) continue;
        int64_t m = r1 - r0;
        float* af = (float*)malloc((size_t)m * k_dim * sizeof(float));
        if (!af) return OR_ENOMEM;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < m * k_dim; ++i) af[i] = bf16_to_f32(a[r0 * k_dim + i]);
        int64_t nblocks = (n_cols + OR_NB - 1) / OR_NB;
        int failed = 0;
#pragma omp parallel
        {
            float* wf = (float*)malloc((size_t)OR_NB * k_dim * sizeof(float));
            if (!wf) {
#pragma omp atomic write
                failed = 1;
            }
#pragma omp for schedule(dynamic, 1)
            for (int64_t nb = 0; nb < nblocks; ++nb) {
                if (!wf) continue;
                int64_t n0 = nb * OR_NB, n1 = n0 + OR_NB < n_cols ? n0 + OR_NB : n_cols;
                for (int64_t n = n0; n < n1; ++n) {
                    const uint16_t* wr = w + ((int64_t)e * n_cols + n) * k_dim;
                    for (int64_t i = 0; i < k_dim; ++i) wf[(n - n0) * k_dim + i] = bf16_to_f32(wr[i]);
                }
                for (int64_t r = 0; r < m; ++r)
                    for (int64_t n = n0; n < n1; ++n)
                        out[(r0 + r) * n_cols + n] =
                            f32_to_bf16(dot_f32(af + r * k_dim, wf + (n - n0) * k_dim, k_dim));
            }
            free(wf);
        }
        free(af);
        if (failed) return OR_ENOMEM;
    }
    return OR_OK;
}

/* ---- token-major expert evaluation: layer.py:200-214 (token_major_oracle) with
 *      the block's rounding points (projection, activation and expert output are
 *      bf16; combine as oracle_combine).  Used to check large configurations on a
 *      subset of tokens: each token's output depends only on its own row. ---- */

int oracle_moe_tokens(const uint16_t* x, const int32_t* ids, const float* weights, const uint16_t* gate_up,
                      const uint16_t* down, int64_t tokens, int hidden, int intermediate, int topk,
                      uint16_t* output) {
    if (tokens < 0 || hidden < 1 || intermediate < 1 || topk < 1) return OR_EINVAL;
    int64_t H = hidden, I = intermediate;
    int64_t work = tokens * topk;
    uint16_t* eo = (uint16_t*)malloc((size_t)(work > 0 ? work : 1) * H * sizeof(uint16_t));
    if (!eo) return OR_ENOMEM;
    int failed = 0;
#pragma omp parallel
    {
        float* xf = (float*)malloc((size_t)H * sizeof(float));
        float* act = (float*)malloc((size_t)I * sizeof(float));
        float* row = (float*)malloc((size_t)(H > I ? H : I) * sizeof(float));
        if (!xf || !act || !row) {
#pragma omp atomic write
            failed = 1;
        }
#pragma omp for schedule(dynamic, 1)
        for (int64_t p = 0; p < work; ++p) {
            if (!xf || !act || !row) continue;
            int64_t t = p / topk;
            int e = ids[p];
            for (int64_t h = 0; h < H; ++h) xf[h] = bf16_to_f32(x[t * H + h]);
            const uint16_t* wg = gate_up + (int64_t)e * 2 * I * H;
            for (int64_t c = 0; c < I; ++c) {
                for (int64_t h = 0; h < H; ++h) row[h] = bf16_to_f32(wg[c * H + h]);
                float g = bf16_to_f32(f32_to_bf16(dot_f32(xf, row, H)));
                for (int64_t h = 0; h < H; ++h) row[h] = bf16_to_f32(wg[(I + c) * H + h]);
                float u = bf16_to_f32(f32_to_bf16(dot_f32(xf, row, H)));
                act[c] = bf16_to_f32(f32_to_bf16(silu_f32(g) * u));
            }
            const uint16_t* wd = down + (int64_t)e * H * I;
            for (int64_t h = 0; h < H; ++h) {
                for (int64_t c = 0; c < I; ++c) row[c] = bf16_to_f32(wd[h * I + c]);
                eo[p * H + h] = f32_to_bf16(dot_f32(act, row, I));
            }
        }
        free(xf);
        free(act);
        free(row);
    }
    if (!failed) {
        for (int64_t t = 0; t < tokens; ++t)
            for (int64_t h = 0; h < H; ++h) {
                float acc = 0.0f;
                for (int k = 0; k < topk; ++k) {
                    int64_t p = t * topk + k;
                    float product = weights[p] * bf16_to_f32(eo[p * H + h]);
                    acc = acc + product;
                }
                output[t * H + h] = f32_to_bf16(acc);
            }
    }
    free(eo);
    return failed ? OR_ENOMEM : OR_OK;
}

/* ---- expert-parallel receive layout.  No reference counterpart (the
 *      reference is single-GPU, README.md:161-163); the layout is defined so
 *      that grouped rows equal what one GPU packs for the same experts:
 *      received rows are source-major, each source's rows expert-major; the
 *      grouped layout is expert-major (spans rounded up to `alignment`) and
 *      source-major inside an expert. ---- */

int oracle_ep_layout(const int32_t* counts, int ranks, int experts, int alignment,
                     int32_t* src_start, int32_t* dst_start, int32_t* offsets) {
    if (ranks < 1 || experts < 1 || alignment < 1) return OR_EINVAL;
    int32_t run = 0;
    for (int p = 0; p < ranks; ++p)
        for (int e = 0; e < experts; ++e) {
            src_start[p * experts + e] = run;
            run += counts[p * experts + e];
        }
    offsets[0] = 0;
    for (int e = 0; e < experts; ++e) {
        int32_t total = 0;
        for (int p = 0; p < ranks; ++p) {
            dst_start[p * experts + e] = offsets[e] + total;
            total += counts[p * experts + e];
        }
        const int32_t span = alignment > 1 ? (total + alignment - 1) / alignment * alignment : total;
        offsets[e + 1] = offsets[e] + span;
    }
    return OR_OK;
}

int oracle_ep_regroup(const void* from, int dtype, void* to, const int32_t* counts,
                      const int32_t* src_start, const int32_t* dst_start, const int32_t* offsets,
                      int ranks, int experts, int64_t hidden, int64_t grouped_rows, int grouping) {
    if (ranks < 1 || experts < 1 || hidden < 1) return OR_EINVAL;
    const size_t row_bytes = (size_t)hidden * elem_bytes(dtype);
    for (int p = 0; p < ranks; ++p)
        for (int e = 0; e < experts; ++e) {
            const int i = p * experts + e;
            for (int32_t r = 0; r < counts[i]; ++r) {
                const int64_t recv_row = (int64_t)src_start[i] + r;
                const int64_t grouped_row = (int64_t)dst_start[i] + r;
                if (grouped_row >= grouped_rows) continue;
                if (grouping)
                    memcpy((char*)to + grouped_row * row_bytes, (const char*)from + recv_row * row_bytes,
                           row_bytes);
                else
                    memcpy((char*)to + recv_row * row_bytes, (const char*)from + grouped_row * row_bytes,
                           row_bytes);
            }
        }
    if (grouping)
        for (int e = 0; e < experts; ++e) {
            int64_t filled = offsets[e];
            for (int p = 0; p < ranks; ++p) filled += counts[p * experts + e];
            for (int64_t r = filled; r < offsets[e + 1] && r < grouped_rows; ++r)
                memset((char*)to + r * row_bytes, 0, row_bytes);
        }
    return OR_OK;
}

/* ---------------------------------------------------------------- e4m3
 * The FP8 expert path has no counterpart in the reference (its experts are
 * bf16 only, layer.py:97-98); this restates the engine's own definition so the
 * GPU quantiser can be checked bit for bit.  e4m3 here is the "fn" format:
 * 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no infinities, largest
 * finite 448 (0x7E), NaN 0x7F, subnormals m * 2^-9.  Conversion rounds to
 * nearest, ties to even, and saturates finite values at +-448. */
static uint8_t f32_to_e4m3(float f) {
    const uint8_t sign = signbit(f) ? 0x80 : 0x00;
    if (isnan(f)) return 0x7F;
    const double a = fabs((double)f);
    if (a >= 448.0) return sign | 0x7E;
    if (a < 0.015625) {                       /* below 2^-6: subnormal steps of 2^-9 */
        const double m = nearbyint(a * 512.0);  /* 0..8; 8 is the smallest normal */
        return sign | (uint8_t)m;               /* m = 8 encodes exponent 1, mantissa 0 */
    }
    int e2;
    frexp(a, &e2);
    int e = e2 - 1;                           /* a in [2^e, 2^(e+1)), e in -6..8 */
    double m = nearbyint(ldexp(a, 3 - e));    /* 8..16 */
    if (m >= 16.0) {
        m = 8.0;
        e += 1;
    }
    if (e > 8 || (e == 8 && m > 14.0)) return sign | 0x7E;
    return sign | (uint8_t)(((e + 7) << 3) | ((int)m - 8));
}

uint8_t oracle_f32_to_e4m3(float f) { return f32_to_e4m3(f); }

/* Per-row e4m3 quantisation of bf16 rows (the engine's moe_quantize_rows_e4m3):
 * amax = max |x|, inv = 448 / amax (fp32 division), scale = amax / 448,
 * q = e4m3(x * inv) in fp32; an all-zero row gets scale 1 and zeros. */
int oracle_quantize_rows_e4m3(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q,
                              float* scale) {
    if (rows < 0 || cols < 0) return OR_EINVAL;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * cols;
        float amax = 0.0f;
        for (int64_t c = 0; c < cols; ++c) amax = fmaxf(amax, fabsf(bf16_to_f32(xr[c])));
        const float inv = amax > 0.0f ? 448.0f / amax : 0.0f;
        scale[r] = amax > 0.0f ? amax / 448.0f : 1.0f;
        for (int64_t c = 0; c < cols; ++c) q[r * cols + c] = f32_to_e4m3(bf16_to_f32(xr[c]) * inv);
    }
    return OR_OK;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
