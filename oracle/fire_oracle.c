/*
 * fire_oracle.c - TEST INFRASTRUCTURE ONLY (the parity oracle).
 *
 * CPU restatement of Fire's decode path; see fire_oracle.h for the rules it keeps.
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp). Never linked into
 * the fire_b200 product library.
 */
#include "fire_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void fo_set_threads(int n) { g_threads = n; }

int fo_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

float fo_bf16_to_f32(uint16_t bits) {
    /* src/op/kernels/cpu/bf16.h:8-14: BF16 is the upper half of an FP32 value. */
    uint32_t u = (uint32_t)bits << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* tools/quant.py:227-255: even k in the low nibble, w = s * (float(q) - float(z)). */
static inline float w4_value(const uint8_t* qrow, const float* srow, const uint8_t* zrow,
                             int64_t k, int group) {
    const uint8_t b = qrow[k >> 1];
    const int q = (k & 1) ? (b >> 4) : (b & 15);
    const int64_t g = k / group;
    return srow[g] * ((float)q - (float)zrow[g]);
}

void fo_dequant_int4(const uint8_t* qw, const float* scales, const uint8_t* zeros, float* w,
                     int64_t n, int64_t k, int group) {
    const int64_t groups = k / group;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
    for (int64_t r = 0; r < n; ++r) {
        const uint8_t* qrow = qw + r * (k / 2);
        const float* srow = scales + r * groups;
        const uint8_t* zrow = zeros + r * groups;
        for (int64_t c = 0; c < k; ++c) w[r * k + c] = w4_value(qrow, srow, zrow, c, group);
    }
}

/* Row-blocked forms. Each output row keeps the reference's sequential accumulation
 * order over k (sum = sum + x[k]*w[k], one rounding per operation); eight rows advance in
 * lock step in the lanes of one vector, so the results are bit-identical to the one-row
 * loops (the *_scalar functions below, kept for the test that checks exactly that). */
typedef float fo_v8 __attribute__((vector_size(32)));
enum { FO_RB = 8, FO_CB = 256 };

/* one block of up to 8 rows: tile[j][r] holds w[r0 + r][c0 + j] for a chunk of columns */
typedef void (*fo_fill_fn)(const void* ctx, int64_t r0, int nr, int64_t c0, int cn, fo_v8* tile);

static void fo_rows8(const float* xr, const void* ctx, fo_fill_fn fill, float scale, float* y,
                     int64_t r0, int nr, int64_t k) {
    fo_v8 tile[FO_CB];
    fo_v8 acc = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t c0 = 0; c0 < k; c0 += FO_CB) {
        const int cn = (int)((k - c0) < FO_CB ? (k - c0) : FO_CB);
        fill(ctx, r0, nr, c0, cn, tile);
        for (int j = 0; j < cn; ++j) {
            const fo_v8 xv = {xr[c0 + j], xr[c0 + j], xr[c0 + j], xr[c0 + j],
                              xr[c0 + j], xr[c0 + j], xr[c0 + j], xr[c0 + j]};
            acc = acc + xv * tile[j];
        }
    }
    for (int r = 0; r < nr; ++r) y[r0 + r] = scale == 1.0f ? acc[r] : acc[r] * scale;
}

static void fo_blocked(const float* x, const void* ctx, fo_fill_fn fill, float scale, float* y,
                       int64_t m, int64_t n, int64_t k) {
    const int64_t blocks = (n + FO_RB - 1) / FO_RB;
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
        float* yr = y + row * n;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t b = 0; b < blocks; ++b) {
            const int64_t r0 = b * FO_RB;
            const int nr = (int)((n - r0) < FO_RB ? (n - r0) : FO_RB);
            fo_rows8(xr, ctx, fill, scale, yr, r0, nr, k);
        }
    }
}

typedef struct { const float* w; int64_t k; } fo_f32_ctx;
static void fill_f32(const void* p, int64_t r0, int nr, int64_t c0, int cn, fo_v8* tile) {
    const fo_f32_ctx* c = (const fo_f32_ctx*)p;
    for (int r = 0; r < FO_RB; ++r) {
        const float* wr = c->w + (r0 + (r < nr ? r : 0)) * c->k + c0;
        for (int j = 0; j < cn; ++j) tile[j][r] = r < nr ? wr[j] : 0.0f;
    }
}

typedef struct { const uint16_t* w; int64_t k; } fo_bf16_ctx;
static void fill_bf16(const void* p, int64_t r0, int nr, int64_t c0, int cn, fo_v8* tile) {
    const fo_bf16_ctx* c = (const fo_bf16_ctx*)p;
    for (int r = 0; r < FO_RB; ++r) {
        const uint16_t* wr = c->w + (r0 + (r < nr ? r : 0)) * c->k + c0;
        for (int j = 0; j < cn; ++j) tile[j][r] = r < nr ? fo_bf16_to_f32(wr[j]) : 0.0f;
    }
}

typedef struct { const uint8_t* qw; const float* s; const uint8_t* z; int64_t k; int group; } fo_w4_ctx;
/* tools/quant.py:227-255 per element: s * (float(q) - float(z)), even k in the low nibble */
static void fill_w4(const void* p, int64_t r0, int nr, int64_t c0, int cn, fo_v8* tile) {
    const fo_w4_ctx* c = (const fo_w4_ctx*)p;
    const int64_t groups = c->k / c->group;
    for (int r = 0; r < FO_RB; ++r) {
        if (r >= nr) {
            for (int j = 0; j < cn; ++j) tile[j][r] = 0.0f;
            continue;
        }
        const uint8_t* qrow = c->qw + (r0 + r) * (c->k / 2);
        const float* srow = c->s + (r0 + r) * groups;
        const uint8_t* zrow = c->z + (r0 + r) * groups;
        int64_t g = c0 / c->group, gend = (g + 1) * c->group;
        float s = srow[g], zf = (float)zrow[g];
        for (int j = 0; j < cn; ++j) {
            const int64_t col = c0 + j;
            if (col == gend) {
                ++g;
                gend += c->group;
                s = srow[g];
                zf = (float)zrow[g];
            }
            const uint8_t b = qrow[col >> 1];
            const int q = (col & 1) ? (b >> 4) : (b & 15);
            tile[j][r] = s * ((float)q - zf);
        }
    }
}

/* Fast forms for the decode shapes: eight rows per vector, eight columns per step. A
 * 32-bit word of each row holds its next eight nibbles (INT4) or two BF16 values, so every
 * column becomes a lane-wise shift / mask / convert, with the same per-element arithmetic
 * and the same per-row order as above. Compiled twice: AVX2 when the host has it, else
 * the baseline vector code (identical results either way: no FMA, one rounding per op). */
typedef uint32_t fo_v8u __attribute__((vector_size(32)));
typedef int32_t fo_v8i __attribute__((vector_size(32)));

static inline uint32_t fo_ld32(const void* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}

#define FO_W4_BODY                                                                              \
    const int64_t groups = k / group;                                                           \
    fo_v8 acc = {0, 0, 0, 0, 0, 0, 0, 0};                                                       \
    const uint8_t* q[FO_RB];                                                                    \
    for (int r = 0; r < FO_RB; ++r) q[r] = qw + (r0 + (r < nr ? r : 0)) * (k / 2);               \
    for (int64_t g = 0; g < groups; ++g) {                                                      \
        fo_v8 s, zf;                                                                            \
        for (int r = 0; r < FO_RB; ++r) {                                                       \
            const int64_t rr = r0 + (r < nr ? r : 0);                                           \
            s[r] = scales[rr * groups + g];                                                     \
            zf[r] = (float)zeros[rr * groups + g];                                              \
        }                                                                                       \
        for (int64_t c = g * group; c < (g + 1) * group; c += 8) {                              \
            fo_v8u wv;                                                                          \
            for (int r = 0; r < FO_RB; ++r) wv[r] = fo_ld32(q[r] + (c >> 1));                   \
            for (int j = 0; j < 8; ++j) {                                                       \
                const fo_v8i qi = (fo_v8i)((wv >> (4u * (unsigned)j)) & 15u);                  \
                const fo_v8 w = s * (__builtin_convertvector(qi, fo_v8) - zf);                  \
                const float xs = xr[c + j];                                                     \
                const fo_v8 xv = {xs, xs, xs, xs, xs, xs, xs, xs};                              \
                acc = acc + xv * w;                                                             \
            }                                                                                   \
        }                                                                                       \
    }                                                                                           \
    for (int r = 0; r < nr; ++r) y[r0 + r] = acc[r];

#define FO_BF16_BODY                                                                            \
    fo_v8 acc = {0, 0, 0, 0, 0, 0, 0, 0};                                                       \
    const uint16_t* wp[FO_RB];                                                                  \
    for (int r = 0; r < FO_RB; ++r) wp[r] = w + (r0 + (r < nr ? r : 0)) * k;                     \
    for (int64_t c = 0; c < k; c += 2) {                                                        \
        fo_v8u wv;                                                                              \
        for (int r = 0; r < FO_RB; ++r) wv[r] = fo_ld32(wp[r] + c);                             \
        const fo_v8u lo = wv << 16u, hi = wv & 0xFFFF0000u;                                     \
        fo_v8 w0, w1;                                                                           \
        memcpy(&w0, &lo, sizeof w0);                                                            \
        memcpy(&w1, &hi, sizeof w1);                                                            \
        const fo_v8 x0 = {xr[c], xr[c], xr[c], xr[c], xr[c], xr[c], xr[c], xr[c]};              \
        const fo_v8 x1 = {xr[c + 1], xr[c + 1], xr[c + 1], xr[c + 1],                           \
                          xr[c + 1], xr[c + 1], xr[c + 1], xr[c + 1]};                          \
        acc = acc + x0 * w0;                                                                    \
        acc = acc + x1 * w1;                                                                    \
    }                                                                                           \
    for (int r = 0; r < nr; ++r) y[r0 + r] = acc[r] * scale;

__attribute__((target("avx2"))) static void w4_rows8_avx2(const float* xr, const uint8_t* qw,
                                                          const float* scales,
                                                          const uint8_t* zeros, float* y,
                                                          int64_t r0, int nr, int64_t k,
                                                          int group) {
    FO_W4_BODY
}
static void w4_rows8_base(const float* xr, const uint8_t* qw, const float* scales,
                          const uint8_t* zeros, float* y, int64_t r0, int nr, int64_t k,
                          int group) {
    FO_W4_BODY
}
__attribute__((target("avx2"))) static void bf16_rows8_avx2(const float* xr, const uint16_t* w,
                                                            float scale, float* y, int64_t r0,
                                                            int nr, int64_t k) {
    FO_BF16_BODY
}
static void bf16_rows8_base(const float* xr, const uint16_t* w, float scale, float* y,
                            int64_t r0, int nr, int64_t k) {
    FO_BF16_BODY
}

static int fo_avx2(void) {
    static int v = -1;
    if (v < 0) v = __builtin_cpu_supports("avx2") ? 1 : 0;
    return v;
}

void fo_linear_f32(const float* x, const float* w, float scale, float* y, int64_t m, int64_t n,
                   int64_t k) {
    const fo_f32_ctx c = {w, k};
    fo_blocked(x, &c, fill_f32, scale, y, m, n, k);
}

void fo_linear_bf16(const float* x, const uint16_t* w, float scale, float* y, int64_t m,
                    int64_t n, int64_t k) {
    if (k % 2) {
        const fo_bf16_ctx c = {w, k};
        fo_blocked(x, &c, fill_bf16, scale, y, m, n, k);
        return;
    }
    const int avx2 = fo_avx2();
    const int64_t blocks = (n + FO_RB - 1) / FO_RB;
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
        float* yr = y + row * n;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t b = 0; b < blocks; ++b) {
            const int64_t r0 = b * FO_RB;
            const int nr = (int)((n - r0) < FO_RB ? (n - r0) : FO_RB);
            if (avx2)
                bf16_rows8_avx2(xr, w, scale, yr, r0, nr, k);
            else
                bf16_rows8_base(xr, w, scale, yr, r0, nr, k);
        }
    }
}

void fo_linear_int4(const float* x, const uint8_t* qw, const float* scales,
                    const uint8_t* zeros, float* y, int64_t m, int64_t n, int64_t k, int group) {
    if (group % 8 || k % 8) {
        const fo_w4_ctx c = {qw, scales, zeros, k, group};
        fo_blocked(x, &c, fill_w4, 1.0f, y, m, n, k);
        return;
    }
    const int avx2 = fo_avx2();
    const int64_t blocks = (n + FO_RB - 1) / FO_RB;
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
        float* yr = y + row * n;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t b = 0; b < blocks; ++b) {
            const int64_t r0 = b * FO_RB;
            const int nr = (int)((n - r0) < FO_RB ? (n - r0) : FO_RB);
            if (avx2)
                w4_rows8_avx2(xr, qw, scales, zeros, yr, r0, nr, k, group);
            else
                w4_rows8_base(xr, qw, scales, zeros, yr, r0, nr, k, group);
        }
    }
}

/* One row at a time, exactly as the reference CPU kernels loop (the yardstick the
 * row-blocked forms above are checked against, bit for bit). */
void fo_linear_f32_scalar(const float* x, const float* w, float scale, float* y, int64_t m,
                          int64_t n, int64_t k) {
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t f = 0; f < n; ++f) {
            const float* wr = w + f * k;
            float sum = 0.0f;
            for (int64_t c = 0; c < k; ++c) sum += xr[c] * wr[c];
            y[row * n + f] = sum * scale;
        }
    }
}

void fo_linear_bf16_scalar(const float* x, const uint16_t* w, float scale, float* y, int64_t m,
                           int64_t n, int64_t k) {
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t f = 0; f < n; ++f) {
            const uint16_t* wr = w + f * k;
            float sum = 0.0f;
            for (int64_t c = 0; c < k; ++c) sum += xr[c] * fo_bf16_to_f32(wr[c]);
            y[row * n + f] = sum * scale;
        }
    }
}

void fo_linear_int4_scalar(const float* x, const uint8_t* qw, const float* scales,
                           const uint8_t* zeros, float* y, int64_t m, int64_t n, int64_t k,
                           int group) {
    const int64_t groups = k / group;
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t f = 0; f < n; ++f) {
            const uint8_t* qrow = qw + f * (k / 2);
            const float* srow = scales + f * groups;
            const uint8_t* zrow = zeros + f * groups;
            float sum = 0.0f;
            for (int64_t c = 0; c < k; ++c) sum += xr[c] * w4_value(qrow, srow, zrow, c, group);
            y[row * n + f] = sum;
        }
    }
}

void fo_linear_int4_f64(const float* x, const uint8_t* qw, const float* scales,
                        const uint8_t* zeros, double* y, int64_t m, int64_t n, int64_t k,
                        int group) {
    const int64_t groups = k / group;
    for (int64_t row = 0; row < m; ++row) {
        const float* xr = x + row * k;
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
        for (int64_t f = 0; f < n; ++f) {
            const uint8_t* qrow = qw + f * (k / 2);
            const float* srow = scales + f * groups;
            const uint8_t* zrow = zeros + f * groups;
            double sum = 0.0;
            for (int64_t c = 0; c < k; ++c)
                sum += (double)xr[c] * (double)w4_value(qrow, srow, zrow, c, group);
            y[row * n + f] = sum;
        }
    }
}

void fo_rmsnorm(const float* x, const float* w, float* y, int64_t size, float eps) {
    float sum = 0.0f;
    for (int64_t i = 0; i < size; ++i) sum += x[i] * x[i];
    const float rs = 1.0f / sqrtf(sum / (float)size + eps);
    for (int64_t i = 0; i < size; ++i) y[i] = x[i] * w[i] * rs;
}

void fo_rmsnorm_rows(const float* x, const float* w, float* y, int64_t rows, int64_t width,
                     float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* xr = x + r * width;
        float* yr = y + r * width;
        float sq = 0.0f;
        for (int64_t c = 0; c < width; ++c) sq += xr[c] * xr[c];
        const float sc = 1.0f / sqrtf(sq / (float)width + eps);
        for (int64_t c = 0; c < width; ++c) yr[c] = xr[c] * w[c] * sc;
    }
}

void fo_rope_cache(int head_size, int max_seq, float theta, float* sin_cache, float* cos_cache) {
    const int half = head_size / 2;
    for (int d = 0; d < half; ++d) {
        const float freq = 1.0f / powf(theta, 2.0f * (float)d / (float)head_size);
        for (int p = 0; p < max_seq; ++p) {
            const float a = freq * (float)p;
            sin_cache[(int64_t)p * half + d] = sinf(a);
            cos_cache[(int64_t)p * half + d] = cosf(a);
        }
    }
}

void fo_rope(float* q, float* k, const float* cos_cache, const float* sin_cache, int q_heads,
             int k_heads, int head_size, int pos) {
    const int half = head_size / 2;
    const float* sr = sin_cache + (int64_t)pos * half;
    const float* cr = cos_cache + (int64_t)pos * half;
    for (int h = 0; h < q_heads; ++h) {
        float* qh = q + (int64_t)h * head_size;
        for (int d = 0; d < half; ++d) {
            const float fci = sr[d], fcr = cr[d];
            const float q0 = qh[d], q1 = qh[d + half];
            qh[d] = q0 * fcr - q1 * fci;
            qh[d + half] = q0 * fci + q1 * fcr;
            if (h < k_heads) {
                float* kh = k + (int64_t)h * head_size;
                const float k0 = kh[d], k1 = kh[d + half];
                kh[d] = k0 * fcr - k1 * fci;
                kh[d + half] = k0 * fci + k1 * fcr;
            }
        }
    }
}

void fo_softmax(float* x, int64_t n) {
    float mx = -INFINITY, sum = 0.0f;
    for (int64_t j = 0; j < n; ++j) mx = x[j] > mx ? x[j] : mx;
    for (int64_t j = 0; j < n; ++j) {
        const float v = expf(x[j] - mx);
        x[j] = v;
        sum += v;
    }
    const float inv = 1.0f / sum;
    for (int64_t j = 0; j < n; ++j) x[j] *= inv;
}

void fo_mha(const float* q, const float* key_cache, const float* value_cache, float* score,
            float* out, int q_heads, int kv_heads, int head_dim, int capacity, int layer,
            int pos) {
    const int kv_mul = q_heads / kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const int64_t layer_off = (int64_t)layer * capacity * kv_heads * head_dim;
    /* heads are independent: one thread per head, each head's loops unchanged */
#pragma omp parallel for schedule(static) num_threads(fo_get_threads())
    for (int h = 0; h < q_heads; ++h) {
        float* sh = score + (int64_t)h * capacity;
        const float* qh = q + (int64_t)h * head_dim;
        const int kvh = h / kv_mul;
        for (int t = 0; t <= pos; ++t) {
            const float* kt = key_cache + layer_off + ((int64_t)t * kv_heads + kvh) * head_dim;
            float dot = 0.0f;
            for (int d = 0; d < head_dim; ++d) dot += qh[d] * kt[d];
            sh[t] = dot * scale;
        }
        fo_softmax(sh, pos + 1);
        float* oh = out + (int64_t)h * head_dim;
        for (int d = 0; d < head_dim; ++d) oh[d] = 0.0f;
        for (int t = 0; t <= pos; ++t) {
            const float* vt = value_cache + layer_off + ((int64_t)t * kv_heads + kvh) * head_dim;
            const float a = sh[t];
            for (int d = 0; d < head_dim; ++d) oh[d] += a * vt[d];
        }
    }
}

void fo_swiglu(const float* gate, const float* up, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const float r = 1.0f / (1.0f + expf(-gate[i]));
        out[i] = gate[i] * r * up[i];
    }
}

void fo_add(const float* a, const float* b, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

void fo_embedding(const int32_t* tokens, int64_t count, const void* table, int dtype,
                  int64_t dim, float* out) {
    for (int64_t t = 0; t < count; ++t) {
        const int64_t row = tokens[t];
        if (dtype == 1) {
            const uint16_t* src = (const uint16_t*)table + row * dim;
            for (int64_t c = 0; c < dim; ++c) out[t * dim + c] = fo_bf16_to_f32(src[c]);
        } else {
            memcpy(out + t * dim, (const float*)table + row * dim, (size_t)dim * sizeof(float));
        }
    }
}

int64_t fo_argmax(const float* x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

/* ---------------------------------------------------------------- model ---- */

static void linear_apply(const fo_linear_t* L, const float* x, float* y) {
    switch (L->kind) {
    case FO_W_F32: fo_linear_f32(x, (const float*)L->w, 1.0f, y, 1, L->n, L->k); break;
    case FO_W_BF16: fo_linear_bf16(x, (const uint16_t*)L->w, 1.0f, y, 1, L->n, L->k); break;
    default:
        fo_linear_int4(x, (const uint8_t*)L->w, L->scales, L->zeros, y, 1, L->n, L->k, L->group);
        break;
    }
}

int64_t fo_qwen3_scratch_floats(const fo_qwen3_t* m, int capacity) {
    const int64_t h = m->hidden, q = (int64_t)m->q_heads * m->head_dim;
    const int64_t kv = (int64_t)m->kv_heads * m->head_dim, f = m->intermediate;
    /* hidden, norm, q, k, v, attn_out, attn_proj, attn_res, gate, up, act, down, score */
    return 5 * h + 2 * q + 2 * kv + 3 * f + (int64_t)m->q_heads * capacity + q;
}

void fo_qwen3_prepare(const fo_qwen3_t* m, fo_state_t* st) {
    fo_rope_cache(m->head_dim, st->max_seq, m->theta, st->rope_sin, st->rope_cos);
}

int fo_qwen3_forward(const fo_qwen3_t* m, fo_state_t* st, int token, int pos, float* logits) {
    if (token < 0 || token >= m->vocab) return -1;
    if (pos < 0 || pos >= st->capacity || pos >= st->max_seq) return -2;
    const int64_t H = m->hidden, Q = (int64_t)m->q_heads * m->head_dim;
    const int64_t KV = (int64_t)m->kv_heads * m->head_dim, F = m->intermediate;
    float* p = st->scratch;
    float* hidden = p; p += H;
    float* norm = p; p += H;
    float* attn_proj = p; p += H;
    float* attn_res = p; p += H;
    float* down = p; p += H;
    float* q = p; p += Q;
    float* attn_out = p; p += Q;
    float* k = p; p += KV;
    float* v = p; p += KV;
    float* gate = p; p += F;
    float* up = p; p += F;
    float* act = p; p += F;
    float* score = p;

    fo_embedding(&token, 1, m->embedding, m->emb_dtype, H, hidden);
    for (int l = 0; l < m->layers; ++l) {
        const fo_layer_t* L = &m->layer[l];
        fo_rmsnorm(hidden, L->attention_norm, norm, H, m->eps);
        linear_apply(&L->wq, norm, q);
        linear_apply(&L->wk, norm, k);
        linear_apply(&L->wv, norm, v);
        fo_rmsnorm_rows(q, L->q_norm, q, m->q_heads, m->head_dim, m->eps);
        fo_rmsnorm_rows(k, L->k_norm, k, m->kv_heads, m->head_dim, m->eps);
        fo_rope(q, k, st->rope_cos, st->rope_sin, m->q_heads, m->kv_heads, m->head_dim, pos);
        /* KVCache::write, src/model/kv_cache.cpp:31-73 */
        const int64_t off = ((int64_t)l * st->capacity + pos) * KV;
        memcpy(st->key_cache + off, k, (size_t)KV * sizeof(float));
        memcpy(st->value_cache + off, v, (size_t)KV * sizeof(float));
        fo_mha(q, st->key_cache, st->value_cache, score, attn_out, m->q_heads, m->kv_heads,
               m->head_dim, st->capacity, l, pos);
        linear_apply(&L->wo, attn_out, attn_proj);
        fo_add(hidden, attn_proj, attn_res, H);
        fo_rmsnorm(attn_res, L->ffn_norm, norm, H, m->eps);
        linear_apply(&L->w1, norm, gate);
        linear_apply(&L->w3, norm, up);
        fo_swiglu(gate, up, act, F);
        linear_apply(&L->w2, act, down);
        fo_add(attn_res, down, hidden, H);
    }
    fo_rmsnorm(hidden, m->final_norm, norm, H, m->eps);
    linear_apply(&m->output, norm, logits);
    return 0;
}
