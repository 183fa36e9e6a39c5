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

void fo_linear_f32(const float* x, const float* w, float scale, float* y, int64_t m, int64_t n,
                   int64_t k) {
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

void fo_linear_bf16(const float* x, const uint16_t* w, float scale, float* y, int64_t m,
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

void fo_linear_int4(const float* x, const uint8_t* qw, const float* scales,
                    const uint8_t* zeros, float* y, int64_t m, int64_t n, int64_t k, int group) {
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
