/*
 * fire_oracle.h - TEST INFRASTRUCTURE ONLY (the parity oracle).
 *
 * A plain-C CPU restatement of Fire's single-token Qwen3 decode path. Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, and
 * only as the checker or as the timed CPU baseline; the fire_b200 product never
 * links or calls it. Each function names the reference file:line it restates
 * (paths relative to the Lin-yuqi/Fire source tree).
 *
 * Arithmetic rules kept from the reference CPU kernels:
 *   - FP32 everywhere, sequential accumulation in index order, one rounding per
 *     operation (built with -ffp-contract=off so a*b+c is never fused, as on a
 *     baseline x86-64 -O3 build without -march);
 *   - INT4 weights dequantise element-wise as s * (float(q) - float(z))
 *     (tools/quant.py:249-255) before the FP32 dot product.
 */
#ifndef FIRE_ORACLE_H
#define FIRE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number of OpenMP threads used by the row-parallel loops (0 = runtime default).
 * Row-parallel loops never change a row's own summation order. */
void fo_set_threads(int n);
int fo_get_threads(void);

float fo_bf16_to_f32(uint16_t bits);

/* tools/quant.py:141-261 dequantize_int4_groupwise: w[n,k] = s[n,g]*(q[n,k]-z[n,g]). */
void fo_dequant_int4(const uint8_t* qw, const float* scales, const uint8_t* zeros, float* w,
                     int64_t n, int64_t k, int group);

/* src/op/kernels/cpu/matmul_kernel.cpp:83-117: y[m,n] = scale * sum_k x[m,k]*w[n,k]. The
 * reference's FP32 branch goes through Armadillo (order unpinned); this restates it with
 * the BF16 branch's sequential order (:95-106). */
void fo_linear_f32(const float* x, const float* w, float scale, float* y, int64_t m, int64_t n,
                   int64_t k);
/* src/op/kernels/cpu/matmul_kernel.cpp:92-107 (BF16 weight widened at use). */
void fo_linear_bf16(const float* x, const uint16_t* w, float scale, float* y, int64_t m,
                    int64_t n, int64_t k);
/* Dequantise (tools/quant.py:249-255) then FP32 Linear (matmul_kernel.cpp:95-106).
 * Any group size dividing k, k even. */
void fo_linear_int4(const float* x, const uint8_t* qw, const float* scales,
                    const uint8_t* zeros, float* y, int64_t m, int64_t n, int64_t k, int group);
/* The three linears above compute eight rows in lock step (vector lanes), each row in the
 * reference's sequential order; these one-row-at-a-time forms are the plain loops they must
 * equal bit for bit. */
void fo_linear_f32_scalar(const float* x, const float* w, float scale, float* y, int64_t m,
                          int64_t n, int64_t k);
void fo_linear_bf16_scalar(const float* x, const uint16_t* w, float scale, float* y, int64_t m,
                           int64_t n, int64_t k);
void fo_linear_int4_scalar(const float* x, const uint8_t* qw, const float* scales,
                           const uint8_t* zeros, float* y, int64_t m, int64_t n, int64_t k,
                           int group);
/* Same products accumulated in double: the error yardstick for tolerance tests. */
void fo_linear_int4_f64(const float* x, const uint8_t* qw, const float* scales,
                        const uint8_t* zeros, double* y, int64_t m, int64_t n, int64_t k,
                        int group);

/* src/op/kernels/cpu/rmsnorm_kernel.cpp:6-39 (whole tensor as one row). */
void fo_rmsnorm(const float* x, const float* w, float* y, int64_t size, float eps);
/* src/op/kernels/cpu/rmsnorm_kernel.cpp:41-67 (each row of width `width`). */
void fo_rmsnorm_rows(const float* x, const float* w, float* y, int64_t rows, int64_t width,
                     float eps);

/* src/op/kernels/cpu/rope_kernel.cpp:8-24: caches [max_seq, head/2]. */
void fo_rope_cache(int head_size, int max_seq, float theta, float* sin_cache, float* cos_cache);
/* src/op/kernels/cpu/rope_kernel.cpp:26-52: half-split rotation, in place. */
void fo_rope(float* q, float* k, const float* cos_cache, const float* sin_cache, int q_heads,
             int k_heads, int head_size, int pos);

/* src/op/kernels/cpu/softmax_kernel.cpp:7-40, one row in place. */
void fo_softmax(float* x, int64_t n);

/* src/op/kernels/cpu/mha_kernel.cpp:16-114. Caches [layers, capacity, kv_heads, head_dim];
 * score [q_heads, capacity] (entries 0..pos written); out [q_heads, head_dim]. */
void fo_mha(const float* q, const float* key_cache, const float* value_cache, float* score,
            float* out, int q_heads, int kv_heads, int head_dim, int capacity, int layer,
            int pos);

/* src/op/kernels/cpu/swiglu_kernel.cpp:15-19: out = g * (1/(1+exp(-g))) * u. */
void fo_swiglu(const float* gate, const float* up, float* out, int64_t n);
/* src/op/kernels/cpu/add_kernel.cpp:15-21. */
void fo_add(const float* a, const float* b, float* out, int64_t n);
/* src/op/kernels/cpu/emb_kernel.cpp:9-37 (dtype 0 = FP32 rows, 1 = BF16 rows widened). */
void fo_embedding(const int32_t* tokens, int64_t count, const void* table, int dtype,
                  int64_t dim, float* out);
/* src/op/kernels/cuda/argmax_kernel.cu:18-35 semantics: first index of the maximum. */
int64_t fo_argmax(const float* x, int64_t n);

/* ----- whole-model restatement: src/model/qwen.cpp:155-303 ----- */
enum { FO_W_F32 = 0, FO_W_BF16 = 1, FO_W_INT4 = 2 };

typedef struct {
    int kind;               /* FO_W_* */
    int64_t n, k;           /* logical [n, k] */
    int group;              /* INT4 group size */
    const void* w;          /* FP32 [n,k], BF16 [n,k] or packed u8 [n,k/2] */
    const float* scales;    /* INT4: [n, k/group] */
    const uint8_t* zeros;   /* INT4: [n, k/group] */
} fo_linear_t;

typedef struct {
    const float* attention_norm; /* [hidden] */
    fo_linear_t wq, wk, wv, wo;
    const float* q_norm;         /* [head_dim] */
    const float* k_norm;         /* [head_dim] */
    const float* ffn_norm;       /* [hidden] */
    fo_linear_t w1, w2, w3;      /* gate, down, up */
} fo_layer_t;

typedef struct {
    int hidden, intermediate, layers, q_heads, kv_heads, head_dim;
    int64_t vocab;
    float eps, theta;
    int emb_dtype;               /* 0 FP32, 1 BF16 */
    const void* embedding;       /* [vocab, hidden] */
    const fo_layer_t* layer;     /* [layers] */
    const float* final_norm;     /* [hidden] */
    fo_linear_t output;          /* lm head [vocab, hidden] */
} fo_qwen3_t;

typedef struct {
    int capacity;                /* KV positions */
    int max_seq;                 /* rope cache rows */
    float* key_cache;            /* [layers, capacity, kv_heads, head_dim] */
    float* value_cache;
    float* rope_sin;             /* [max_seq, head_dim/2] */
    float* rope_cos;
    float* scratch;              /* fo_qwen3_scratch_floats() floats */
} fo_state_t;

int64_t fo_qwen3_scratch_floats(const fo_qwen3_t* m, int capacity);
/* Fills the rope caches (Qwen3Model::prepare, src/model/qwen.cpp:143-149). */
void fo_qwen3_prepare(const fo_qwen3_t* m, fo_state_t* st);
/* One token at position pos; writes logits [vocab]. Returns 0 or a negative code. */
int fo_qwen3_forward(const fo_qwen3_t* m, fo_state_t* st, int token, int pos, float* logits);

#ifdef __cplusplus
}
#endif
#endif
