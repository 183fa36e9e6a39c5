// Row-batched kernels of the engine's prefill path (internal, not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

struct PrefillRowsArgs {
    int n;                 // prompt rows in this chunk
    int pos0;              // position of row 0
    int q_heads, kv_heads; // per rank
    float eps, scale;      // RMSNorm eps, 1/sqrt(head_dim)
    const float* qkv;      // [n][q + 2 kv] projections
    const float* q_norm;   // [128]
    const float* k_norm;   // [128]
    const float* rope_sin; // [capacity][64]
    const float* rope_cos;
    float* q_out;          // [n][q] normalised, rotated q
    float* kcache;         // this layer's [capacity][kv_heads][128]
    float* vcache;
    float* attn_out;       // [n][q]
};

cudaError_t qk_rope_kv_rows_launch(const PrefillRowsArgs& a, cudaStream_t s);
cudaError_t causal_attention_launch(const PrefillRowsArgs& a, cudaStream_t s);
// act[r][8t + i] = silu(gu[r][16t + i]) * gu[r][16t + 8 + i] for the packed gate/up tiles
cudaError_t swiglu_packed_rows_launch(const float* gu, float* act, int rows, int f, int num_sms, cudaStream_t s);

}  // namespace fb
