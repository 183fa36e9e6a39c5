// Internal launch interface of the small decode kernels (norm, RoPE, attention,
// embedding, element-wise, argmax). Not part of the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode_state.h"

namespace fb {

struct QkRopeArgs {
    const float* qkv;       // [q_heads*128 + 2*kv_heads*128]
    const float* q_norm;    // [128]
    const float* k_norm;    // [128]
    const float* rope_sin;  // [max_seq, 64]
    const float* rope_cos;
    float* q_out;           // [q_heads*128]
    float* key_cache;       // this layer's [capacity, kv_heads, 128]
    float* value_cache;
    DecodeState* state;     // position source (device), or nullptr to use `pos`
    int pos;
    int q_heads, kv_heads, capacity;
    float eps;
};

struct AttnArgs {
    const float* q;          // [q_heads, hd]
    const float* key_cache;  // this layer's [capacity, kv_heads, hd]
    const float* value_cache;
    float* out;              // [q_heads, hd]
    float* score;            // optional [q_heads, capacity]: softmax probabilities 0..pos
    float* part;             // [q_heads, max_chunks, hd] partial outputs (workspace)
    float* part_ml;          // [q_heads, max_chunks, 2] running max / sum (workspace)
    unsigned* tickets;       // [kv_heads], zero before first use, left zero
    const DecodeState* state;  // position source (device), or nullptr to use `pos`
    int pos;
    int q_heads, kv_heads, hd, capacity, max_chunks;
    float scale;             // 1/sqrt(hd)
    // Fused q/k-norm + RoPE + KV write (decode engine, hd 128): when qkv is set, q, k
    // and v of the current token come raw from qkv = [q | k | v] (all heads of this
    // rank); each CTA normalises and rotates its q heads, and the CTA whose chunk holds
    // `pos` rotates k and writes k and v into the cache (src/model/qwen.cpp:222-240).
    const float* qkv = nullptr;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
    const float* rope_sin = nullptr;  // [capacity, 64]
    const float* rope_cos = nullptr;
    float eps = 0.f;
};

constexpr int kAttnChunk = 64;  // keys per split

cudaError_t rmsnorm_launch(const float* x, const float* w, float* y, int size, float eps,
                           cudaStream_t s, bool pdl);
cudaError_t rmsnorm_rows_launch(const float* x, const float* w, float* y, int rows, int width,
                                float eps, cudaStream_t s);
cudaError_t rope_cache_launch(int head, int max_seq, float theta, float* sin_c, float* cos_c,
                              int num_sms, cudaStream_t s);
cudaError_t rope_launch(float* q, float* k, const float* cos_c, const float* sin_c, int q_heads,
                        int k_heads, int head, int pos, int num_sms, cudaStream_t s);
cudaError_t qk_norm_rope_kv_launch(const QkRopeArgs& a, cudaStream_t s, bool pdl);
cudaError_t embedding_launch(const int32_t* tokens, int count, DecodeState* state, const void* table,
                             bool bf16, int vocab, int dim, float* out, cudaStream_t s, bool pdl);
cudaError_t swiglu_launch(const float* g, const float* u, float* o, int n, int num_sms, cudaStream_t s);
cudaError_t add_launch(const float* a, const float* b, float* o, int n, int num_sms, cudaStream_t s);
size_t argmax_workspace_bytes(int num_sms);
// First index of the maximum of x[0..n). Result: *out_index (if given) and either
// best_out (an 8-byte {float value; int32 index} pair, index offset by base_index) or,
// without best_out, the decode state advanced to the sampled token.
cudaError_t argmax_launch(const float* x, int n, void* workspace, int num_sms, int64_t* out_index,
                          DecodeState* state, int32_t* tokens_out, int max_steps, cudaStream_t s,
                          bool pdl, int base_index = 0, void* best_out = nullptr);
constexpr size_t kArgmaxPairBytes = 8;
// Folds `count` gathered pairs (rank order) and advances the decode state.
cudaError_t argmax_select_launch(const void* parts, int count, DecodeState* state, int32_t* tokens_out,
                                 int max_steps, cudaStream_t s, bool pdl);
cudaError_t set_state_launch(DecodeState* state, int token, int pos, int step, cudaStream_t s, bool pdl);

size_t attention_workspace_bytes(int q_heads, int kv_heads, int hd, int capacity);
cudaError_t attention_launch(const AttnArgs& a, cudaStream_t s, bool pdl);

}  // namespace fb
