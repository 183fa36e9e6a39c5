// Qwen3 single-token decode engine (the B200 implementation behind Fire's
// Qwen3Model, src/model/qwen.cpp:30-303, and Qwen3Loader, src/model/qwen_loader.cpp).
//
// One engine serves one sequence on one GPU, or one tensor-parallel rank of it.
// Weights are imported once into a device arena and repacked for the kernels:
//   * q/k/v rows concatenated into one INT4 matrix (one GEMV launch per layer);
//   * gate/up rows interleaved per GEMV tile (the SwiGLU epilogue sees both halves);
//   * tensor parallel: column-parallel q/k/v/gate/up (heads / FFN rows), row-parallel
//     o/down (group-aligned K slices), vocab-sharded LM head, replicated embedding and
//     norms, KV cache sharded by KV head.
// A decode step is a fixed launch sequence that reads the token and position from a
// device-resident control block, so it is captured once in a CUDA graph and replayed:
//   embedding -> per layer [qkv GEMV (RMSNorm prologue) -> q/k-norm+RoPE+KV write ->
//   split-K attention -> o GEMV (+residual) -> gate/up GEMV (RMSNorm prologue, SwiGLU
//   epilogue) -> down GEMV (+residual)] -> LM head (final-norm prologue) -> argmax.
// Under tensor parallelism the o/down partial sums go through an NCCL all-reduce and
// the residual add moves into the next GEMV's prologue; sampling all-gathers one
// (max, index) pair per rank.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "engine/arena.h"
#include "engine/nccl_shim.h"
#include "kernels/decode_state.h"
#include "kernels/layer_stack.h"

namespace fb {

struct Qwen3Dims {
    int vocab = 0, max_seq = 0, hidden = 0, inter = 0, layers = 0, q_heads = 0, kv_heads = 0, head_dim = 0;
    float eps = 0.f, theta = 0.f;
};

enum SrcDType : int { kSrcF32 = 0, kSrcBF16 = 1, kSrcU8 = 2 };

// One tensor of a Fire checkpoint (names as in tools/export_qwen3.py), host or device.
struct TensorSrc {
    std::string name;
    int dtype = kSrcF32;
    std::vector<int64_t> shape;
    const void* data = nullptr;
    bool on_device = false;
};

struct EngineOptions {
    int tp_rank = 0, tp_size = 1;
    const void* nccl_id = nullptr;  // 128-byte ncclUniqueId shared by all ranks (tp_size > 1)
    bool use_graph = true;
    bool pdl = true;
    int deadline_ms = 0;  // host-side deadline of a synchronising wait under tensor parallelism (0 = 30 s)
};

struct W4Mat {
    uint8_t* qw = nullptr;
    float* s = nullptr;
    uint8_t* z = nullptr;
    int n = 0, k = 0;
};

class Qwen3Engine {
  public:
    static int create(const Qwen3Dims& dims, const std::vector<TensorSrc>& tensors, const EngineOptions& opt,
                      std::unique_ptr<Qwen3Engine>* out, std::string* err);
    ~Qwen3Engine();

    // Model::prepare (include/Fire/model/model.h:25-29): runtime buffers, KV cache,
    // RoPE caches and the captured step graphs for 1 <= capacity <= max_seq.
    int prepare(int capacity);
    // Model::forward: consume `token` at `pos` (== length), logits [vocab] into the
    // engine buffer and, if given, into `logits_out` (device). Asynchronous on `s`.
    int forward(int token, int pos, float* logits_out, cudaStream_t s);
    // Greedy decode on the device: `steps` tokens starting from `first_token` at the
    // current length; tokens_out (device int32 [steps]) receives the sampled ids.
    // No host synchronisation between tokens.
    int generate(int first_token, int steps, int32_t* tokens_out, cudaStream_t s);
    // The reference's host loop (demo/qwen_chat.cpp:231-294): per token an H2D copy of
    // the token id from pinned memory, one step, a D2H copy of the sampled id and a
    // stream synchronisation. Prompt tokens are consumed first (no sampling until the
    // last one); out_host receives `steps` sampled ids.
    int generate_host(const int32_t* prompt, int n_prompt, int steps, int32_t* out_host, cudaStream_t s);
    // Batched prefill: consume n prompt tokens (host ids) at positions length()..,
    // leaving the KV cache and the last token's logits as n forward() calls would, with
    // the projections (FP16 operands) and the causal attention on the tensor cores. Under
    // tensor parallelism each rank multiplies its shards (column-parallel q/k/v and
    // gate/up, row-parallel o and down, whose [rows, hidden] partial sums are all-reduced
    // over NCCL) and the vocab-sharded head is all-gathered. Falls back to forward() per
    // token with the per-op kernels or for fewer than 64 tokens. Synchronises with `s`.
    int prefill(const int32_t* tokens, int n, float* logits_out, cudaStream_t s);
    int reset();
    int truncate(int length);
    // KVCache::key()/value() (include/Fire/model/kv_cache.h:24-28): copy positions
    // [0, length) of every layer of this rank's cache shard to / from `key`, `value`
    // ([layers][length][kv_heads/tp][128] FP32, host or device). Import sets the length.
    // Both synchronise with `s`.
    int kv_export(int length, float* key, float* value, cudaStream_t s) const;
    int kv_import(int length, const float* key, const float* value, cudaStream_t s);
    // Waits for the steps enqueued so far (under tensor parallelism with the host deadline,
    // polling the communicator); FIRE_B200_ERR_DEVICE if a kernel recorded a failure in
    // the decode state (its code in *device_error), FIRE_B200_ERR_TIMEOUT if the deadline
    // ran out (the communicator is then aborted and the engine unusable).
    int status(int* device_error);
    // ncclCommAbort of this rank's communicator (tensor parallel); the engine is then dead
    int abort();

    int length() const { return length_; }
    int capacity() const { return capacity_; }
    const float* logits() const { return tp_ > 1 ? logits_full_ : logits_; }
    size_t weight_bytes() const { return weight_bytes_; }
    size_t runtime_bytes() const { return runtime_arena_ ? runtime_arena_->used() : 0; }
    // Kernels of this library launched per decode step with sampling (graph nodes).
    int kernels_per_step() const;
    // Bytes of weights one decode step reads on this rank (the roofline numerator).
    size_t step_weight_bytes() const { return step_weight_bytes_; }
    int tp_size() const { return tp_; }
    int tp_rank() const { return rank_; }

    bool uses_layer_stack() const { return stack_; }
    // Timeline of the last layer-stack launch ([grid][layers][5][5] %globaltimer stamps,
    // see StackArgs::trace); returns the word count, 0 when tracing is off.
    int64_t stack_trace(uint64_t* host_out, int64_t capacity_words) const;
    // Average device time (ms) of `reps` launches of the layer-stack kernel alone at
    // position length() (the KV row there is rewritten; the length does not change).
    int time_layer_stack(int reps, float* ms_out, cudaStream_t s);

  private:
    Qwen3Engine() = default;
    StackArgs stack_template(int capacity) const;
    int import_weights(const std::vector<TensorSrc>& tensors, std::string* err);
    int enqueue_step(cudaStream_t s, bool sample);
    int prefill_buffers();
    int prefill_chunk(int m, int mp, int pos0, cudaStream_t s);
    int prefill_linear(const float* x, const uint8_t* items, int n, int k, float* y, int mp, cudaStream_t s);
    int capture(bool sample, cudaGraphExec_t* exec);
    int launch_step(cudaStream_t s, bool sample);
    // after a group of steps: the state's error word to the pinned host mirror, and the
    // event that status() waits for
    int mark_steps(cudaStream_t s);
    // FIRE_B200_ERR_DEVICE / _STATE when an earlier step failed or the engine was aborted
    int refuse() const;
    int wait_event(cudaEvent_t ev);

    Qwen3Dims d_;
    EngineOptions opt_;
    int device_ = 0, sms_ = 0;
    int tp_ = 1, rank_ = 0;
    // per-rank dimensions
    int hq_ = 0, hkv_ = 0, q_ = 0, kv_ = 0, f_ = 0, v_ = 0, v_off_ = 0;

    std::unique_ptr<DeviceArena> weight_arena_, runtime_arena_;
    size_t weight_bytes_ = 0, step_weight_bytes_ = 0;

    struct Layer {
        float* attn_norm = nullptr;
        float* q_norm = nullptr;
        float* k_norm = nullptr;
        float* ffn_norm = nullptr;
        W4Mat qkv, o, gu, down;
        uint8_t *qkv_items = nullptr, *o_items = nullptr, *gu_items = nullptr, *down_items = nullptr;
    };
    std::vector<Layer> layers_;
    void* embedding_ = nullptr;
    bool emb_bf16_ = false;
    float* final_norm_ = nullptr;
    int head_kind_ = 0;  // 0 FP32 dense, 1 BF16 dense, 2 INT4
    W4Mat head_w4_;
    void* head_dense_ = nullptr;

    // runtime
    int capacity_ = 0, length_ = 0, max_chunks_ = 0;
    DecodeState* state_ = nullptr;
    float *hidden_ = nullptr, *attn_res_ = nullptr, *qkv_ = nullptr, *q_rot_ = nullptr, *attn_out_ = nullptr;
    float *o_part_ = nullptr, *act_ = nullptr, *down_part_ = nullptr, *logits_ = nullptr, *logits_full_ = nullptr;
    float *kcache_ = nullptr, *vcache_ = nullptr, *rope_sin_ = nullptr, *rope_cos_ = nullptr;
    void* attn_ws_ = nullptr;
    void* argmax_ws_ = nullptr;
    void* best_local_ = nullptr;
    void* best_all_ = nullptr;
    int32_t* tokens_buf_ = nullptr;
    DecodeState* host_state_ = nullptr;  // pinned, for generate_host
    DecodeState* host_seen_ = nullptr;   // pinned: the device state copied back after each step group
    cudaEvent_t steps_done_ = nullptr;   // recorded after that copy
    bool aborted_ = false;               // the communicator was aborted at a deadline
    cudaGraphExec_t graph_fwd_ = nullptr, graph_step_ = nullptr;
    NcclComm comm_ = nullptr;

    // persistent layer-stack kernel: weights in item layout
    bool stack_ = false;
    // tensor parallel with the layer stack: this rank's exchange block (cudaMalloc, so it
    // can be shared by IPC handle) and every rank's block as mapped here (own at [rank])
    void* xchg_ = nullptr;
    void* xchg_peer_[kStackMaxTp] = {};
    int setup_exchange(std::string* err);
    StackLayer* stack_layers_ = nullptr;  // device [layers]
    StackArgs stack_args_{};
    unsigned* stack_sync_ = nullptr;
    size_t stack_sync_bytes_ = 0;
    // batched prefill scratch (allocated on first use)
    std::unique_ptr<DeviceArena> prefill_arena_;
    int32_t* pf_tok_ = nullptr;
    float *pf_x_ = nullptr, *pf_xn_ = nullptr, *pf_qkv_ = nullptr, *pf_q_ = nullptr, *pf_att_ = nullptr;
    float *pf_o_ = nullptr, *pf_gu_ = nullptr, *pf_act_ = nullptr;
    void* pf_gemm_ws_ = nullptr;
    size_t pf_gemm_ws_bytes_ = 0;
    void* pf_w_ = nullptr;  // FP16 copy of the matrix being multiplied (two-pass form)
    int* pf_err_ = nullptr;
    bool stack_trace_on_ = false;  // FIRE_B200_STACK_TRACE=1: record the per-phase timeline
    bool stall_on_ = false;        // FIRE_B200_FAULT_STALL=1 (tests): StackArgs::stall armed by prepare
    int* stall_ = nullptr;         // device flag, cleared by reset()
    size_t stack_trace_words_ = 0;
};

}  // namespace fb
