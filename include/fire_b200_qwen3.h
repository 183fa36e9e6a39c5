/*
 * fire_b200_qwen3.h - C ABI of the Qwen3 single-token decode engine (B200, sm_100a).
 *
 * The engine is the GPU body behind Fire's Model / Qwen3Model / Qwen3Loader
 * (include/Fire/model/model.h:22-52, src/model/qwen.cpp:30-311,
 * src/model/qwen_loader.cpp:123-223): one handle serves one sequence on the current
 * CUDA device, or one tensor-parallel rank of it. Status codes and stream
 * conventions are those of fire_b200.h.
 */
#ifndef FIRE_B200_QWEN3_H
#define FIRE_B200_QWEN3_H

#include <stddef.h>
#include <stdint.h>

#include "fire_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fire_b200_qwen3 fire_b200_qwen3; /* opaque engine handle */

/* Architecture constants: Qwen3Profile (include/Fire/model/model_weights.h:108-137). */
typedef struct {
    int vocab_size, max_seq_len, hidden_size, intermediate_size, num_layers;
    int num_attention_heads, num_kv_heads, head_dim;
    float rms_norm_eps, rope_theta;
} fire_b200_qwen3_profile;

/* One checkpoint tensor, named as Fire's exporter names it (tools/export_qwen3.py:268-395):
 * "tok_embeddings.weight", "layers.{i}.attention.wq.qweight|scales|zero_points", ...,
 * "norm.weight", "output.weight" or "output.qweight|scales|zero_points". */
typedef struct {
    const char* name;
    int dtype;         /* FIRE_B200_F32, FIRE_B200_BF16 or FIRE_B200_U8 */
    int ndim;          /* 1 or 2 */
    int64_t shape[2];
    const void* data;  /* host memory, or device memory of the current device */
    int on_device;
} fire_b200_tensor;

typedef struct {
    int tp_rank;          /* 0 .. tp_size-1 */
    int tp_size;          /* 1 = single GPU; >1 = tensor parallel, one process per GPU */
    const void* nccl_id;  /* 128-byte NCCL unique id, the same on every rank (tp_size > 1) */
    int use_graph;        /* capture each decode step in a CUDA graph (recommended: 1) */
    int pdl;              /* programmatic dependent launch between kernels (recommended: 1) */
    int deadline_ms;      /* tensor parallel: host-side deadline of a synchronising wait
                             (generate_host, status, reset); 0 = 30000 */
} fire_b200_qwen3_options;

/* A new NCCL unique id (128 bytes) for rank 0 to share with the other ranks. */
int fire_b200_nccl_unique_id(void* id128);

/* Import weights (INT4 group-128 projections; FP32/BF16/INT4 LM head; FP32/BF16
 * embedding) into device memory and build the engine: Qwen3Loader::load_weights +
 * Qwen3Model::create. Tensor parallel ranks keep only their shard. When any tensor is in
 * device memory the call first synchronises the device, so tensors still being written by
 * work queued on other streams are read complete. */
int fire_b200_qwen3_create(const fire_b200_qwen3_profile* profile, const fire_b200_tensor* tensors, int count,
                           const fire_b200_qwen3_options* options, fire_b200_qwen3** out);
/* The same from a .fire v1/v2 file (Qwen3Loader::open, src/model/qwen_loader.cpp:12-17). */
int fire_b200_qwen3_open(const char* fire_path, const fire_b200_qwen3_profile* profile,
                         const fire_b200_qwen3_options* options, fire_b200_qwen3** out);
/* Message of the last failed create/open on this thread ("" if none). */
const char* fire_b200_qwen3_last_error(void);

/* Model::prepare: runtime buffers, KV cache and RoPE caches for 1 <= capacity <= max_seq_len;
 * starts an empty sequence. Synchronises the device. */
int fire_b200_qwen3_prepare(fire_b200_qwen3* m, int capacity);
/* Model::forward: consume token_id at pos (must equal the current length); logits [vocab]
 * FP32 land in the engine buffer (fire_b200_qwen3_logits) and, if non-NULL, in `logits`
 * (device). Success advances the length by one. Asynchronous on `stream`. */
int fire_b200_qwen3_forward(fire_b200_qwen3* m, int token_id, int pos, float* logits, void* stream);
/* Greedy decode of `steps` tokens on the device from `first_token` at the current length:
 * tokens_out (device int32 [steps]) receives the argmax ids (first index on ties); no host
 * round trip between tokens. Advances the length by `steps`. */
int fire_b200_qwen3_generate(fire_b200_qwen3* m, int first_token, int steps, int32_t* tokens_out, void* stream);
/* The reference's host decode loop (demo/qwen_chat.cpp:231-294 + ArgmaxSampler): prompt tokens
 * one by one, then per generated token an H2D copy of its input id, one step, a D2H copy of
 * the sampled id and a stream synchronisation. prompt/out are host arrays; out gets `steps` ids. */
int fire_b200_qwen3_generate_host(fire_b200_qwen3* m, const int32_t* prompt, int n_prompt, int steps,
                                  int32_t* out, void* stream);
/* Model::reset: empty the sequence, keep weights and capacity. Also clears a failure
 * recorded by an earlier step (see fire_b200_qwen3_status). */
int fire_b200_qwen3_reset(fire_b200_qwen3* m);
/* Outcome of the steps enqueued so far. Launches are asynchronous ("CUDA success means
 * submission", include/Fire/model/model.h:41-42), so a kernel that fails a step records a
 * code in the engine's device-side decode state instead: 1 position rejected, 2 token
 * rejected, 3 a bounded wait of the layer-stack kernel ran out (a peer or a CTA that never
 * arrived). This call waits for the last step and returns FIRE_B200_OK, or
 * FIRE_B200_ERR_DEVICE with the code in *device_error (if not NULL). After a failure every
 * step entry point returns FIRE_B200_ERR_DEVICE until fire_b200_qwen3_reset. Under tensor
 * parallelism the wait has the host deadline of the options; when it runs out, or NCCL
 * reports an asynchronous error, the communicator is aborted (ncclCommAbort) and the call
 * returns FIRE_B200_ERR_TIMEOUT; the engine is then only fit for destroy. */
int fire_b200_qwen3_status(fire_b200_qwen3* m, int* device_error);
/* Leave a tensor-parallel group without waiting for the peers: abort this rank's NCCL
 * communicator (ncclCommAbort ends its kernels in flight). No reference counterpart (Fire
 * is single-device). The engine then returns FIRE_B200_ERR_TIMEOUT from every step and is
 * only fit for destroy. A no-op at tp_size 1. */
int fire_b200_qwen3_abort(fire_b200_qwen3* m);
/* KVCache::key() / value() (include/Fire/model/kv_cache.h:24-28): copy the FP32 K and V
 * of positions [0, length) of every layer out of the engine. `key` and `value` are
 * [num_layers][length][kv_heads_local][head_dim], kv_heads_local = num_kv_heads / tp_size
 * (this rank's heads), host or device memory; length <= fire_b200_qwen3_length.
 * Synchronises with `stream`. */
int fire_b200_qwen3_kv_export(const fire_b200_qwen3* m, int length, float* key, float* value, void* stream);
/* The reverse: load a KV prefix of `length` positions (same layout) and make it the current
 * sequence, as if those tokens had been consumed (a saved prompt, or a prefix shared with a
 * checker). Synchronises with `stream`. */
int fire_b200_qwen3_kv_import(fire_b200_qwen3* m, int length, const float* key, const float* value, void* stream);
/* Shorten the sequence to `length` tokens (0 <= length <= current length), keeping the KV
 * cache of the kept prefix, so a shared prompt can be decoded from again. */
int fire_b200_qwen3_truncate(fire_b200_qwen3* m, int length);
int fire_b200_qwen3_length(const fire_b200_qwen3* m);
/* Device pointer to the last logits [vocab] (full vocabulary on every rank). */
const float* fire_b200_qwen3_logits(const fire_b200_qwen3* m);
/* Kernels of this library one sampled decode step launches (CUDA graph nodes). */
int fire_b200_qwen3_kernels_per_step(const fire_b200_qwen3* m);

/* Batched prefill (the reference prefills token by token, demo/qwen_chat.cpp:202-213):
 * consume n prompt ids (host memory) at positions length()..length()+n-1 and leave the KV
 * cache, the length and the last token's logits (engine buffer, and logits_out if not
 * NULL) as n calls of fire_b200_qwen3_forward would. With 64 or more tokens the projections
 * and the causal attention run on the tensor cores in chunks of up to 2048 rows (FP16
 * operands with FP32 accumulation for the projections; FP16 q.K^T and BF16 P.V with an FP32
 * softmax for attention), so the values match forward() to about 1e-3; under tensor parallelism each
 * rank multiplies its shards and the row-parallel o / down outputs are all-reduced over NCCL.
 * Otherwise (fewer tokens, or the per-op kernels) it is forward() per token. Synchronises
 * with `stream` before returning. */
int fire_b200_qwen3_prefill(fire_b200_qwen3* m, const int32_t* tokens, int n, float* logits_out,
                            void* stream);

/* Diagnostics (no reference counterpart): with FIRE_B200_STACK_TRACE=1 in the
 * environment at create time, the persistent layer-stack kernel records a per-phase
 * timeline of its last launch, [CTAs][layers][5 phases][13 values]: 5 stamps of the
 * GPU's nanosecond timer (phase entered, input ready, input staged, last unit done, last
 * item issued) and 2 SM-cycle totals (consumer warps waiting for ring items, the
 * producer waiting for free slots), then 6 attention stamps (chunk partial written,
 * ticket taken, merge done; warp 0's scores, local softmax and P.V done). Copies up to capacity_words words into out (may be
 * NULL) after a device synchronisation; returns the word count, 0 when tracing is off,
 * -1 on a CUDA error. */
int64_t fire_b200_qwen3_stack_trace(const fire_b200_qwen3* m, uint64_t* out, int64_t capacity_words);
/* Diagnostics: average device time in milliseconds of `reps` launches of the layer-stack
 * kernel alone at position length() (its KV row is rewritten, the length is unchanged),
 * timed with CUDA events on `stream` (NULL = default). FIRE_B200_ERR_STATE when the
 * engine does not use the layer-stack kernel (tensor parallel, or switched off). */
int fire_b200_qwen3_time_layer_stack(fire_b200_qwen3* m, int reps, float* ms_out, void* stream);
/* Weight bytes one decode step reads on this rank (projections, head, norms, one
 * embedding row): the numerator of the HBM roofline. */
uint64_t fire_b200_qwen3_step_weight_bytes(const fire_b200_qwen3* m);
void fire_b200_qwen3_destroy(fire_b200_qwen3* m);

#ifdef __cplusplus
}
#endif
#endif /* FIRE_B200_QWEN3_H */
