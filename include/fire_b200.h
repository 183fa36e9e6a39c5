/*
 * fire_b200.h - C ABI of the fire_b200 sm_100a decode kernels and Qwen3 engine.
 *
 * Plain pointers, sizes and an opaque CUDA stream (cudaStream_t passed as void*;
 * NULL = the legacy default stream). No C++ or torch types cross this boundary.
 * Every entry point replaces one function behind Fire's src/op kernel dispatch
 * (src/op/kernels/kernels_interface.h:9-66); the citation on each names it
 * (paths relative to the Lin-yuqi/Fire source tree).
 *
 * Conventions (mirroring Fire's kernel contracts):
 *  - All tensors are caller-owned device memory, dense row-major. No entry point
 *    allocates, frees or synchronises; launches are asynchronous on `stream`
 *    ("CUDA success means submission", include/Fire/model/model.h:35-36).
 *  - Return value: FIRE_B200_OK (0); a negative FIRE_B200_ERR_* when the host-side
 *    argument check rejects the call (nothing is launched); or a positive
 *    cudaError_t from the launch.
 *  - Scratch memory (workspace) is passed in by the caller, sized by the matching
 *    *_workspace_bytes() call. A workspace must be zero-filled before its first use;
 *    every call leaves it zero-filled again. Calls that share a workspace must not
 *    overlap on the GPU.
 */
#ifndef FIRE_B200_H
#define FIRE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FIRE_B200_ABI_VERSION 1

enum {
    FIRE_B200_OK = 0,
    FIRE_B200_ERR_INVALID = -1,     /* bad pointer, shape, size or index */
    FIRE_B200_ERR_UNSUPPORTED = -2, /* valid request outside what this build implements */
    FIRE_B200_ERR_NO_DEVICE = -3,   /* no CUDA device / driver */
    FIRE_B200_ERR_STATE = -4,       /* engine used out of order (e.g. position mismatch) */
    FIRE_B200_ERR_IO = -5,          /* checkpoint file could not be read or is malformed */
    FIRE_B200_ERR_NOMEM = -6,       /* device memory reservation failed */
    FIRE_B200_ERR_DEVICE = -7,      /* a kernel of an earlier step reported failure (a bounded
                                       wait ran out, or it rejected the decode state); the
                                       engine refuses steps until it is reset */
    FIRE_B200_ERR_TIMEOUT = -8      /* a host-side deadline ran out (a tensor-parallel peer
                                       stopped answering); the communicator was aborted */
};

/* Element types: dense weights and embedding tables (F32, BF16); packed INT4 and
 * zero points (U8). */
enum { FIRE_B200_F32 = 0, FIRE_B200_BF16 = 1, FIRE_B200_U8 = 2 };

int fire_b200_abi_version(void);
const char* fire_b200_status_string(int status);

/* ------------------------------------------------------------------ Linear ---- */

/* INT4 group-wise Linear on Fire's .fire v2 layout, FP32 activations.
 * Replaces kernel::matmul_quant_kernel_cu (src/op/kernels/cuda/matmul_kernel.cu:280-314)
 * reached from LinearOp::forward (src/op/linear.cpp:19-25).
 *   x [rows, k] f32, qweight [n, k/2] u8 (even k in the low nibble),
 *   scales [n, k/group] f32, zero_points [n, k/group] u8 (0..15), y [rows, n] f32:
 *   y[r, j] = sum_k x[r, k] * (q[j, k] - z[j, k/group]) * s[j, k/group].
 * Requires rows >= 1, n >= 1, k even, group > 0 dividing k. rows == 1, group == 128,
 * k % 128 == 0 and a 16-byte aligned qweight take the sm_100a streaming GEMV; other
 * shapes and alignments take a slower general kernel with the same result. */
int fire_b200_linear_w4(const float* x, const uint8_t* qweight, const float* scales,
                        const uint8_t* zero_points, float* y, int rows, int n, int k,
                        int group_size, void* stream);

/* INT4 group-128 Linear for many rows (prefill, M >= 128) on the tcgen05 tensor cores.
 * Replaces matmul_quant_int4_fp32_naive for rows > 1 (src/op/kernels/cuda/matmul_kernel.cu:
 * 202-227, dispatched from :280-314). Same arguments and meaning as fire_b200_linear_w4,
 * but the product is taken on FP16 tensor cores: each weight s * (q - z) rounded once to
 * FP16, each row of x scaled by a power of two (its largest |x| into [2^14, 2^15)) and
 * rounded once to FP16, FP32 accumulation, the row scale undone exactly. Requires
 * rows % 128 == 0, n % 128 == 0, k % 128 == 0, group_size == 128, 16-byte aligned x, y and
 * workspace, 4-byte aligned qweight and scales. workspace: at least fire_b200_linear_w4_prefill_workspace_bytes(rows,
 * n, k) bytes of device memory. status_dev: optional device int (NULL: a word inside the
 * library) that the kernel sets non-zero: 1-3 if a bounded wait gives up, 4 if a group's
 * weights can leave the FP16 range (|s| * max(z, 15 - z) > 65504). */
size_t fire_b200_linear_w4_prefill_workspace_bytes(int rows, int n, int k);
int fire_b200_linear_w4_prefill(const float* x, const uint8_t* qweight, const float* scales,
                                const uint8_t* zero_points, float* y, int rows, int n, int k,
                                int group_size, void* workspace, size_t workspace_bytes,
                                int* status_dev, void* stream);

/* Dense Linear, FP32 or BF16 weights widened to FP32: y = scale * x W^T.
 * Replaces kernel::matmul_kernel_cu (src/op/kernels/cuda/matmul_kernel.cu:146-199)
 * reached from LinearOp::forward (src/op/linear.cpp:27-29); the LM head at M = 1.
 *   x [rows, k] f32, weight [n, k] (weight_dtype FIRE_B200_F32 or FIRE_B200_BF16). */
int fire_b200_linear_dense(const float* x, const void* weight, int weight_dtype, float scale,
                           float* y, int rows, int n, int k, void* stream);

/* -------------------------------------------------------- norms, RoPE, misc ---- */

/* RMSNorm over the whole vector: y = x * w / sqrt(mean(x^2) + eps).
 * Replaces kernel::rmsnorm_kernel_cu (src/op/kernels/cuda/rmsnorm_kernel.cu:152-175). */
int fire_b200_rmsnorm(const float* x, const float* w, float* y, int size, float eps,
                      void* stream);

/* RMSNorm of each row of width `width` with one shared weight [width] (q_norm/k_norm).
 * Replaces kernel::rmsnorm_kernel_cu_dim (src/op/kernels/cuda/rmsnorm_kernel.cu:177-201). */
int fire_b200_rmsnorm_rows(const float* x, const float* w, float* y, int rows, int width,
                           float eps, void* stream);

/* RoPE sin/cos caches [max_seq, head_size/2]: angle = pos / theta^(2d/head_size).
 * Replaces kernel::sin_cos_cache_kernel_cu (src/op/kernels/cuda/rope_kernel.cu:35-48). */
int fire_b200_rope_cache(int head_size, int max_seq, float theta, float* sin_cache,
                         float* cos_cache, void* stream);

/* Half-split rotary embedding of q [q_heads, head_size] and k [k_heads, head_size] in place
 * at position pos (0 <= pos < max_seq; caches [max_seq, head_size/2]).
 * Replaces kernel::rope_kernel_cu (src/op/kernels/cuda/rope_kernel.cu:81-105). */
int fire_b200_rope(float* q, float* k, const float* cos_cache, const float* sin_cache,
                   int q_heads, int k_heads, int head_size, int max_seq, int pos, void* stream);

/* GQA decode attention for one token at position pos of layer `layer`.
 * Replaces kernel::mha_kernel_cu (src/op/kernels/cuda/mha_kernel.cu:104-144).
 *   q [q_heads, head_dim]; key_cache/value_cache [layers, capacity, kv_heads, head_dim];
 *   out [q_heads, head_dim]; score [q_heads, capacity] or NULL: when given, entries
 *   0..pos of each row receive the softmax probabilities (as the reference does) and
 *   the rest are left untouched. q_heads % kv_heads == 0, q_heads/kv_heads <= 16,
 *   head_dim <= 256. workspace: fire_b200_mha_workspace_bytes(...) bytes. */
size_t fire_b200_mha_workspace_bytes(int q_heads, int kv_heads, int head_dim, int capacity);
int fire_b200_mha_decode(const float* q, const float* key_cache, const float* value_cache,
                         float* score, float* out, int layers, int capacity, int q_heads,
                         int kv_heads, int head_dim, int layer, int pos, void* workspace,
                         size_t workspace_bytes, void* stream);

/* The same attention for callers that cannot allocate device memory or pass a workspace:
 * e.g. a plug-in behind an interface that hands it only the tensors it computes on (the
 * query, the caches, the score buffer and the output; no scratch argument), or a program
 * whose device memory is fixed at start-up so nothing may be allocated later. This entry
 * point has no counterpart in the reference. Its scratch is a 4 MiB array inside the
 * library (held in every GPU's memory from library load to process exit), so it calls no
 * allocator; shapes whose scratch,
 * fire_b200_mha_workspace_bytes(q_heads, kv_heads, head_dim, capacity), exceeds
 * 4 MiB are rejected with FIRE_B200_ERR_UNSUPPORTED (e.g. 32 q heads of dim 128 fit up
 * to capacity 16128). The first call on each device looks the array's device address
 * up (make that first call before any stream capture); the address is kept for the life
 * of the process, so after a cudaDeviceReset this entry point must not be called again
 * on that device. All calls share the array: calls that overlap on the GPU race and must
 * be serialised by the caller. */
int fire_b200_mha_decode_noalloc(const float* q, const float* key_cache, const float* value_cache,
                                 float* score, float* out, int layers, int capacity, int q_heads,
                                 int kv_heads, int head_dim, int layer, int pos, void* stream);

/* Embedding row gather, BF16 rows widened to FP32: out[i, :] = table[tokens[i], :].
 * Replaces kernel::emb_kernel_cu (src/op/kernels/cuda/emb_kernel.cu:64-86). tokens are
 * device int32 [count]; out-of-range tokens leave their output row untouched. */
int fire_b200_embedding(const int32_t* tokens, int count, const void* table, int table_dtype,
                        int vocab, int dim, float* out, void* stream);

/* out = silu(gate) * up. Replaces kernel::swiglu_kernel_cu (src/op/kernels/cuda/swiglu_kernel.cu:15-28). */
int fire_b200_swiglu(const float* gate, const float* up, float* out, int n, void* stream);

/* out = a + b. Replaces kernel::add_kernel_cu (src/op/kernels/cuda/add_kernel.cu:12-31). */
int fire_b200_add(const float* a, const float* b, float* out, int n, void* stream);

/* Index of the first maximum of x[0..n), written to *out_index (device int64).
 * Replaces kernel::argmax_kernel_cu (src/op/kernels/cuda/argmax_kernel.cu:39-61) without its
 * per-call allocation and host synchronisation. */
size_t fire_b200_argmax_workspace_bytes(void);
int fire_b200_argmax(const float* x, int64_t n, int64_t* out_index, void* workspace,
                     size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FIRE_B200_H */
