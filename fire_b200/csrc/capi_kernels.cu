// extern "C" kernel-level entry points (include/fire_b200.h): host-side argument
// checks, then dispatch to the sm_100a kernels. Nothing here allocates, frees or
// synchronises.
#include "fire_b200.h"

#include <cuda_runtime.h>

#include <cstdint>

#include "device_info.h"
#include "kernels/dense_gemv.h"
#include "kernels/ops.h"
#include "kernels/w4_gemv.h"
#include "kernels/w4_prefill.h"

namespace {

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline int rc(cudaError_t e) { return e == cudaSuccess ? FIRE_B200_OK : static_cast<int>(e); }

}  // namespace

extern "C" {

int fire_b200_abi_version(void) { return FIRE_B200_ABI_VERSION; }

const char* fire_b200_status_string(int status) {
    switch (status) {
    case FIRE_B200_OK: return "ok";
    case FIRE_B200_ERR_INVALID: return "invalid argument";
    case FIRE_B200_ERR_UNSUPPORTED: return "unsupported";
    case FIRE_B200_ERR_NO_DEVICE: return "no CUDA device";
    case FIRE_B200_ERR_STATE: return "invalid state";
    case FIRE_B200_ERR_IO: return "checkpoint I/O or format error";
    case FIRE_B200_ERR_NOMEM: return "out of device memory";
    case FIRE_B200_ERR_DEVICE: return "a kernel reported a failed step (reset the engine)";
    case FIRE_B200_ERR_TIMEOUT: return "host deadline ran out (communicator aborted)";
    default:
        return status > 0 ? cudaGetErrorString(static_cast<cudaError_t>(status)) : "unknown status";
    }
}

int fire_b200_linear_w4(const float* x, const uint8_t* qweight, const float* scales,
                        const uint8_t* zero_points, float* y, int rows, int n, int k,
                        int group_size, void* stream) {
    if (!x || !qweight || !scales || !zero_points || !y) return FIRE_B200_ERR_INVALID;
    if (rows < 1 || n < 1 || k < 2 || (k & 1) || group_size <= 0 || k % group_size)
        return FIRE_B200_ERR_INVALID;
    if (!aligned(x, 4) || !aligned(scales, 4) || !aligned(y, 4)) return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    // The streaming kernels stage x (k floats) in shared memory: k <= 53248 (208 KiB).
    if (rows == 1 && group_size == 128 && k % 128 == 0 && k <= 53248 && aligned(qweight, 16)) {
        fb::W4Args a{};
        a.x = x;
        a.qw = qweight;
        a.scales = scales;
        a.zeros = zero_points;
        a.y = y;
        a.N = n;
        a.K = k;
        return rc(fb::w4g128_gemv_launch(a, fb::kW4Store, sms, S(stream), false));
    }
    return rc(fb::w4_linear_generic_launch(x, qweight, scales, zero_points, y, rows, n, k,
                                           group_size, sms, S(stream)));
}

namespace {
__device__ int g_prefill_status;  // status word for callers that pass none
}  // namespace

size_t fire_b200_linear_w4_prefill_workspace_bytes(int rows, int n, int k) {
    if (rows < 1 || n < 1 || k < 1) return 0;
    return fb::prefill_workspace_bytes(rows, n, k);
}

int fire_b200_linear_w4_prefill(const float* x, const uint8_t* qweight, const float* scales,
                                const uint8_t* zero_points, float* y, int rows, int n, int k,
                                int group_size, void* workspace, size_t workspace_bytes,
                                int* status_dev, void* stream) {
    if (!x || !qweight || !scales || !zero_points || !y || !workspace) return FIRE_B200_ERR_INVALID;
    if (!fb::prefill_supported(rows, n, k, group_size)) return FIRE_B200_ERR_UNSUPPORTED;
    if (workspace_bytes < fb::prefill_workspace_bytes(rows, n, k)) return FIRE_B200_ERR_INVALID;
    if (!aligned(x, 16) || !aligned(y, 16) || !aligned(workspace, 16) || !aligned(qweight, 4) ||
        !aligned(scales, 4))
        return FIRE_B200_ERR_INVALID;
    int* st = status_dev;
    if (st == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_prefill_status) != cudaSuccess) return FIRE_B200_ERR_STATE;
        st = static_cast<int*>(p);
    }
    return rc(fb::prefill_w4_launch(x, qweight, scales, zero_points, y, rows, n, k, workspace, workspace_bytes,
                                    st, S(stream)));
}

int fire_b200_linear_dense(const float* x, const void* weight, int weight_dtype, float scale,
                           float* y, int rows, int n, int k, void* stream) {
    if (!x || !weight || !y || rows < 1 || n < 1 || k < 1) return FIRE_B200_ERR_INVALID;
    if (weight_dtype != FIRE_B200_F32 && weight_dtype != FIRE_B200_BF16) return FIRE_B200_ERR_INVALID;
    if (!aligned(x, 4) || !aligned(y, 4) || !aligned(weight, weight_dtype == FIRE_B200_BF16 ? 2 : 4))
        return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    const bool bf16 = weight_dtype == FIRE_B200_BF16;
    if (rows == 1 && k % 8 == 0 && k <= 53248 && aligned(weight, 16)) {
        fb::DenseArgs a{};
        a.x = x;
        a.w = weight;
        a.scale = scale;
        a.y = y;
        a.N = n;
        a.K = k;
        return rc(fb::dense_gemv_launch(a, bf16, sms, S(stream), false));
    }
    return rc(fb::dense_generic_launch(x, weight, bf16, scale, y, rows, n, k, sms, S(stream)));
}

int fire_b200_rmsnorm(const float* x, const float* w, float* y, int size, float eps, void* stream) {
    if (!x || !w || !y || size < 1 || !(eps >= 0.0f)) return FIRE_B200_ERR_INVALID;
    return rc(fb::rmsnorm_launch(x, w, y, size, eps, S(stream), false));
}

int fire_b200_rmsnorm_rows(const float* x, const float* w, float* y, int rows, int width, float eps,
                           void* stream) {
    if (!x || !w || !y || rows < 1 || width < 1 || !(eps >= 0.0f)) return FIRE_B200_ERR_INVALID;
    return rc(fb::rmsnorm_rows_launch(x, w, y, rows, width, eps, S(stream)));
}

int fire_b200_rope_cache(int head_size, int max_seq, float theta, float* sin_cache, float* cos_cache,
                         void* stream) {
    if (!sin_cache || !cos_cache || head_size < 2 || (head_size & 1) || max_seq < 1 || !(theta > 0.0f))
        return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    return rc(fb::rope_cache_launch(head_size, max_seq, theta, sin_cache, cos_cache, sms, S(stream)));
}

int fire_b200_rope(float* q, float* k, const float* cos_cache, const float* sin_cache, int q_heads,
                   int k_heads, int head_size, int max_seq, int pos, void* stream) {
    if (!q || !k || !cos_cache || !sin_cache || q_heads < 1 || k_heads < 0 || k_heads > q_heads ||
        head_size < 2 || (head_size & 1) || pos < 0 || pos >= max_seq)
        return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    return rc(fb::rope_launch(q, k, cos_cache, sin_cache, q_heads, k_heads, head_size, pos, sms, S(stream)));
}

size_t fire_b200_mha_workspace_bytes(int q_heads, int kv_heads, int head_dim, int capacity) {
    if (q_heads < 1 || kv_heads < 1 || head_dim < 1 || capacity < 1) return 0;
    return fb::attention_workspace_bytes(q_heads, kv_heads, head_dim, capacity);
}

int fire_b200_mha_decode(const float* q, const float* key_cache, const float* value_cache, float* score,
                         float* out, int layers, int capacity, int q_heads, int kv_heads, int head_dim,
                         int layer, int pos, void* workspace, size_t workspace_bytes, void* stream) {
    if (!q || !key_cache || !value_cache || !out || !workspace) return FIRE_B200_ERR_INVALID;
    if (layers < 1 || capacity < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || head_dim > 256 ||
        q_heads % kv_heads || q_heads / kv_heads > 16 || kv_heads > 64)
        return FIRE_B200_ERR_INVALID;
    if (layer < 0 || layer >= layers || pos < 0 || pos >= capacity) return FIRE_B200_ERR_INVALID;
    const size_t need = fb::attention_workspace_bytes(q_heads, kv_heads, head_dim, capacity);
    const int group = q_heads / kv_heads, chunks = (capacity + fb::kAttnChunk - 1) / fb::kAttnChunk;
    const size_t smem = (static_cast<size_t>(group) * (head_dim + fb::kAttnChunk + 2 + chunks) +
                         static_cast<size_t>(fb::kAttnChunk) * (head_dim + 1)) * sizeof(float);
    if (smem > 227 * 1024) return FIRE_B200_ERR_UNSUPPORTED;
    if (workspace_bytes < need || !aligned(workspace, 16)) return FIRE_B200_ERR_INVALID;
    const int max_chunks = (capacity + fb::kAttnChunk - 1) / fb::kAttnChunk;
    const size_t layer_off = static_cast<size_t>(layer) * capacity * kv_heads * head_dim;
    fb::AttnArgs a{};
    a.q = q;
    a.key_cache = key_cache + layer_off;
    a.value_cache = value_cache + layer_off;
    a.out = out;
    a.score = score;
    a.tickets = static_cast<unsigned*>(workspace);
    a.part_ml = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    a.part = a.part_ml + static_cast<size_t>(q_heads) * max_chunks * 2;
    a.state = nullptr;
    a.pos = pos;
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.hd = head_dim;
    a.capacity = capacity;
    a.max_chunks = max_chunks;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    return rc(fb::attention_launch(a, S(stream), false));
}

int fire_b200_embedding(const int32_t* tokens, int count, const void* table, int table_dtype, int vocab,
                        int dim, float* out, void* stream) {
    if (!tokens || !table || !out || count < 1 || vocab < 1 || dim < 1) return FIRE_B200_ERR_INVALID;
    if (table_dtype != FIRE_B200_F32 && table_dtype != FIRE_B200_BF16) return FIRE_B200_ERR_INVALID;
    return rc(fb::embedding_launch(tokens, count, nullptr, table, table_dtype == FIRE_B200_BF16, vocab, dim,
                                   out, S(stream), false));
}

int fire_b200_swiglu(const float* gate, const float* up, float* out, int n, void* stream) {
    if (!gate || !up || !out || n < 1) return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    return rc(fb::swiglu_launch(gate, up, out, n, sms, S(stream)));
}

int fire_b200_add(const float* a, const float* b, float* out, int n, void* stream) {
    if (!a || !b || !out || n < 1) return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    return rc(fb::add_launch(a, b, out, n, sms, S(stream)));
}

size_t fire_b200_argmax_workspace_bytes(void) { return fb::argmax_workspace_bytes(fb::kMaxSms); }

int fire_b200_argmax(const float* x, int64_t n, int64_t* out_index, void* workspace, size_t workspace_bytes,
                     void* stream) {
    if (!x || !out_index || !workspace || n < 1 || n > INT32_MAX) return FIRE_B200_ERR_INVALID;
    if (workspace_bytes < fb::argmax_workspace_bytes(fb::kMaxSms) || !aligned(workspace, 16))
        return FIRE_B200_ERR_INVALID;
    int sms = 0;
    if (int e = fb::device_sms(&sms)) return e;
    if (sms > fb::kMaxSms) sms = fb::kMaxSms;
    return rc(fb::argmax_launch(x, static_cast<int>(n), workspace, sms, out_index, nullptr, nullptr, 0,
                                S(stream), false));
}

}  // extern "C"
