// fire_b200_mha_decode_noalloc: the decode-attention entry point for callers that
// cannot allocate device memory and cannot hand over a workspace.
//
// Some callers only ever pass the tensors they already own: a plug-in behind an
// interface that hands over only the query, the caches, the score buffer and the output
// (no scratch argument), or a host program whose device memory is planned once at
// start-up so that nothing may be allocated afterwards. This entry point serves them by keeping the split-K
// scratch (per-chunk partial outputs and the per-KV-head tickets) in a fixed array
// in device memory that belongs to the library itself.
//
// The array is kNoAllocScratchBytes (4 MiB) in every GPU's memory once the library is
// loaded, until the process exits. In host code its name stands for a host-side
// symbol, not a device address, so the device address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and passed to the
// kernel. The looked-up address is cached for the life of the process: a
// cudaDeviceReset invalidates it, so the entry point must not be used on a device after
// that device was reset. Every call shares the array: calls that overlap on the GPU
// (concurrent streams, or several host threads) race on it and must be serialised by
// the caller.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "fire_b200.h"
#include "kernels/ops.h"

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

// File-scope scratch in device memory: [256 B tickets][per-chunk max/sum][partial outputs].
static __device__ __align__(256) unsigned char g_mha_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kTicketBytes = 256;  // the tickets at the start of the scratch

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_mha_scratch on the current device (looked up on first use).
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FIRE_B200_ERR_NO_DEVICE;
    if (dev < 0 || dev >= kMaxDevices) return FIRE_B200_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_mha_scratch);
        if (e != cudaSuccess) return static_cast<int>(e);
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return FIRE_B200_OK;
}

}  // namespace

extern "C" int fire_b200_mha_decode_noalloc(const float* q, const float* key_cache, const float* value_cache,
                                            float* score, float* out, int layers, int capacity, int q_heads,
                                            int kv_heads, int head_dim, int layer, int pos, void* stream) {
    if (!q || !key_cache || !value_cache || !out) return FIRE_B200_ERR_INVALID;
    if (layers < 1 || capacity < 1 || q_heads < 1 || kv_heads < 1 || head_dim < 1 || head_dim > 256 ||
        q_heads % kv_heads || q_heads / kv_heads > 16 || kv_heads > 64)
        return FIRE_B200_ERR_INVALID;
    if (layer < 0 || layer >= layers || pos < 0 || pos >= capacity) return FIRE_B200_ERR_INVALID;
    // The scratch this shape needs must fit the fixed array: reject, never overrun.
    if (fb::attention_workspace_bytes(q_heads, kv_heads, head_dim, capacity) > kNoAllocScratchBytes)
        return FIRE_B200_ERR_UNSUPPORTED;
    const int group = q_heads / kv_heads, chunks = (capacity + fb::kAttnChunk - 1) / fb::kAttnChunk;
    const size_t smem = (static_cast<size_t>(group) * (head_dim + fb::kAttnChunk + 2 + chunks) +
                         static_cast<size_t>(fb::kAttnChunk) * (head_dim + 1)) * sizeof(float);
    if (smem > 227 * 1024) return FIRE_B200_ERR_UNSUPPORTED;
    void* scratch = nullptr;
    if (const int rc = scratch_address(&scratch)) return rc;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The tickets must start at zero; the array keeps whatever the last call left.
    if (const cudaError_t e = cudaMemsetAsync(scratch, 0, kTicketBytes, s)) return static_cast<int>(e);
    const size_t layer_off = static_cast<size_t>(layer) * capacity * kv_heads * head_dim;
    fb::AttnArgs a{};
    a.q = q;
    a.key_cache = key_cache + layer_off;
    a.value_cache = value_cache + layer_off;
    a.out = out;
    a.score = score;
    a.tickets = static_cast<unsigned*>(scratch);
    a.part_ml = reinterpret_cast<float*>(static_cast<char*>(scratch) + kTicketBytes);
    a.part = a.part_ml + static_cast<size_t>(q_heads) * chunks * 2;
    a.state = nullptr;
    a.pos = pos;
    a.q_heads = q_heads;
    a.kv_heads = kv_heads;
    a.hd = head_dim;
    a.capacity = capacity;
    a.max_chunks = chunks;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    const cudaError_t e = fb::attention_launch(a, s, false);
    return e == cudaSuccess ? FIRE_B200_OK : static_cast<int>(e);
}
