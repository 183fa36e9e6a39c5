// Device memory pool behind include/fire_b200_alloc.h (Fire's GPU DeviceAllocator,
// src/base/alloc_cu.cpp:11-151, rebuilt thread-safe with returned errors).
//
// Blocks are cudaMalloc'd in size classes and cached per device after release, so a
// steady allocate/release pattern (Fire's per-call scratch tensors) stops reaching the
// CUDA allocator after the first round. One registry maps every block this pool made to
// its device, class and state; all calls take one mutex (allocation is off the decode
// hot path, which allocates nothing).
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "fire_b200_alloc.h"

namespace {

constexpr size_t kGranule = 256;
constexpr size_t kSmall = 4096;
constexpr size_t kHugeFrom = size_t(64) << 20;
constexpr size_t kHugeGranule = size_t(2) << 20;
constexpr size_t kTrimAbove = size_t(1) << 30;  // cached free bytes per device before a trim
constexpr int kMaxDevices = 64;

// Size class of a request: 256-byte granules up to 4 KiB, four classes per power of two
// up to 64 MiB, 2 MiB granules above.
size_t size_class(size_t b) {
    if (b == 0) b = 1;
    if (b <= kSmall) return (b + kGranule - 1) / kGranule * kGranule;
    if (b > kHugeFrom) return (b + kHugeGranule - 1) / kHugeGranule * kHugeGranule;
    size_t p = kSmall;
    while (p * 2 < b) p *= 2;  // p < b <= 2p
    const size_t step = p / 4;
    return p + (b - p + step - 1) / step * step;
}

struct Block {
    int device;
    size_t bytes;
    bool busy;
};

struct DevicePool {
    std::unordered_map<size_t, std::vector<void*>> free_blocks;  // class -> cached blocks
    size_t reserved = 0, in_use = 0, free_bytes = 0, live = 0;
};

std::mutex g_mu;
std::unordered_map<void*, Block> g_blocks;
DevicePool g_pools[kMaxDevices];

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// free every cached block of `device` (g_mu held)
int trim_locked(int device) {
    DevicePool& p = g_pools[device];
    DeviceGuard g(device);
    int rc = FIRE_B200_OK;
    for (auto& kv : p.free_blocks) {
        for (void* ptr : kv.second) {
            const cudaError_t e = cudaFree(ptr);
            if (e != cudaSuccess && rc == FIRE_B200_OK) rc = static_cast<int>(e);
            g_blocks.erase(ptr);
            p.reserved -= kv.first;
            p.free_bytes -= kv.first;
        }
        kv.second.clear();
    }
    return rc;
}

}  // namespace

extern "C" {

int fire_b200_device_alloc(size_t bytes, void** out) {
    if (out == nullptr) return FIRE_B200_ERR_INVALID;
    *out = nullptr;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return FIRE_B200_ERR_NO_DEVICE;
    }
    if (dev < 0 || dev >= kMaxDevices) return FIRE_B200_ERR_UNSUPPORTED;
    const size_t cls = size_class(bytes);
    std::lock_guard<std::mutex> lk(g_mu);
    DevicePool& p = g_pools[dev];
    auto it = p.free_blocks.find(cls);
    if (it != p.free_blocks.end() && !it->second.empty()) {
        void* ptr = it->second.back();
        it->second.pop_back();
        g_blocks[ptr].busy = true;
        p.free_bytes -= cls;
        p.in_use += cls;
        ++p.live;
        *out = ptr;
        return FIRE_B200_OK;
    }
    void* ptr = nullptr;
    cudaError_t e = cudaMalloc(&ptr, cls);
    if (e == cudaErrorMemoryAllocation && p.free_bytes > 0) {
        (void)cudaGetLastError();
        trim_locked(dev);  // the cache held the room: give it back and try once more
        e = cudaMalloc(&ptr, cls);
    }
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? FIRE_B200_ERR_NOMEM : static_cast<int>(e);
    }
    g_blocks[ptr] = Block{dev, cls, true};
    p.reserved += cls;
    p.in_use += cls;
    ++p.live;
    *out = ptr;
    return FIRE_B200_OK;
}

int fire_b200_device_release(void* ptr) {
    if (ptr == nullptr) return FIRE_B200_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_blocks.find(ptr);
    if (it == g_blocks.end() || !it->second.busy) return FIRE_B200_ERR_INVALID;
    Block& b = it->second;
    DevicePool& p = g_pools[b.device];
    b.busy = false;
    p.free_blocks[b.bytes].push_back(ptr);
    p.in_use -= b.bytes;
    p.free_bytes += b.bytes;
    --p.live;
    if (p.free_bytes > kTrimAbove) return trim_locked(b.device);
    return FIRE_B200_OK;
}

int fire_b200_device_memset_zero(void* ptr, size_t bytes, void* stream, int sync) {
    if (ptr == nullptr && bytes > 0) return FIRE_B200_ERR_INVALID;
    if (bytes == 0) return FIRE_B200_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ptr, 0, bytes, s);
    if (e == cudaSuccess && sync) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) (void)cudaGetLastError();
    return static_cast<int>(e);
}

int fire_b200_device_memcpy(const void* src, void* dst, size_t bytes, int kind, void* stream, int sync) {
    if ((src == nullptr || dst == nullptr) && bytes > 0) return FIRE_B200_ERR_INVALID;
    if (kind < FIRE_B200_CPU2GPU || kind > FIRE_B200_GPU2GPU) return FIRE_B200_ERR_INVALID;
    if (bytes == 0) return FIRE_B200_OK;
    if (kind == FIRE_B200_CPU2CPU) {
        std::memcpy(dst, src, bytes);
        return FIRE_B200_OK;
    }
    const cudaMemcpyKind k = kind == FIRE_B200_CPU2GPU   ? cudaMemcpyHostToDevice
                             : kind == FIRE_B200_GPU2CPU ? cudaMemcpyDeviceToHost
                                                         : cudaMemcpyDeviceToDevice;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, k, s);
    if (e == cudaSuccess && sync) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) (void)cudaGetLastError();
    return static_cast<int>(e);
}

int fire_b200_device_pool_stats(int device, size_t* reserved, size_t* in_use, size_t* live_blocks) {
    if (device < 0 || device >= kMaxDevices) return FIRE_B200_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    const DevicePool& p = g_pools[device];
    if (reserved) *reserved = p.reserved;
    if (in_use) *in_use = p.in_use;
    if (live_blocks) *live_blocks = p.live;
    return FIRE_B200_OK;
}

int fire_b200_device_pool_trim(int device) {
    if (device < 0 || device >= kMaxDevices) return FIRE_B200_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    return trim_locked(device);
}

}  // extern "C"
