#include "engine/arena.h"

#include <cuda_runtime.h>

namespace fb {

namespace {
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};
constexpr size_t kMinBlock = size_t(64) << 20;
}  // namespace

DeviceArena::~DeviceArena() {
    DeviceGuard g(device_);
    for (auto& b : blocks_) cudaFree(b.base);
}

int DeviceArena::grow_locked(size_t bytes) {
    DeviceGuard g(device_);
    const size_t size = bytes < kMinBlock ? kMinBlock : bytes;
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, size);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return static_cast<int>(e);
    }
    blocks_.push_back(Block{static_cast<char*>(p), size, 0});
    reserved_ += size;
    return 0;
}

int DeviceArena::reserve(size_t bytes) {
    std::lock_guard<std::mutex> lk(mu_);
    if (!blocks_.empty() && blocks_.back().size - blocks_.back().off >= bytes) return 0;
    return grow_locked(bytes);
}

void* DeviceArena::alloc(size_t bytes, size_t align) {
    if (bytes == 0) bytes = 1;
    std::lock_guard<std::mutex> lk(mu_);
    for (int attempt = 0; attempt < 2; ++attempt) {
        if (!blocks_.empty()) {
            Block& b = blocks_.back();
            const size_t off = (b.off + align - 1) / align * align;
            if (off + bytes <= b.size) {
                b.off = off + bytes;
                used_ += bytes;
                return b.base + off;
            }
        }
        if (attempt == 0 && grow_locked(bytes + align) != 0) return nullptr;
    }
    return nullptr;
}

size_t DeviceArena::used() const {
    std::lock_guard<std::mutex> lk(mu_);
    return used_;
}

size_t DeviceArena::reserved() const {
    std::lock_guard<std::mutex> lk(mu_);
    return reserved_;
}

}  // namespace fb
