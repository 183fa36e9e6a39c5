// Device memory arena: few large reservations, 256-byte aligned sub-allocations.
//
// Replaces Fire's per-tensor cudaMalloc caching allocator (src/base/alloc_cu.cpp:11-151)
// for the decode engine: weights and runtime buffers are carved out of a handful of
// reservations made once at load / prepare time, so nothing is allocated on the
// decode path. Every sub-allocation is 256-byte aligned (TMA and 128-bit loads need
// 16). Thread-safe; bound to one device.
#pragma once
#include <cstddef>
#include <mutex>
#include <vector>

namespace fb {

class DeviceArena {
  public:
    explicit DeviceArena(int device) : device_(device) {}
    ~DeviceArena();
    DeviceArena(const DeviceArena&) = delete;
    DeviceArena& operator=(const DeviceArena&) = delete;

    // Make one reservation of at least `bytes` so the next allocations fit in it.
    // Returns 0 or a cudaError_t.
    int reserve(size_t bytes);
    // Aligned sub-allocation; grows by a new reservation when needed. nullptr on failure.
    void* alloc(size_t bytes, size_t align = 256);
    size_t used() const;
    size_t reserved() const;
    int device() const { return device_; }

  private:
    struct Block {
        char* base;
        size_t size;
        size_t off;
    };
    int grow_locked(size_t bytes);
    mutable std::mutex mu_;
    int device_;
    std::vector<Block> blocks_;
    size_t used_ = 0;
    size_t reserved_ = 0;
};

}  // namespace fb
