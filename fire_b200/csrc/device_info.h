// Per-device launch facts (SM count), queried once per device and cached.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

#include "fire_b200.h"

namespace fb {

// Upper bound on SMs any supported GPU has; sizes the fixed argmax workspace.
constexpr int kMaxSms = 256;

// SM count of the current device; returns FIRE_B200_OK or an error status.
inline int device_sms(int* out) {
    static std::atomic<int> cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FIRE_B200_ERR_NO_DEVICE;
    if (dev >= 0 && dev < 64) {
        const int v = cache[dev].load(std::memory_order_relaxed);
        if (v > 0) {
            *out = v;
            return FIRE_B200_OK;
        }
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
        return FIRE_B200_ERR_NO_DEVICE;
    if (dev >= 0 && dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
    *out = sms;
    return FIRE_B200_OK;
}

}  // namespace fb
