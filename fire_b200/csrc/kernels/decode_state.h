// Device-resident control block of one decode sequence. Kernels read the current
// token and position from it, so a whole decode step can be captured once in a
// CUDA graph and replayed for every token.
#pragma once
#include <stdint.h>

namespace fb {

struct DecodeState {
    int32_t token;  // token consumed by the next step
    int32_t pos;    // its position (== current sequence length)
    int32_t step;   // tokens produced by the device-side greedy loop
    int32_t error;  // non-zero when a kernel rejected the state (e.g. pos >= capacity)
};

}  // namespace fb
