// Internal launch interface of the INT4 GEMV kernels (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

enum W4Epilogue : int { kW4Store = 0, kW4Residual = 1, kW4Swiglu = 2 };

// Rows per warp tile. The SwiGLU epilogue expects gate/up packed per tile:
// kW4TileRows/2 gate rows followed by the matching kW4TileRows/2 up rows.
constexpr int kW4TileRows = 4;

struct W4Args {
    const float* x;          // [K] input (the raw hidden state when norm_w is set)
    const float* x_add;      // optional [K]: the input is x + x_add (residual fused into the prologue)
    float* x_sum_out;        // optional [K]: CTA 0 stores x + x_add here (the new residual stream)
    const float* norm_w;     // optional RMSNorm weight [K] applied to the (summed) input
    float eps;
    const uint8_t* qw;       // [N, K/2], 16-byte aligned
    const float* scales;     // [N, K/128]
    const uint8_t* zeros;    // [N, K/128]
    float* y;                // [N] (SwiGLU: [N/2])
    const float* residual;   // residual epilogue: y = residual + W x
    int N, K;                // K % 128 == 0
    int prefetch;            // issue an L2 bulk prefetch of each warp's first tile
    uint32_t magic = 0x4B000000u;  // float 2^23 bits, passed at run time (keeps one LOP3 per weight)
    int* err = nullptr;      // optional device word set non-zero if a bounded wait gives up
};

cudaError_t w4g128_gemv_launch(const W4Args& a, int epilogue, int num_sms, cudaStream_t stream,
                               bool pdl);
// Tensor-core path (w4_mma.cu): exact u8 x s8 integer MMAs on fixed-point digits of x.
bool w4_mma_supported(const W4Args& a);
cudaError_t w4_mma_launch(const W4Args& a, int epilogue, int num_sms, cudaStream_t stream, bool pdl);

cudaError_t w4_linear_generic_launch(const float* x, const uint8_t* qw, const float* scales,
                                     const uint8_t* zeros, float* y, int rows, int N, int K,
                                     int group, int num_sms, cudaStream_t stream);

}  // namespace fb
