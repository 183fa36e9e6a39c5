// Internal launch interface of the dense (BF16/FP32 weight) GEMV kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

struct DenseArgs {
    const float* x;   // [K] (the raw hidden state when norm_w is set)
    const float* x_add;   // optional [K]: the input is x + x_add
    float* x_sum_out;     // optional [K]: CTA 0 stores x + x_add here
    const float* norm_w;  // optional RMSNorm weight [K] applied to x first
    float eps;
    const void* w;    // [N, K] BF16 bits or FP32, 16-byte aligned, K % 8 == 0
    float scale;
    float* y;         // [N]
    int N, K;
    int prefetch;
};

cudaError_t dense_gemv_launch(const DenseArgs& a, bool bf16, int num_sms, cudaStream_t stream, bool pdl);
cudaError_t dense_generic_launch(const float* x, const void* w, bool bf16, float scale, float* y, int rows,
                                 int N, int K, int num_sms, cudaStream_t stream);

}  // namespace fb
