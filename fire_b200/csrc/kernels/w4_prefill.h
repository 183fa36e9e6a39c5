// INT4 group-128 Linear for many rows (prefill, M >= 64) on the 5th-generation tensor
// cores: Y[M, N] = X[M, K] . dequant(W)[N, K]^T, FP32 in and out, BF16 operands, FP32
// accumulation in tensor memory. Replaces matmul_quant_int4_fp32_naive for rows > 1
// (src/op/kernels/cuda/matmul_kernel.cu:202-227, dispatched from :280-314).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

constexpr int kPrefillBM = 128;  // rows of X per CTA tile (UMMA M)
constexpr int kPrefillBN = 128;  // rows of W per CTA tile (UMMA N)
constexpr int kPrefillBK = 64;   // K per pipeline stage (one 128-byte swizzle row of BF16)

// Shapes the tensor-core path takes: M % 128 == 0, N % 128 == 0, K % 128 == 0, group 128.
bool prefill_supported(int M, int N, int K, int group);
// Scratch: BF16 x_hi and x_lo [M, K] and the dequantised W [N, K].
size_t prefill_workspace_bytes(int M, int N, int K);
// The two halves of prefill_w4_launch, for callers that keep their own weight layout:
// dequantise (.fire rows, or layer-stack items in their row order) into BF16 [N, K], then
// Y = X . W^T with X split into BF16 hi/lo terms (scratch prefill_gemm_workspace_bytes).
size_t prefill_gemm_workspace_bytes(int M, int K);
cudaError_t prefill_dequant_rows_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K,
                                        void* w_bf16, cudaStream_t s);
cudaError_t prefill_dequant_items_launch(const uint8_t* items, int N, int K, void* w_bf16, cudaStream_t s);
cudaError_t prefill_gemm_launch(const float* x, const void* w_bf16, float* y, int M, int N, int K, void* workspace,
                                size_t workspace_bytes, int* err, cudaStream_t s);
// One pass: W (INT4 .fire rows with scales and zero points, or layer-stack items when
// `items`) dequantised into shared memory inside the GEMM pipeline; only X's hi/lo split
// uses the workspace (prefill_gemm_workspace_bytes). Bit-identical to dequantise + GEMM.
cudaError_t prefill_w4_fused_launch(const float* x, const uint8_t* w, const float* scales, const uint8_t* zeros,
                                    bool items, float* y, int M, int N, int K, void* workspace,
                                    size_t workspace_bytes, int* err, cudaStream_t s);
// FIRE_B200_PREFILL_TWO_PASS=1 selects the two-pass form (BF16 scratch in HBM, then the GEMM)
bool prefill_two_pass();
cudaError_t prefill_w4_launch(const float* x, const uint8_t* qw, const float* scales, const uint8_t* zeros, float* y,
                              int M, int N, int K, void* workspace, size_t workspace_bytes, int* err,
                              cudaStream_t s);

}  // namespace fb
