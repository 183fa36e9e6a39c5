// INT4 group-128 Linear for many rows (prefill, M >= 128) on the 5th-generation tensor
// cores: Y[M, N] = X[M, K] . dequant(W)[N, K]^T, FP32 in and out, FP16 operands (X scaled
// per row by a power of two, W = s * (q - z) rounded once), FP32 accumulation in tensor
// memory. Replaces matmul_quant_int4_fp32_naive for rows > 1
// (src/op/kernels/cuda/matmul_kernel.cu:202-227, dispatched from :280-314).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

constexpr int kPrefillBM = 128;  // rows of X per CTA tile (UMMA M)
constexpr int kPrefillBN = 128;  // rows of W per CTA tile (UMMA N)
constexpr int kPrefillBK = 64;   // K per pipeline stage (one 128-byte swizzle row of FP16)

// Shapes the tensor-core path takes: M % 128 == 0, N % 128 == 0, K % 128 == 0, group 128.
bool prefill_supported(int M, int N, int K, int group);
// Scratch of prefill_w4_launch: X in FP16 with its row scales, and W in FP16 [N, K] (the
// two-pass form).
size_t prefill_workspace_bytes(int M, int N, int K);
// Scratch of the GEMM proper: X in FP16 [M, K] and M row scales.
size_t prefill_gemm_workspace_bytes(int M, int K);
// The two halves of the two-pass form, for callers that keep their own weight layout:
// dequantise (.fire rows, or layer-stack items in their row order) into FP16 [N, K], then
// Y = X . W^T. `err` (device int) receives 4 when a group's weights can leave the FP16 range.
cudaError_t prefill_dequant_rows_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K,
                                        void* w_f16, int* err, cudaStream_t s);
cudaError_t prefill_dequant_items_launch(const uint8_t* items, int N, int K, void* w_f16, int* err, cudaStream_t s);
cudaError_t prefill_gemm_launch(const float* x, const void* w_f16, float* y, int M, int N, int K, void* workspace,
                                size_t workspace_bytes, int* err, cudaStream_t s);
// One pass: W (INT4 .fire rows with scales and zero points, or layer-stack items when
// `items`) dequantised into shared memory inside the GEMM pipeline; only X uses the
// workspace (prefill_gemm_workspace_bytes). Bit-identical to dequantise + GEMM.
cudaError_t prefill_w4_fused_launch(const float* x, const uint8_t* w, const float* scales, const uint8_t* zeros,
                                    bool items, float* y, int M, int N, int K, void* workspace,
                                    size_t workspace_bytes, int* err, cudaStream_t s);
// FIRE_B200_PREFILL_FUSED=1 selects the one-pass form (read once per process)
bool prefill_one_pass();
// .fire rows: the two-pass form (or the one-pass form when selected). `err` (device int)
// receives a non-zero code if a bounded wait gives up (1-3) or the weights leave the FP16
// range (4).
cudaError_t prefill_w4_launch(const float* x, const uint8_t* qw, const float* scales, const uint8_t* zeros, float* y,
                              int M, int N, int K, void* workspace, size_t workspace_bytes, int* err,
                              cudaStream_t s);

}  // namespace fb
