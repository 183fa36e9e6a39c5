// Dense (BF16 or FP32 weight) GEMV: the LM head and Fire's plain Linear at M = 1.
//
// Replaces GEMV_bf16_fp32_v1 / launch_dense_gemv / matmul_kernel_cu
// (src/op/kernels/cuda/matmul_kernel.cu:78-199): y[n] = scale * sum_k x[k] * w[n,k],
// BF16 widened to FP32 before FP32 accumulation.
//
// Same structure as the INT4 GEMV: x staged once per CTA (transposed, so lanes read
// consecutive 16-byte words), each lane streams 16-byte weight chunks with
// L1-bypassing loads, a warp owns R rows to reuse x, packed FP32 FMAs. A BF16 word
// holds two weights; the upper one is the word with its low half cleared and the
// lower one is the word shifted left by 16, both exact FP32 values.
#include "common.cuh"
#include "dense_gemv.h"

namespace fb {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;

template <int R, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) dense_gemv_kernel(const DenseArgs a) {
    extern __shared__ float4 xs[];
    const int K = a.K, N = a.N;
    constexpr int kPerChunk = BF16 ? 8 : 4;      // weights per 16-byte chunk
    constexpr int kF4 = kPerChunk / 4;           // float4 of x per chunk
    const int chunks = K / kPerChunk;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tiles = (N + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(K) * (BF16 ? 2 : 4);

    if (a.prefetch && lane == 0) {
        const int t = blockIdx.x + gridDim.x * warp;
        if (t < tiles) {
            const int rows = min(R, N - t * R);
            prefetch_l2_bulk(static_cast<const uint8_t*>(a.w) + static_cast<size_t>(t) * R * row_bytes,
                             static_cast<uint32_t>(rows * row_bytes));
        }
    }
    pdl_wait();
    float nscale = 1.0f;
    if (a.norm_w != nullptr) {
        __shared__ float red[32];
        float ss = 0.0f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const float v = a.x_add != nullptr ? __fadd_rn(a.x[k], a.x_add[k]) : a.x[k];
            ss = fmaf(v, v, ss);
        }
        ss = block_sum(ss, red);
        nscale = 1.0f / sqrtf(ss / static_cast<float>(K) + a.eps);
    }
    for (int k4 = threadIdx.x; k4 < (K >> 2); k4 += blockDim.x) {
        float4 v = make_float4(load_input(a.x, a.x_add, a.x_sum_out, 4 * k4),
                               load_input(a.x, a.x_add, a.x_sum_out, 4 * k4 + 1),
                               load_input(a.x, a.x_add, a.x_sum_out, 4 * k4 + 2),
                               load_input(a.x, a.x_add, a.x_sum_out, 4 * k4 + 3));
        if (a.norm_w != nullptr) {
            const float* nw = a.norm_w + 4 * k4;
            v = make_float4(v.x * nw[0] * nscale, v.y * nw[1] * nscale, v.z * nw[2] * nscale,
                            v.w * nw[3] * nscale);
        }
        xs[(k4 % kF4) * chunks + k4 / kF4] = v;
    }
    __syncthreads();
    pdl_launch_dependents();

    for (int t = blockIdx.x + gridDim.x * warp; t < tiles; t += gridDim.x * kWarps) {
        const int row0 = t * R;
        float2 acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = make_float2(0.f, 0.f);
        for (int c0 = lane; c0 < chunks; c0 += 64) {
            const int c1 = c0 + 32;
            const bool has1 = c1 < chunks;
            uint4 w0[R], w1[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int row = min(row0 + r, N - 1);
                const uint8_t* wr = static_cast<const uint8_t*>(a.w) + static_cast<size_t>(row) * row_bytes;
                w0[r] = ldg_stream(wr + static_cast<size_t>(c0) * 16);
                if (has1) w1[r] = ldg_stream(wr + static_cast<size_t>(c1) * 16);
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (half == 1 && !has1) break;
                const int c = half ? c1 : c0;
                float4 xv[kF4];
#pragma unroll
                for (int i = 0; i < kF4; ++i) xv[i] = xs[i * chunks + c];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const uint4 w = half ? w1[r] : w0[r];
                    if constexpr (BF16) {
                        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const float2 wf = make_float2(__uint_as_float(ws[m] << 16),
                                                          __uint_as_float(ws[m] & 0xFFFF0000u));
                            const float4 x4 = xv[m >> 1];
                            const float2 xp = (m & 1) ? make_float2(x4.z, x4.w) : make_float2(x4.x, x4.y);
                            acc[r] = __ffma2_rn(xp, wf, acc[r]);
                        }
                    } else {
                        const float4 x4 = xv[0];
                        acc[r] = __ffma2_rn(make_float2(x4.x, x4.y),
                                            make_float2(__uint_as_float(w.x), __uint_as_float(w.y)), acc[r]);
                        acc[r] = __ffma2_rn(make_float2(x4.z, x4.w),
                                            make_float2(__uint_as_float(w.z), __uint_as_float(w.w)), acc[r]);
                    }
                }
            }
        }
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = warp_sum(acc[r].x + acc[r].y);
        if (lane < R) {
            float out = v[0];
#pragma unroll
            for (int j = 1; j < R; ++j)
                if (lane == j) out = v[j];
            const int row = row0 + lane;
            if (row < N) a.y[row] = out * a.scale;
        }
    }
}

// Any K / alignment / row count: one warp per output, scalar loads.
__global__ void dense_generic_kernel(const float* __restrict__ x, const void* __restrict__ w, int bf16,
                                     float scale, float* __restrict__ y, int rows, int N, int K) {
    const int lane = threadIdx.x & 31;
    const long long warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    const long long total = static_cast<long long>(rows) * N;
    for (long long o = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; o < total;
         o += warps) {
        const int m = static_cast<int>(o / N), n = static_cast<int>(o % N);
        const float* xr = x + static_cast<size_t>(m) * K;
        float sum = 0.0f;
        if (bf16) {
            const uint16_t* wr = static_cast<const uint16_t*>(w) + static_cast<size_t>(n) * K;
            for (int k = lane; k < K; k += 32) sum = fmaf(xr[k], bf16_bits_to_float(wr[k]), sum);
        } else {
            const float* wr = static_cast<const float*>(w) + static_cast<size_t>(n) * K;
            for (int k = lane; k < K; k += 32) sum = fmaf(xr[k], wr[k], sum);
        }
        sum = warp_sum(sum);
        if (lane == 0) y[static_cast<size_t>(m) * N + n] = sum * scale;
    }
}

template <int R, bool BF16>
cudaError_t launch_t(const DenseArgs& a, int num_sms, cudaStream_t stream, bool pdl) {
    auto kern = dense_gemv_kernel<R, BF16>;
    const int smem = a.K * 4;
    if (smem > 46 * 1024) {  // static shared memory also counts against the 48 KiB default
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int tiles = (a.N + R - 1) / R;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles < num_sms ? tiles : num_sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

cudaError_t dense_gemv_launch(const DenseArgs& a, bool bf16, int num_sms, cudaStream_t stream, bool pdl) {
    return bf16 ? launch_t<4, true>(a, num_sms, stream, pdl) : launch_t<4, false>(a, num_sms, stream, pdl);
}

cudaError_t dense_generic_launch(const float* x, const void* w, bool bf16, float scale, float* y, int rows,
                                 int N, int K, int num_sms, cudaStream_t stream) {
    long long blocks = (static_cast<long long>(rows) * N + 7) / 8;
    if (blocks > static_cast<long long>(num_sms) * 8) blocks = static_cast<long long>(num_sms) * 8;
    dense_generic_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, w, bf16 ? 1 : 0, scale, y,
                                                                            rows, N, K);
    return cudaGetLastError();
}

}  // namespace fb
