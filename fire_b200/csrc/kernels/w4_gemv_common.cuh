// Shared pieces of the INT4 group-128 GEMV kernels (w4_gemv*.cu): the nibble
// extraction, the x staging with its 16^-p pre-scaling and per-chunk sums.
#pragma once
#include "common.cuh"
#include "w4_gemv.h"

namespace fb {
namespace w4 {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kMagic = 0x4B000000u;  // float 2^23

// (v & mask) | magic in one LOP3 (LUT 0xEA = (a & b) | c). `magic` arrives in a
// register (a kernel argument), so the mask is the instruction's only immediate.
template <uint32_t kMask>
__device__ __forceinline__ float nib(uint32_t v, uint32_t magic) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "n"(kMask), "r"(magic));
    return __uint_as_float(r);
}

// sum_k x'[k] * q[k]*16^p(k) over the 32 weights of one 16-byte chunk, added to
// `init`, where x' = x * 16^-p(k) (pre-scaled in shared memory): each nibble becomes
// the exact float 2^23 + q*16^p and one packed add of -2^23 leaves q*16^p exactly.
__device__ __forceinline__ float chunk_dot(const uint4 w, const float4* xv, float init, uint32_t magic) {
    const float2 nm = make_float2(-8388608.0f, -8388608.0f);
    float2 acc0 = make_float2(init, 0.f), acc1 = make_float2(0.f, 0.f);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const uint32_t v = ws[m], t = v >> 12;
        const float2 d01 = __fadd2_rn(make_float2(nib<0xFu>(v, magic), nib<0xF0u>(v, magic)), nm);
        const float2 d23 = __fadd2_rn(make_float2(nib<0xF00u>(v, magic), nib<0xF000u>(v, magic)), nm);
        const float2 d45 = __fadd2_rn(make_float2(nib<0xF0000u>(v, magic), nib<0xF00u>(t, magic)), nm);
        const float2 d67 = __fadd2_rn(make_float2(nib<0xF000u>(t, magic), nib<0xF0000u>(t, magic)), nm);
        const float4 xa = xv[2 * m], xb = xv[2 * m + 1];
        acc0 = __ffma2_rn(make_float2(xa.x, xa.y), d01, acc0);
        acc1 = __ffma2_rn(make_float2(xa.z, xa.w), d23, acc1);
        acc0 = __ffma2_rn(make_float2(xb.x, xb.y), d45, acc0);
        acc1 = __ffma2_rn(make_float2(xb.z, xb.w), d67, acc1);
    }
    return (acc0.x + acc1.x) + (acc0.y + acc1.y);
}

// Stage x (optionally residual-summed and RMS-normalised) into xs[i][c] scaled by
// 16^-p, and the plain per-chunk sums xsum[c] = sum of the chunk's 32 x values.
__device__ __forceinline__ void stage_x(const W4Args& a, float4* xs, float* xsum, float* red) {
    const int K = a.K, chunks = K >> 5;
    float scale = 1.0f;
    if (a.norm_w != nullptr) {
        float ss = 0.0f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const float v = a.x_add != nullptr ? __fadd_rn(a.x[k], a.x_add[k]) : a.x[k];
            ss = fmaf(v, v, ss);
        }
        ss = block_sum(ss, red);
        scale = 1.0f / sqrtf(ss / static_cast<float>(K) + a.eps);
    }
    // one warp per chunk at a time: lane l < 8 handles float4 l of the chunk
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int c0 = warp * 4; c0 < chunks; c0 += nwarps * 4) {
        const int c = c0 + (lane >> 3), i = lane & 7;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < chunks) {
            const int k = c * 32 + 4 * i;
            v = make_float4(load_input(a.x, a.x_add, a.x_sum_out, k), load_input(a.x, a.x_add, a.x_sum_out, k + 1),
                            load_input(a.x, a.x_add, a.x_sum_out, k + 2), load_input(a.x, a.x_add, a.x_sum_out, k + 3));
            if (a.norm_w != nullptr) {
                const float* w = a.norm_w + k;
                v = make_float4(v.x * w[0] * scale, v.y * w[1] * scale, v.z * w[2] * scale, v.w * w[3] * scale);
            }
        }
        // chunk sum over the 8 lanes of this chunk (fixed order: pairs, then tree)
        float cs = (v.x + v.y) + (v.z + v.w);
        cs += __shfl_xor_sync(0xffffffffu, cs, 1);
        cs += __shfl_xor_sync(0xffffffffu, cs, 2);
        cs += __shfl_xor_sync(0xffffffffu, cs, 4);
        if (c < chunks) {
            if (i == 0) xsum[c] = cs;
            if ((i & 1) == 0) {
                v.y *= 0.0625f;
                v.z *= 0.00390625f;
                v.w *= 0.000244140625f;
            } else {
                v.x *= 1.52587890625e-05f;
                v.y *= 0.00390625f;
                v.z *= 0.000244140625f;
                v.w *= 1.52587890625e-05f;
            }
            xs[i * chunks + c] = v;
        }
    }
}

}  // namespace w4
}  // namespace fb
