// Shared device helpers for the fire_b200 sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fb {

constexpr int kWarp = 32;

// Programmatic dependent launch (PDL). A kernel launched with the
// programmatic-stream-serialization attribute may start while the previous
// kernel on the stream is still running; pdl_wait() blocks until that kernel has
// finished and its writes are visible. Both are no-ops without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Streaming 128-bit load that bypasses L1 (weights are read exactly once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Ask L2 to start fetching [p, p+bytes) (bulk prefetch, no destination).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; every thread gets the result. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nwarps ? red[lane] : 0.0f;
    return warp_sum(t);
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Element i of the GEMV input: x[i] (+ x_add[i]); CTA 0 also records the sum.
__device__ __forceinline__ float load_input(const float* x, const float* x_add, float* x_sum_out, int i) {
    float v = x[i];
    if (x_add != nullptr) {
        v = __fadd_rn(v, x_add[i]);
        if (x_sum_out != nullptr && blockIdx.x == 0) x_sum_out[i] = v;
    }
    return v;
}

// a' = a*cos - b*sin, b' = a*sin + b*cos with every product rounded separately, as
// Fire's CPU RoPE computes it (src/op/kernels/cpu/rope_kernel.cpp:38-49).
__device__ __forceinline__ void rope_rotate(float& a, float& b, float fcr, float fci) {
    const float a0 = a, b0 = b;
    a = __fsub_rn(__fmul_rn(a0, fcr), __fmul_rn(b0, fci));
    b = __fadd_rn(__fmul_rn(a0, fci), __fmul_rn(b0, fcr));
}

// One 128-wide head held by a warp, lane l owning dims 4l..4l+3: per-head RMSNorm with
// weights w4 = nw[4l..4l+3] (rmsnorm_kernel.cpp:41-67) then half-split RoPE with
// s4 / c4 = sin_row / cos_row [4(l & 15)..+3] of this position (rope_kernel.cpp:26-52);
// the RoPE partner of lane l is lane l^16. The weights and rows come in as arguments
// so a caller can load them early.
__device__ __forceinline__ void head_norm_rope_loaded(float (&v)[4], float4 w4, float4 s4, float4 c4, float eps) {
    const int lane = threadIdx.x & 31;
    float ss = fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], v[3] * v[3])));
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / 128.0f + eps);
    v[0] = v[0] * w4.x * scale;
    v[1] = v[1] * w4.y * scale;
    v[2] = v[2] * w4.z * scale;
    v[3] = v[3] * w4.w * scale;
    const float sn[4] = {s4.x, s4.y, s4.z, s4.w}, cs[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, v[j], 16);
        float a0, b0;
        if (lane < 16) { a0 = v[j]; b0 = other; } else { a0 = other; b0 = v[j]; }
        rope_rotate(a0, b0, cs[j], sn[j]);
        v[j] = lane < 16 ? a0 : b0;
    }
}

__device__ __forceinline__ void head_norm_rope(float (&v)[4], const float* nw, const float* sin_row,
                                               const float* cos_row, float eps) {
    const int lane = threadIdx.x & 31;
    head_norm_rope_loaded(v, reinterpret_cast<const float4*>(nw)[lane], reinterpret_cast<const float4*>(sin_row)[lane & 15],
                          reinterpret_cast<const float4*>(cos_row)[lane & 15], eps);
}

}  // namespace fb
