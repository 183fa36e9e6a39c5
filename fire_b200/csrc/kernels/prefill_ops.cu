// Row-batched ops of the engine's prefill (many prompt tokens per step): per-token
// q/k RMSNorm + RoPE with the KV-cache write, causal GQA attention over the cache, and
// the SwiGLU of the packed gate/up GEMM output. The per-token arithmetic is the decode
// path's (src/model/qwen.cpp:222-281); only the batching differs.
#include <cuda_fp16.h>

#include "common.cuh"
#include "prefill_ops.h"

namespace fb {
namespace {

// one warp per (token, head): q heads normalised + rotated into q_out, k heads normalised +
// rotated and v copied into the cache rows pos0 + t (kv_cache.cpp:31-73)
__global__ void qk_rope_kv_rows_kernel(const PrefillRowsArgs a) {
    const int lane = threadIdx.x & 31;
    const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int heads = a.q_heads + a.kv_heads;
    if (w >= static_cast<long long>(a.n) * heads) return;
    const int t = static_cast<int>(w / heads), h = static_cast<int>(w % heads);
    const int pos = a.pos0 + t;
    const int row_w = (a.q_heads + 2 * a.kv_heads) * 128;
    const float* row = a.qkv + static_cast<size_t>(t) * row_w;
    const float* srow = a.rope_sin + static_cast<size_t>(pos) * 64;
    const float* crow = a.rope_cos + static_cast<size_t>(pos) * 64;
    if (h < a.q_heads) {
        const float4 r4 = reinterpret_cast<const float4*>(row + h * 128)[lane];
        float v[4] = {r4.x, r4.y, r4.z, r4.w};
        head_norm_rope(v, a.q_norm, srow, crow, a.eps);
        reinterpret_cast<float4*>(a.q_out + static_cast<size_t>(t) * a.q_heads * 128 + h * 128)[lane] =
            make_float4(v[0], v[1], v[2], v[3]);
    } else {
        const int kh = h - a.q_heads;
        const float4 k4 = reinterpret_cast<const float4*>(row + a.q_heads * 128 + kh * 128)[lane];
        const float4 v4 = reinterpret_cast<const float4*>(row + (a.q_heads + a.kv_heads) * 128 + kh * 128)[lane];
        float kv[4] = {k4.x, k4.y, k4.z, k4.w};
        head_norm_rope(kv, a.k_norm, srow, crow, a.eps);
        const size_t dst = static_cast<size_t>(pos) * a.kv_heads * 128 + kh * 128;
        reinterpret_cast<float4*>(a.kcache + dst)[lane] = make_float4(kv[0], kv[1], kv[2], kv[3]);
        reinterpret_cast<float4*>(a.vcache + dst)[lane] = v4;
    }
}

// Causal GQA attention for prompt rows on the tensor cores (mma.sync m16n8k16, FP32
// accumulation). CTA = 16 queries x one KV head, one warp per q head of the group (G warps).
// Per chunk of 64 keys the CTA stages K as FP16 [key][dim] and V transposed as BF16
// [dim][key] in shared memory; each warp takes the chunk in two halves of 32 keys: S = q.K^T
// (FP16 operands: q and k are RMS-normalised per head), the causal mask, the online softmax
// in FP32 (expf, the softmax of mha_kernel.cu:50-144 merged per half chunk), then O += P.V
// (BF16 operands, clear of FP16's range limit for V). q is staged once as FP16. Row strides
// of 68 words (K, q) and 36 words (V^T) make every fragment load conflict-free.
constexpr int kMQ = 16;  // queries per CTA
constexpr int kMK = 64;  // keys per staged chunk
constexpr int kKW = 68;  // K / q row stride in 32-bit words (64 FP16 pairs + 4)
constexpr int kVW = 36;  // V^T row stride in 32-bit words (32 BF16 pairs + 4)

__device__ __forceinline__ uint32_t h2bits(__half2 v) { return *reinterpret_cast<const uint32_t*>(&v); }
__device__ __forceinline__ uint32_t b2bits(__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); }

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int G>
constexpr size_t attn_smem_bytes() {
    return static_cast<size_t>(G * kMQ * kKW + kMK * kKW + 128 * kVW) * 4;
}

// Fragment layout of m16n8k16 (lane = 4 * gr + tg): A rows gr and gr + 8, k pairs tg and
// tg + 4 of the 16; B column (n) gr, k pairs tg and tg + 4; C rows gr / gr + 8, columns
// 2 tg, 2 tg + 1.
template <int G>
__global__ void __launch_bounds__(32 * G, G <= 4 ? 2 : 1) causal_attention_kernel(const PrefillRowsArgs a) {
    extern __shared__ uint32_t smw[];
    uint32_t* qs = smw;                  // [G][kMQ][kKW]  FP16 pairs of q
    uint32_t* ks = qs + G * kMQ * kKW;   // [kMK][kKW]     FP16 pairs of K
    uint32_t* vt = ks + kMK * kKW;       // [128][kVW]     BF16 pairs of V^T (two keys per word)
    const int tid = threadIdx.x, lane = tid & 31, g = tid >> 5;
    const int gr = lane >> 2, tg = lane & 3;
    const int q0 = blockIdx.x * kMQ, h = blockIdx.y, head = h * G + g;
    const int nq = min(kMQ, a.n - q0);
    const size_t qrow = static_cast<size_t>(a.q_heads) * 128;
    // this warp's q rows (its head) as FP16 pairs
    for (int i = lane; i < kMQ * 64; i += 32) {
        const int r = i >> 6, c = i & 63;
        float2 v = make_float2(0.0f, 0.0f);
        if (r < nq) v = *reinterpret_cast<const float2*>(a.q_out + (q0 + r) * qrow + head * 128 + 2 * c);
        qs[(g * kMQ + r) * kKW + c] = h2bits(__floats2half2_rn(v.x, v.y));
    }
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows gr and gr + 8
    const int last = a.pos0 + q0 + nq - 1;  // the last key any row of the CTA sees
    const int qp0 = a.pos0 + q0 + gr, qp1 = qp0 + 8;
    const bool rv0 = gr < nq, rv1 = gr + 8 < nq;
    const size_t rs = static_cast<size_t>(a.kv_heads) * 128;
    const uint32_t* qw = qs + g * kMQ * kKW;
    for (int c0 = 0; c0 <= last; c0 += kMK) {
        const int nk = min(kMK, last + 1 - c0);
        __syncthreads();  // the previous chunk is consumed (and q is staged)
        for (int i = tid; i < kMK * 32; i += 32 * G) {  // K: one float4 of a key row per step
            const int kr = i >> 5, c4 = i & 31;
            float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (kr < nk) kv = *reinterpret_cast<const float4*>(a.kcache + (c0 + kr) * rs + h * 128 + 4 * c4);
            *reinterpret_cast<uint2*>(ks + kr * kKW + 2 * c4) =
                make_uint2(h2bits(__floats2half2_rn(kv.x, kv.y)), h2bits(__floats2half2_rn(kv.z, kv.w)));
        }
        for (int i = tid; i < 32 * 128; i += 32 * G) {  // V^T: keys 2j, 2j + 1 of dim d
            const int j = i >> 7, d = i & 127;
            const float v0 = 2 * j < nk ? a.vcache[(c0 + 2 * j) * rs + h * 128 + d] : 0.0f;
            const float v1 = 2 * j + 1 < nk ? a.vcache[(c0 + 2 * j + 1) * rs + h * 128 + d] : 0.0f;
            vt[d * kVW + j] = b2bits(__floats2bfloat162_rn(v0, v1));  // .x = lower key
        }
        __syncthreads();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int kb = c0 + 32 * half;  // first key of this half
            if (kb > last) break;
            // S = q . K^T for keys kb .. kb + 31: 4 key tiles x 8 dim steps
            float sc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t a0 = qw[gr * kKW + 8 * kk + tg], a1 = qw[(gr + 8) * kKW + 8 * kk + tg];
                const uint32_t a2 = qw[gr * kKW + 8 * kk + 4 + tg], a3 = qw[(gr + 8) * kKW + 8 * kk + 4 + tg];
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const uint32_t* kr = ks + (32 * half + 8 * nt + gr) * kKW + 8 * kk;
                    mma_f16(sc[nt], a0, a1, a2, a3, kr[tg], kr[4 + tg]);
                }
            }
            // causal mask (key <= query position; padded rows see nothing), running maxima
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int kp = kb + 8 * nt + 2 * tg + e;
                    sc[nt][e] = rv0 && kp <= qp0 ? sc[nt][e] * a.scale : -INFINITY;
                    sc[nt][2 + e] = rv1 && kp <= qp1 ? sc[nt][2 + e] * a.scale : -INFINITY;
                    mx0 = fmaxf(mx0, sc[nt][e]);
                    mx1 = fmaxf(mx1, sc[nt][2 + e]);
                }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
            // rescale what was accumulated under the old maximum (1 while nothing is visible)
            const float cr0 = mn0 == -INFINITY ? 1.0f : expf(m0 - mn0);
            const float cr1 = mn1 == -INFINITY ? 1.0f : expf(m1 - mn1);
            m0 = mn0;
            m1 = mn1;
            l0 *= cr0;
            l1 *= cr1;
#pragma unroll
            for (int dt = 0; dt < 16; ++dt) {
                o[dt][0] *= cr0;
                o[dt][1] *= cr0;
                o[dt][2] *= cr1;
                o[dt][3] *= cr1;
            }
            // P = exp(s - m) as BF16 A fragments (0 where masked)
            uint32_t pa[4][2];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const float p00 = sc[nt][0] == -INFINITY ? 0.0f : expf(sc[nt][0] - mn0);
                const float p01 = sc[nt][1] == -INFINITY ? 0.0f : expf(sc[nt][1] - mn0);
                const float p10 = sc[nt][2] == -INFINITY ? 0.0f : expf(sc[nt][2] - mn1);
                const float p11 = sc[nt][3] == -INFINITY ? 0.0f : expf(sc[nt][3] - mn1);
                l0 += p00 + p01;
                l1 += p10 + p11;
                pa[nt][0] = b2bits(__floats2bfloat162_rn(p00, p01));
                pa[nt][1] = b2bits(__floats2bfloat162_rn(p10, p11));
            }
            // O += P . V over keys kb .. kb + 31: 2 key steps x 16 dim tiles
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0], a3 = pa[2 * kk + 1][1];
#pragma unroll
                for (int dt = 0; dt < 16; ++dt) {
                    const uint32_t* vr = vt + (8 * dt + gr) * kVW + 16 * half + 8 * kk;
                    mma_bf16(o[dt], a0, a1, a2, a3, vr[tg], vr[4 + tg]);
                }
            }
        }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (rv0) {
        const float inv = 1.0f / l0;
        float* dst = a.attn_out + (q0 + gr) * qrow + head * 128 + 2 * tg;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
            *reinterpret_cast<float2*>(dst + 8 * dt) = make_float2(o[dt][0] * inv, o[dt][1] * inv);
    }
    if (rv1) {
        const float inv = 1.0f / l1;
        float* dst = a.attn_out + (q0 + gr + 8) * qrow + head * 128 + 2 * tg;
#pragma unroll
        for (int dt = 0; dt < 16; ++dt)
            *reinterpret_cast<float2*>(dst + 8 * dt) = make_float2(o[dt][2] * inv, o[dt][3] * inv);
    }
}

// act[r][8t + i] = silu(gu[r][16t + i]) * gu[r][16t + 8 + i]  (packed gate/up row tiles)
__global__ void swiglu_packed_rows_kernel(const float* __restrict__ gu, float* __restrict__ act, int rows, int f) {
    const long long total = static_cast<long long>(rows) * f;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / f), j = static_cast<int>(i % f);
        const float* src = gu + static_cast<size_t>(r) * 2 * f + (j >> 3) * 16 + (j & 7);
        const float g = src[0];
        const float silu = g * 1.0f / (1.0f + expf(-g));  // swiglu_kernel.cu:11-12
        act[i] = silu * src[8];
    }
}

}  // namespace

cudaError_t qk_rope_kv_rows_launch(const PrefillRowsArgs& a, cudaStream_t s) {
    const long long warps = static_cast<long long>(a.n) * (a.q_heads + a.kv_heads);
    const int block = 256;
    qk_rope_kv_rows_kernel<<<static_cast<int>((warps * 32 + block - 1) / block), block, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t causal_attention_launch(const PrefillRowsArgs& a, cudaStream_t s) {
    if (a.kv_heads <= 0 || a.q_heads % a.kv_heads != 0 || a.n <= 0) return cudaErrorInvalidValue;
    const int G = a.q_heads / a.kv_heads;
    void (*kern)(const PrefillRowsArgs) = nullptr;
    size_t smem = 0;
    switch (G) {
    case 1: kern = causal_attention_kernel<1>; smem = attn_smem_bytes<1>(); break;
    case 2: kern = causal_attention_kernel<2>; smem = attn_smem_bytes<2>(); break;
    case 4: kern = causal_attention_kernel<4>; smem = attn_smem_bytes<4>(); break;
    case 5: kern = causal_attention_kernel<5>; smem = attn_smem_bytes<5>(); break;
    case 8: kern = causal_attention_kernel<8>; smem = attn_smem_bytes<8>(); break;
    default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>((a.n + kMQ - 1) / kMQ), static_cast<unsigned>(a.kv_heads));
    kern<<<grid, 32 * G, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t swiglu_packed_rows_launch(const float* gu, float* act, int rows, int f, int num_sms, cudaStream_t s) {
    const long long total = static_cast<long long>(rows) * f;
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(num_sms) * 16));
    swiglu_packed_rows_kernel<<<grid, 256, 0, s>>>(gu, act, rows, f);
    return cudaGetLastError();
}

}  // namespace fb
