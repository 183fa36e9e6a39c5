// Row-batched ops of the engine's prefill (many prompt tokens per step): per-token
// q/k RMSNorm + RoPE with the KV-cache write, causal GQA attention over the cache, and
// the SwiGLU of the packed gate/up GEMM output. The per-token arithmetic is the decode
// path's (src/model/qwen.cpp:222-281); only the batching differs.
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

// Causal GQA attention for prompt rows: CTA = (16 queries, one KV head), 16 warps, each
// warp 4 (query, q head) pairs for G <= 4 (G x 16 / 16 in general); keys stream through
// shared memory in chunks of 64 (K rows padded to 132 floats: conflict-free float4 reads
// down a column), online softmax per pair (mha_kernel.cu:50-144's softmax, merged per
// chunk), lane d4 owns dims 4*d4..4*d4+3 of the output.
constexpr int kQB = 16;     // queries per CTA
constexpr int kKC = 64;     // keys per chunk
constexpr int kKS = 132;    // padded K row stride (floats)
constexpr int kAttnWarps = 16;

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32) causal_attention_kernel(const PrefillRowsArgs a) {
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    float* qs = sm;                         // [kQB][G][128]
    float* ks = qs + kQB * G * 128;         // [kKC][kKS]
    float* vs = ks + kKC * kKS;             // [kKC][128]
    float* ps = vs + kKC * 128;             // [warps][pairs/warp][kKC]
    constexpr int kPairs = kQB * G;
    constexpr int kPerWarp = (kPairs + kAttnWarps - 1) / kAttnWarps;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int q0 = blockIdx.x * kQB, h = blockIdx.y;
    const int nq = min(kQB, a.n - q0);
    // stage the block's rotated q rows of this KV head's G q heads
    for (int i = tid; i < kQB * G * 32; i += blockDim.x) {
        const int qi = i / (G * 32), rem = i % (G * 32), g = rem / 32, d4 = rem % 32;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < nq)
            v = reinterpret_cast<const float4*>(a.q_out + static_cast<size_t>(q0 + qi) * a.q_heads * 128 +
                                                static_cast<size_t>(h * G + g) * 128)[d4];
        reinterpret_cast<float4*>(qs + (qi * G + g) * 128)[d4] = v;
    }
    float m[kPerWarp], l[kPerWarp];
    float4 acc[kPerWarp];
#pragma unroll
    for (int p = 0; p < kPerWarp; ++p) {
        m[p] = -INFINITY;
        l[p] = 0.0f;
        acc[p] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int last_pos = a.pos0 + q0 + nq - 1;
    const size_t row_stride = static_cast<size_t>(a.kv_heads) * 128;
    for (int c0 = 0; c0 <= last_pos; c0 += kKC) {
        const int nk = min(kKC, last_pos + 1 - c0);
        __syncthreads();  // previous chunk consumed (and q staged)
        for (int i = tid; i < kKC * 32; i += blockDim.x) {
            const int kr = i >> 5, d4 = i & 31;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (kr < nk) {
                const size_t off = static_cast<size_t>(c0 + kr) * row_stride + static_cast<size_t>(h) * 128;
                kv = reinterpret_cast<const float4*>(a.kcache + off)[d4];
                vv = reinterpret_cast<const float4*>(a.vcache + off)[d4];
            }
            reinterpret_cast<float4*>(ks + kr * kKS)[d4] = kv;
            reinterpret_cast<float4*>(vs + kr * 128)[d4] = vv;
        }
        __syncthreads();
#pragma unroll
        for (int p = 0; p < kPerWarp; ++p) {
            const int pair = warp * kPerWarp + p;
            if (pair >= kPairs) break;
            const int qi = pair / G;
            const int qpos = a.pos0 + q0 + qi;
            // scores of keys lane and lane + 32
            const float4* q4 = reinterpret_cast<const float4*>(qs + pair * 128);
            const float4* k0 = reinterpret_cast<const float4*>(ks + lane * kKS);
            const float4* k1 = reinterpret_cast<const float4*>(ks + (lane + 32) * kKS);
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
            for (int d4 = 0; d4 < 32; ++d4) {
                const float4 q = q4[d4], x0 = k0[d4], x1 = k1[d4];
                s0 = fmaf(q.x, x0.x, fmaf(q.y, x0.y, fmaf(q.z, x0.z, fmaf(q.w, x0.w, s0))));
                s1 = fmaf(q.x, x1.x, fmaf(q.y, x1.y, fmaf(q.z, x1.z, fmaf(q.w, x1.w, s1))));
            }
            const bool ok0 = qi < nq && lane < nk && c0 + lane <= qpos;
            const bool ok1 = qi < nq && lane + 32 < nk && c0 + lane + 32 <= qpos;
            s0 = ok0 ? s0 * a.scale : -INFINITY;
            s1 = ok1 ? s1 * a.scale : -INFINITY;
            const float cm = warp_max(fmaxf(s0, s1));
            const float mn = fmaxf(m[p], cm);
            if (mn == -INFINITY) continue;  // no visible key yet for this pair
            const float e0 = ok0 ? expf(s0 - mn) : 0.0f, e1 = ok1 ? expf(s1 - mn) : 0.0f;
            const float corr = m[p] == -INFINITY ? 0.0f : expf(m[p] - mn);
            l[p] = l[p] * corr + warp_sum(e0 + e1);
            m[p] = mn;
            float* pw = ps + (warp * kPerWarp + p) * kKC;
            pw[lane] = e0;
            pw[lane + 32] = e1;
            __syncwarp();
            float4 o = make_float4(acc[p].x * corr, acc[p].y * corr, acc[p].z * corr, acc[p].w * corr);
            for (int kr = 0; kr < nk; ++kr) {
                const float pr = pw[kr];
                const float4 v = reinterpret_cast<const float4*>(vs + kr * 128)[lane];
                o.x = fmaf(pr, v.x, o.x);
                o.y = fmaf(pr, v.y, o.y);
                o.z = fmaf(pr, v.z, o.z);
                o.w = fmaf(pr, v.w, o.w);
            }
            acc[p] = o;
            __syncwarp();
        }
    }
#pragma unroll
    for (int p = 0; p < kPerWarp; ++p) {
        const int pair = warp * kPerWarp + p;
        if (pair >= kPairs) break;
        const int qi = pair / G, g = pair % G;
        if (qi >= nq) continue;
        const float inv = 1.0f / l[p];
        reinterpret_cast<float4*>(a.attn_out + static_cast<size_t>(q0 + qi) * a.q_heads * 128 +
                                  static_cast<size_t>(h * G + g) * 128)[lane] =
            make_float4(acc[p].x * inv, acc[p].y * inv, acc[p].z * inv, acc[p].w * inv);
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
    const int G = a.q_heads / a.kv_heads;
    auto smem_for = [&](int g) {
        const int per_warp = (kQB * g + kAttnWarps - 1) / kAttnWarps;
        return static_cast<size_t>(kQB * g * 128 + kKC * kKS + kKC * 128 + kAttnWarps * per_warp * kKC) * 4;
    };
    void (*kern)(const PrefillRowsArgs) = nullptr;
    switch (G) {
    case 1: kern = causal_attention_kernel<1>; break;
    case 2: kern = causal_attention_kernel<2>; break;
    case 4: kern = causal_attention_kernel<4>; break;
    case 5: kern = causal_attention_kernel<5>; break;
    case 8: kern = causal_attention_kernel<8>; break;
    default: return cudaErrorInvalidValue;
    }
    const size_t smem = smem_for(G);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>((a.n + kQB - 1) / kQB), static_cast<unsigned>(a.kv_heads));
    kern<<<grid, kAttnWarps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t swiglu_packed_rows_launch(const float* gu, float* act, int rows, int f, int num_sms, cudaStream_t s) {
    const long long total = static_cast<long long>(rows) * f;
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(num_sms) * 16));
    swiglu_packed_rows_kernel<<<grid, 256, 0, s>>>(gu, act, rows, f);
    return cudaGetLastError();
}

}  // namespace fb
