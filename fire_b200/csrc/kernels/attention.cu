// Single-token GQA decode attention over the FP32 KV cache (split-K "flash decoding").
//
// Replaces mha_kernel_cu_fp32 + softmax_gpu (src/op/kernels/cuda/mha_kernel.cu:9-144):
//   score[h,t] = (q_h . k_t) / sqrt(hd),  p = softmax(score[h, 0..pos]),
//   out[h] = sum_t p[h,t] v_t,  kv head = h / (q_heads / kv_heads).
// Cache layout [layers, capacity, kv_heads, hd] (src/model/kv_cache.cpp:12-29).
//
// One CTA per (64-key chunk, KV head). All q heads of a KV group share one read of
// the chunk's K rows (staged in shared memory with a padded row stride, so the
// per-key dot products are bank-conflict free) and V rows (read once, coalesced).
// Each CTA leaves (max, sum, unnormalised P.V) per q head; the last CTA of a KV head
// (atomic ticket, no waiting) folds the partials in chunk order, so the result is
// deterministic. The position may come from device memory, so the launch can be
// captured once and replayed for every token; chunks past the position exit at once.
#include "common.cuh"
#include "ops.h"

#include <math.h>

namespace fb {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxGroup = 16;  // q heads per KV head

__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnArgs a) {
    extern __shared__ float sm[];
    __shared__ bool last;
    const int hd = a.hd, G = a.q_heads / a.kv_heads;
    const int c = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = kThreads >> 5;
    float* qs = sm;                                  // [G][hd]
    float* ks = qs + G * hd;                         // [64][hd+1]
    float* ps = ks + kAttnChunk * (hd + 1);          // [G][64]
    float* ml = ps + G * kAttnChunk;                 // [G][2]
    float* wc = ml + 2 * G;                          // [G][max_chunks] combine factors

    pdl_wait();
    const int pos = a.state != nullptr ? a.state->pos : a.pos;
    if (pos < 0 || pos >= a.capacity) return;
    const int n = pos + 1;
    const int nchunks = (n + kAttnChunk - 1) / kAttnChunk;
    if (c >= nchunks) return;
    const int t0 = c * kAttnChunk;
    const int T = min(kAttnChunk, n - t0);
    const size_t row_stride = static_cast<size_t>(a.kv_heads) * hd;
    const float* kbase = a.key_cache + static_cast<size_t>(t0) * row_stride + static_cast<size_t>(h) * hd;
    const float* vbase = a.value_cache + static_cast<size_t>(t0) * row_stride + static_cast<size_t>(h) * hd;

    for (int i = tid; i < G * hd; i += kThreads) qs[i] = a.q[static_cast<size_t>(h) * G * hd + i];
    for (int i = tid; i < T * hd; i += kThreads) {
        const int t = i / hd, d = i - t * hd;
        ks[t * (hd + 1) + d] = kbase[static_cast<size_t>(t) * row_stride + d];
    }
    __syncthreads();

    // scores (mha_kernel.cu:71-79 / cpu mha_kernel.cpp:189-201)
    for (int j = tid; j < G * T; j += kThreads) {
        const int g = j / T, t = j - g * T;
        const float* qv = qs + g * hd;
        const float* kv = ks + t * (hd + 1);
        float dot = 0.0f;
        for (int d = 0; d < hd; ++d) dot = fmaf(qv[d], kv[d], dot);
        const float s = dot * a.scale;
        ps[g * kAttnChunk + t] = s;
        if (a.score != nullptr)
            a.score[static_cast<size_t>(h * G + g) * a.capacity + t0 + t] = s;
    }
    __syncthreads();

    // chunk-local softmax statistics
    for (int g = warp; g < G; g += nwarps) {
        float* pg = ps + g * kAttnChunk;
        float m = -INFINITY;
        for (int t = lane; t < T; t += 32) m = fmaxf(m, pg[t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < T; t += 32) {
            const float e = expf(pg[t] - m);
            pg[t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * g] = m; ml[2 * g + 1] = l; }
    }
    __syncthreads();

    // unnormalised P.V for every q head of the group
    for (int d = tid; d < hd; d += kThreads) {
        float acc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.0f;
        for (int t = 0; t < T; ++t) {
            const float v = vbase[static_cast<size_t>(t) * row_stride + d];
#pragma unroll
            for (int g = 0; g < kMaxGroup; ++g)
                if (g < G) acc[g] = fmaf(ps[g * kAttnChunk + t], v, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g)
            if (g < G) a.part[(static_cast<size_t>(h * G + g) * a.max_chunks + c) * hd + d] = acc[g];
    }
    if (tid < G) {
        float* dst = a.part_ml + (static_cast<size_t>(h * G + tid) * a.max_chunks + c) * 2;
        dst[0] = ml[2 * tid];
        dst[1] = ml[2 * tid + 1];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&a.tickets[h], 1u) == static_cast<unsigned>(nchunks - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();

    // combine: M = max m_c, S = sum l_c e^(m_c - M), out = sum part_c e^(m_c - M) / S
    for (int g = warp; g < G; g += nwarps) {
        const float* pm = a.part_ml + static_cast<size_t>(h * G + g) * a.max_chunks * 2;
        float M = -INFINITY;
        for (int cc = lane; cc < nchunks; cc += 32) M = fmaxf(M, __ldcg(pm + 2 * cc));
        M = warp_max(M);
        float S = 0.0f;
        for (int cc = lane; cc < nchunks; cc += 32) {
            const float f = expf(__ldcg(pm + 2 * cc) - M);
            wc[g * a.max_chunks + cc] = f;
            S += __ldcg(pm + 2 * cc + 1) * f;
        }
        S = warp_sum(S);
        if (lane == 0) { ml[2 * g] = M; ml[2 * g + 1] = S; }
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += kThreads) {
        const int g = i / hd, d = i - g * hd;
        const float* pp = a.part + static_cast<size_t>(h * G + g) * a.max_chunks * hd + d;
        float o = 0.0f;
        for (int cc = 0; cc < nchunks; ++cc) o = fmaf(__ldcg(pp + static_cast<size_t>(cc) * hd), wc[g * a.max_chunks + cc], o);
        a.out[static_cast<size_t>(h * G + g) * hd + d] = o / ml[2 * g + 1];
    }
    if (a.score != nullptr) {
        for (int i = tid; i < G * n; i += kThreads) {
            const int g = i / n, t = i - g * n;
            float* sp = a.score + static_cast<size_t>(h * G + g) * a.capacity + t;
            *sp = expf(__ldcg(sp) - ml[2 * g]) / ml[2 * g + 1];
        }
    }
    if (tid == 0) a.tickets[h] = 0u;
    pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// head_dim 128 (every Qwen3 profile): 128 keys per CTA, 256 threads. All K and V rows
// of the chunk are copied to shared memory with cp.async at once (16 bytes per lane,
// one 512-byte row per warp instruction), so each SM has its whole share of the cache
// in flight; scores, softmax and P.V then run from shared memory. K rows use a
// 132-float stride so the per-key float4 reads of a quarter warp hit distinct banks.
constexpr int kChunk128 = 128;
constexpr int kThreads128 = 256;
constexpr int kKStride = 132;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__global__ void __launch_bounds__(kThreads128) attention128_kernel(const AttnArgs a) {
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    __shared__ bool last;
    const int G = a.q_heads / a.kv_heads;
    const int c = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = kThreads128 >> 5;
    float* ks = sm;                              // [128][132]
    float* vs = ks + kChunk128 * kKStride;       // [128][128]
    float* qs = vs + kChunk128 * 128;            // [G][128]
    float* ps = qs + G * 128;                    // [G][128]
    float* ml = ps + G * kChunk128;              // [G][2]
    float* wc = ml + 2 * G;                      // [G][max_chunks]

    pdl_wait();
    const int pos = a.state != nullptr ? a.state->pos : a.pos;
    if (pos < 0 || pos >= a.capacity) return;
    const int n = pos + 1;
    const int nchunks = (n + kChunk128 - 1) / kChunk128;
    if (c >= nchunks) return;
    const int t0 = c * kChunk128;
    const int T = min(kChunk128, n - t0);
    const size_t row_stride = static_cast<size_t>(a.kv_heads) * 128;
    const float* kbase = a.key_cache + static_cast<size_t>(t0) * row_stride + static_cast<size_t>(h) * 128;
    const float* vbase = a.value_cache + static_cast<size_t>(t0) * row_stride + static_cast<size_t>(h) * 128;
    const bool fused = a.qkv != nullptr;
    // in fused mode the current token's row (pos, the last of the last chunk) is not in
    // the cache yet: it is computed below instead of copied
    const bool holds_pos = fused && c == nchunks - 1;
    const int T_copy = holds_pos ? T - 1 : T;
    for (int t = warp; t < T_copy; t += nwarps) {
        cp_async16(ks + t * kKStride + 4 * lane, kbase + static_cast<size_t>(t) * row_stride + 4 * lane);
        cp_async16(vs + t * 128 + 4 * lane, vbase + static_cast<size_t>(t) * row_stride + 4 * lane);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (!fused) {
        for (int i = tid; i < G * 128; i += kThreads128) qs[i] = a.q[static_cast<size_t>(h) * G * 128 + i];
    } else {
        const float* srow = a.rope_sin + static_cast<size_t>(pos) * 64;
        const float* crow = a.rope_cos + static_cast<size_t>(pos) * 64;
        for (int g = warp; g < G; g += nwarps) {
            const float4 r4 = reinterpret_cast<const float4*>(a.qkv + static_cast<size_t>(h * G + g) * 128)[lane];
            float v[4] = {r4.x, r4.y, r4.z, r4.w};
            head_norm_rope(v, a.q_norm, srow, crow, a.eps);
            reinterpret_cast<float4*>(qs + g * 128)[lane] = make_float4(v[0], v[1], v[2], v[3]);
        }
        if (holds_pos && warp == nwarps - 1) {
            const size_t qd = static_cast<size_t>(a.q_heads) * 128, kvd = static_cast<size_t>(a.kv_heads) * 128;
            const float4 k4 = reinterpret_cast<const float4*>(a.qkv + qd + static_cast<size_t>(h) * 128)[lane];
            const float4 v4 = reinterpret_cast<const float4*>(a.qkv + qd + kvd + static_cast<size_t>(h) * 128)[lane];
            float kv[4] = {k4.x, k4.y, k4.z, k4.w};
            head_norm_rope(kv, a.k_norm, srow, crow, a.eps);
            const float4 kr = make_float4(kv[0], kv[1], kv[2], kv[3]);
            const int tp = T - 1;  // == pos - t0
            reinterpret_cast<float4*>(ks + tp * kKStride)[lane] = kr;
            reinterpret_cast<float4*>(vs + tp * 128)[lane] = v4;
            // KVCache::write (src/model/kv_cache.cpp:31-73): keep them for later steps
            float* kdst = const_cast<float*>(kbase) + static_cast<size_t>(tp) * row_stride;
            float* vdst = const_cast<float*>(vbase) + static_cast<size_t>(tp) * row_stride;
            reinterpret_cast<float4*>(kdst)[lane] = kr;
            reinterpret_cast<float4*>(vdst)[lane] = v4;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    // scores: one (head, key) dot product per thread and pass
    for (int j = tid; j < G * kChunk128; j += kThreads128) {
        const int g = j / kChunk128, t = j % kChunk128;
        if (t < T) {
            const float4* kv = reinterpret_cast<const float4*>(ks + t * kKStride);
            const float4* qv = reinterpret_cast<const float4*>(qs + g * 128);
            float dot = 0.0f;
#pragma unroll 8
            for (int d4 = 0; d4 < 32; ++d4) {
                const float4 k4 = kv[d4], q4 = qv[d4];
                dot = fmaf(q4.x, k4.x, dot);
                dot = fmaf(q4.y, k4.y, dot);
                dot = fmaf(q4.z, k4.z, dot);
                dot = fmaf(q4.w, k4.w, dot);
            }
            const float sc = dot * a.scale;
            ps[g * kChunk128 + t] = sc;
            if (a.score != nullptr) a.score[static_cast<size_t>(h * G + g) * a.capacity + t0 + t] = sc;
        }
    }
    __syncthreads();
    for (int g = warp; g < G; g += nwarps) {
        float* pg = ps + g * kChunk128;
        float m = -INFINITY;
        for (int t = lane; t < T; t += 32) m = fmaxf(m, pg[t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < kChunk128; t += 32) {
            const float e = t < T ? expf(pg[t] - m) : 0.0f;
            pg[t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { ml[2 * g] = m; ml[2 * g + 1] = l; }
    }
    __syncthreads();
    // unnormalised P.V: thread = (head, dim)
    for (int j = tid; j < G * 128; j += kThreads128) {
        const int g = j >> 7, d = j & 127;
        const float* pg = ps + g * kChunk128;
        float o0 = 0.f, o1 = 0.f;
        int t = 0;
        for (; t + 1 < T; t += 2) {
            o0 = fmaf(pg[t], vs[t * 128 + d], o0);
            o1 = fmaf(pg[t + 1], vs[(t + 1) * 128 + d], o1);
        }
        if (t < T) o0 = fmaf(pg[t], vs[t * 128 + d], o0);
        a.part[(static_cast<size_t>(h * G + g) * a.max_chunks + c) * 128 + d] = o0 + o1;
    }
    if (tid < G) {
        float* dst = a.part_ml + (static_cast<size_t>(h * G + tid) * a.max_chunks + c) * 2;
        dst[0] = ml[2 * tid];
        dst[1] = ml[2 * tid + 1];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(&a.tickets[h], 1u) == static_cast<unsigned>(nchunks - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int g = warp; g < G; g += nwarps) {
        const float* pm = a.part_ml + static_cast<size_t>(h * G + g) * a.max_chunks * 2;
        float M = -INFINITY;
        for (int cc = lane; cc < nchunks; cc += 32) M = fmaxf(M, __ldcg(pm + 2 * cc));
        M = warp_max(M);
        float S = 0.0f;
        for (int cc = lane; cc < nchunks; cc += 32) {
            const float f = expf(__ldcg(pm + 2 * cc) - M);
            wc[g * a.max_chunks + cc] = f;
            S += __ldcg(pm + 2 * cc + 1) * f;
        }
        S = warp_sum(S);
        if (lane == 0) { ml[2 * g] = M; ml[2 * g + 1] = S; }
    }
    __syncthreads();
    for (int j = tid; j < G * 128; j += kThreads128) {
        const int g = j >> 7, d = j & 127;
        const float* pp = a.part + static_cast<size_t>(h * G + g) * a.max_chunks * 128 + d;
        float o = 0.0f;
#pragma unroll 4
        for (int cc = 0; cc < nchunks; ++cc)
            o = fmaf(__ldcg(pp + static_cast<size_t>(cc) * 128), wc[g * a.max_chunks + cc], o);
        a.out[static_cast<size_t>(h * G + g) * 128 + d] = o / ml[2 * g + 1];
    }
    if (a.score != nullptr) {
        for (int i = tid; i < G * n; i += kThreads128) {
            const int g = i / n, t = i - g * n;
            float* sp = a.score + static_cast<size_t>(h * G + g) * a.capacity + t;
            *sp = expf(__ldcg(sp) - ml[2 * g]) / ml[2 * g + 1];
        }
    }
    if (tid == 0) a.tickets[h] = 0u;
    pdl_launch_dependents();
}

}  // namespace

size_t attention_workspace_bytes(int q_heads, int kv_heads, int hd, int capacity) {
    (void)kv_heads;
    const size_t chunks = static_cast<size_t>((capacity + kAttnChunk - 1) / kAttnChunk);
    return 256 + static_cast<size_t>(q_heads) * chunks * (static_cast<size_t>(hd) + 2) * sizeof(float);
}

cudaError_t attention_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int G = a.q_heads / a.kv_heads;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cfg.stream = s;
    const bool aligned16 = (reinterpret_cast<uintptr_t>(a.key_cache) % 16 == 0) &&
                           (reinterpret_cast<uintptr_t>(a.value_cache) % 16 == 0);
    if (a.hd == 128 && aligned16) {
        // partial slots are laid out with a.max_chunks (64-key chunks) as the stride;
        // 128-key chunks use the first half of them
        const size_t smem = (static_cast<size_t>(kChunk128) * (kKStride + 128) + static_cast<size_t>(G) * (128 + kChunk128 + 2) +
                             static_cast<size_t>(G) * a.max_chunks) * sizeof(float);
        if (smem <= 227 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(attention128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            cfg.gridDim = dim3(static_cast<unsigned>((a.capacity + kChunk128 - 1) / kChunk128),
                               static_cast<unsigned>(a.kv_heads));
            cfg.blockDim = dim3(kThreads128);
            cfg.dynamicSmemBytes = smem;
            return cudaLaunchKernelEx(&cfg, attention128_kernel, a);
        }
    }
    if (a.qkv != nullptr) return cudaErrorInvalidValue;  // the fused prologue exists for hd 128 only
    const size_t smem = (static_cast<size_t>(G) * a.hd + static_cast<size_t>(kAttnChunk) * (a.hd + 1) +
                         static_cast<size_t>(G) * kAttnChunk + 2 * G + static_cast<size_t>(G) * a.max_chunks) *
                        sizeof(float);
    if (smem > 46 * 1024) {  // static shared memory also counts against the 48 KiB default
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    cfg.gridDim = dim3(static_cast<unsigned>(a.max_chunks), static_cast<unsigned>(a.kv_heads));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    return cudaLaunchKernelEx(&cfg, attention_kernel, a);
}

}  // namespace fb
