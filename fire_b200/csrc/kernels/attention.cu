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

}  // namespace

size_t attention_workspace_bytes(int q_heads, int kv_heads, int hd, int capacity) {
    (void)kv_heads;
    const size_t chunks = static_cast<size_t>((capacity + kAttnChunk - 1) / kAttnChunk);
    return 256 + static_cast<size_t>(q_heads) * chunks * (static_cast<size_t>(hd) + 2) * sizeof(float);
}

cudaError_t attention_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const int G = a.q_heads / a.kv_heads;
    const size_t smem = (static_cast<size_t>(G) * a.hd + static_cast<size_t>(kAttnChunk) * (a.hd + 1) +
                         static_cast<size_t>(G) * kAttnChunk + 2 * G + static_cast<size_t>(G) * a.max_chunks) *
                        sizeof(float);
    if (smem > 46 * 1024) {  // static shared memory also counts against the 48 KiB default
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.max_chunks), static_cast<unsigned>(a.kv_heads));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attention_kernel, a);
}

}  // namespace fb
