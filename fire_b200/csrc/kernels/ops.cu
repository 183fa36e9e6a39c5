// Small decode-path kernels: RMSNorm, RoPE (cache + rotation), the fused
// q/k-norm + RoPE + KV-cache write, embedding gather, SwiGLU, add and argmax.
//
// Arithmetic follows Fire's CPU kernels where that costs nothing (explicit
// __fmul_rn/__fadd_rn where the CPU rounds each product separately), so the
// element-wise results agree with the CPU path bit for bit; reductions use a
// tree order and agree within FP32 rounding.
#include "common.cuh"
#include "decode_state.h"
#include "ops.h"

#include <math.h>

namespace fb {
namespace {

// ------------------------------------------------------------------ RMSNorm
// src/op/kernels/cpu/rmsnorm_kernel.cpp:6-39: y = x * w * (1/sqrt(mean(x^2) + eps)).
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ y, int size, float eps) {
    __shared__ float red[32];
    pdl_wait();
    float ss = 0.0f;
    for (int i = threadIdx.x; i < size; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(size) + eps);
    pdl_launch_dependents();
    for (int i = threadIdx.x; i < size; i += blockDim.x) y[i] = x[i] * w[i] * scale;
}

// src/op/kernels/cpu/rmsnorm_kernel.cpp:41-67: each row of `width` normalised
// independently, the weight shared by all rows. One warp per row.
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                    float* __restrict__ y, int rows, int width, float eps) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* xr = x + static_cast<size_t>(row) * width;
    float* yr = y + static_cast<size_t>(row) * width;
    float ss = 0.0f;
    for (int c = lane; c < width; c += 32) ss = fmaf(xr[c], xr[c], ss);
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(width) + eps);
    for (int c = lane; c < width; c += 32) yr[c] = xr[c] * w[c] * scale;
}

// --------------------------------------------------------------------- RoPE
// Cache [max_seq, head/2] as src/op/kernels/cpu/rope_kernel.cpp:8-24 computes it:
// freq = 1/theta^(2d/head) and angle = freq*pos in FP32; powf/sinf/cosf are evaluated
// in double and rounded once, i.e. correctly rounded in practice, as glibc's are.
__global__ void rope_cache_kernel(int head, int max_seq, float theta, float* __restrict__ sin_c,
                                  float* __restrict__ cos_c) {
    const int half = head / 2;
    const long long total = static_cast<long long>(max_seq) * half;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(i / half), d = static_cast<int>(i % half);
        const float e = 2.0f * static_cast<float>(d) / static_cast<float>(head);
        const float pw = static_cast<float>(pow(static_cast<double>(theta), static_cast<double>(e)));
        const float freq = 1.0f / pw;
        const float ang = freq * static_cast<float>(p);
        sin_c[i] = static_cast<float>(sin(static_cast<double>(ang)));
        cos_c[i] = static_cast<float>(cos(static_cast<double>(ang)));
    }
}

__device__ __forceinline__ void rotate(float& a, float& b, float fcr, float fci) { rope_rotate(a, b, fcr, fci); }

// Half-split rotation of q [q_heads, head] and k [k_heads, head] at `pos`;
// one thread per (head, pair), q heads first.
__global__ void rope_kernel(float* __restrict__ q, float* __restrict__ k,
                            const float* __restrict__ cos_c, const float* __restrict__ sin_c,
                            int q_heads, int k_heads, int head, int pos) {
    const int half = head / 2;
    const long long total = static_cast<long long>(q_heads + k_heads) * half;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int h = static_cast<int>(i / half), d = static_cast<int>(i % half);
        const float fci = sin_c[static_cast<size_t>(pos) * half + d];
        const float fcr = cos_c[static_cast<size_t>(pos) * half + d];
        float* v = h < q_heads ? q + static_cast<size_t>(h) * head
                               : k + static_cast<size_t>(h - q_heads) * head;
        float a = v[d], b = v[d + half];
        rotate(a, b, fcr, fci);
        v[d] = a;
        v[d + half] = b;
    }
}

// Decode-engine fusion of Qwen3Model::forward's q_norm/k_norm, RoPE and KV write
// (src/model/qwen.cpp:222-240): qkv = [q (Hq*128) | k (Hk*128) | v (Hk*128)].
// One warp per head; lane l holds dims 4l..4l+3, its RoPE partner is lane l^16.
__global__ void qk_norm_rope_kv_kernel(QkRopeArgs a) {
    const int lane = threadIdx.x & 31;
    const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int total = a.q_heads + 2 * a.kv_heads;
    pdl_wait();
    if (head >= total) return;
    const int pos = a.state != nullptr ? a.state->pos : a.pos;
    if (pos < 0 || pos >= a.capacity) {
        if (head == 0 && lane == 0 && a.state != nullptr) a.state->error = 1;
        return;
    }
    const float4 v4 = reinterpret_cast<const float4*>(a.qkv + static_cast<size_t>(head) * 128)[lane];
    float v[4] = {v4.x, v4.y, v4.z, v4.w};
    float* dst;
    const size_t slot = (static_cast<size_t>(pos) * a.kv_heads) * 128;
    if (head < a.q_heads + a.kv_heads) {
        const bool is_q = head < a.q_heads;
        const float* nw = is_q ? a.q_norm : a.k_norm;
        float ss = fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], v[3] * v[3])));
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / 128.0f + a.eps);
        const float4 w4 = reinterpret_cast<const float4*>(nw)[lane];
        v[0] = v[0] * w4.x * scale;
        v[1] = v[1] * w4.y * scale;
        v[2] = v[2] * w4.z * scale;
        v[3] = v[3] * w4.w * scale;
        const int d0 = (lane & 15) * 4;  // pair index of v[0]
        const float4 s4 = reinterpret_cast<const float4*>(a.rope_sin + static_cast<size_t>(pos) * 64)[lane & 15];
        const float4 c4 = reinterpret_cast<const float4*>(a.rope_cos + static_cast<size_t>(pos) * 64)[lane & 15];
        const float sn[4] = {s4.x, s4.y, s4.z, s4.w}, cs[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float other = __shfl_xor_sync(0xffffffffu, v[j], 16);
            float a0, b0;
            if (lane < 16) { a0 = v[j]; b0 = other; } else { a0 = other; b0 = v[j]; }
            rotate(a0, b0, cs[j], sn[j]);
            v[j] = lane < 16 ? a0 : b0;
        }
        (void)d0;
        dst = is_q ? a.q_out + static_cast<size_t>(head) * 128
                   : a.key_cache + slot + static_cast<size_t>(head - a.q_heads) * 128;
    } else {
        dst = a.value_cache + slot + static_cast<size_t>(head - a.q_heads - a.kv_heads) * 128;
    }
    reinterpret_cast<float4*>(dst)[lane] = make_float4(v[0], v[1], v[2], v[3]);
    pdl_launch_dependents();
}

// ---------------------------------------------------------------- embedding
// src/op/kernels/cuda/emb_kernel.cu:8-61: one block per token, BF16 widened.
__global__ void embedding_kernel(const int32_t* __restrict__ tokens, DecodeState* state,
                                 const void* __restrict__ table, int bf16, int vocab, int dim,
                                 float* __restrict__ out) {
    pdl_wait();
    const int tok = state != nullptr ? state->token : tokens[blockIdx.x];
    if (tok < 0 || tok >= vocab) {
        if (state != nullptr && threadIdx.x == 0) state->error = 2;
        return;
    }
    float* o = out + static_cast<size_t>(blockIdx.x) * dim;
    if (bf16) {
        const uint16_t* row = static_cast<const uint16_t*>(table) + static_cast<size_t>(tok) * dim;
        for (int c = threadIdx.x; c < dim; c += blockDim.x) o[c] = bf16_bits_to_float(row[c]);
    } else {
        const float* row = static_cast<const float*>(table) + static_cast<size_t>(tok) * dim;
        for (int c = threadIdx.x; c < dim; c += blockDim.x) o[c] = row[c];
    }
    pdl_launch_dependents();
}

// ------------------------------------------------------------- elementwise
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u,
                              float* __restrict__ o, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        const float silu = x * 1.0f / (1.0f + expf(-x));  // swiglu_kernel.cu:11-12
        o[i] = silu * u[i];
    }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ o, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        o[i] = __fadd_rn(a[i], b[i]);
}

// ------------------------------------------------------------------- argmax
// First index of the maximum (cub::ArgMax semantics, argmax_kernel.cu:18-35), no
// allocation and no host synchronisation: each block reduces a strided slice, the
// last block to finish (atomic ticket) folds the per-block partials in block order.
struct ArgmaxPart {
    float v;
    int32_t i;
};

__device__ __forceinline__ void better(float& bv, int& bi, float v, int i) {
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
}

__device__ __forceinline__ void advance_state(DecodeState* state, int32_t* tokens_out, int max_steps, int tok) {
    if (tokens_out != nullptr && state->step < max_steps) tokens_out[state->step] = tok;
    state->step += 1;
    state->token = tok;
    state->pos += 1;
}

__global__ void argmax_kernel(const float* __restrict__ x, int n, ArgmaxPart* parts,
                              unsigned* ticket, int64_t* out_index, DecodeState* state,
                              int32_t* tokens_out, int max_steps, int base_index, ArgmaxPart* best_out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ bool last;
    pdl_wait();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        better(bv, bi, x[i], i);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, ov, oi);
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
        parts[blockIdx.x] = ArgmaxPart{bv, bi};
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (threadIdx.x == 0) {
        float fv = -INFINITY;
        int fi = 0x7fffffff;
        for (int b = 0; b < static_cast<int>(gridDim.x); ++b) {
            const float v = __ldcg(&parts[b].v);
            const int i = __ldcg(&parts[b].i);
            better(fv, fi, v, i);
        }
        if (fi == 0x7fffffff) fi = 0;  // all NaN / -inf: index 0, as a scan from 0 would give
        fi += base_index;
        if (out_index != nullptr) *out_index = fi;
        if (best_out != nullptr) {
            *best_out = ArgmaxPart{fv, fi};
        } else if (state != nullptr) {
            advance_state(state, tokens_out, max_steps, fi);
        }
        *ticket = 0u;  // leave the workspace ready for the next launch
    }
    pdl_launch_dependents();
}

// Tensor-parallel sampling: each rank's (max, global index) pair, gathered in rank
// order, folded with the same first-maximum rule (a lower rank holds lower indices).
__global__ void argmax_select_kernel(const ArgmaxPart* parts, int count, DecodeState* state,
                                     int32_t* tokens_out, int max_steps) {
    pdl_wait();
    if (threadIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = 0; r < count; ++r) better(bv, bi, parts[r].v, parts[r].i);
    if (bi == 0x7fffffff) bi = 0;
    advance_state(state, tokens_out, max_steps, bi);
}

// Sets the decode control block from host values passed as kernel arguments, so a
// host-driven step needs no host buffer that must outlive the launch. The error word is
// left as it is: a failure recorded by an earlier step stays visible (and makes the
// layer-stack kernel return at once) until the engine is reset.
__global__ void set_state_kernel(DecodeState* state, int token, int pos, int step) {
    pdl_wait();
    state->token = token;
    state->pos = pos;
    state->step = step;
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                            cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

unsigned grid_for(long long n, int threads, int num_sms) {
    long long b = (n + threads - 1) / threads;
    const long long cap = static_cast<long long>(num_sms) * 8;
    if (b > cap) b = cap;
    if (b < 1) b = 1;
    return static_cast<unsigned>(b);
}

}  // namespace

cudaError_t rmsnorm_launch(const float* x, const float* w, float* y, int size, float eps,
                           cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3(1), dim3(1024), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, rmsnorm_kernel, x, w, y, size, eps);
}

cudaError_t rmsnorm_rows_launch(const float* x, const float* w, float* y, int rows, int width,
                                float eps, cudaStream_t s) {
    const int warps = 8;
    rmsnorm_rows_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(x, w, y, rows, width, eps);
    return cudaGetLastError();
}

cudaError_t rope_cache_launch(int head, int max_seq, float theta, float* sin_c, float* cos_c,
                              int num_sms, cudaStream_t s) {
    rope_cache_kernel<<<grid_for(static_cast<long long>(max_seq) * (head / 2), 256, num_sms), 256, 0, s>>>(
        head, max_seq, theta, sin_c, cos_c);
    return cudaGetLastError();
}

cudaError_t rope_launch(float* q, float* k, const float* cos_c, const float* sin_c, int q_heads,
                        int k_heads, int head, int pos, int num_sms, cudaStream_t s) {
    rope_kernel<<<grid_for(static_cast<long long>(q_heads + k_heads) * (head / 2), 256, num_sms), 256, 0, s>>>(
        q, k, cos_c, sin_c, q_heads, k_heads, head, pos);
    return cudaGetLastError();
}

cudaError_t qk_norm_rope_kv_launch(const QkRopeArgs& a, cudaStream_t s, bool pdl) {
    const int heads = a.q_heads + 2 * a.kv_heads;
    const int warps = 8;
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3((heads + warps - 1) / warps), dim3(warps * 32), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, qk_norm_rope_kv_kernel, a);
}

cudaError_t embedding_launch(const int32_t* tokens, int count, DecodeState* state, const void* table,
                             bool bf16, int vocab, int dim, float* out, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3(count), dim3(256), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, embedding_kernel, tokens, state, table, bf16 ? 1 : 0, vocab, dim, out);
}

cudaError_t swiglu_launch(const float* g, const float* u, float* o, int n, int num_sms, cudaStream_t s) {
    swiglu_kernel<<<grid_for(n, 256, num_sms), 256, 0, s>>>(g, u, o, n);
    return cudaGetLastError();
}

cudaError_t add_launch(const float* a, const float* b, float* o, int n, int num_sms, cudaStream_t s) {
    add_kernel<<<grid_for(n, 256, num_sms), 256, 0, s>>>(a, b, o, n);
    return cudaGetLastError();
}

size_t argmax_workspace_bytes(int num_sms) {
    return static_cast<size_t>(num_sms) * sizeof(ArgmaxPart) + 256;
}

cudaError_t argmax_launch(const float* x, int n, void* workspace, int num_sms, int64_t* out_index,
                          DecodeState* state, int32_t* tokens_out, int max_steps, cudaStream_t s,
                          bool pdl, int base_index, void* best_out) {
    // layout: [ticket (256 B, zero before first use)][parts]
    unsigned* ticket = static_cast<unsigned*>(workspace);
    ArgmaxPart* parts = reinterpret_cast<ArgmaxPart*>(static_cast<char*>(workspace) + 256);
    unsigned blocks = grid_for(n, 1024, num_sms);
    if (blocks > static_cast<unsigned>(num_sms)) blocks = static_cast<unsigned>(num_sms);
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3(blocks), dim3(1024), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, x, n, parts, ticket, out_index, state, tokens_out,
                              max_steps, base_index, static_cast<ArgmaxPart*>(best_out));
}

cudaError_t argmax_select_launch(const void* parts, int count, DecodeState* state, int32_t* tokens_out,
                                 int max_steps, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3(1), dim3(32), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, argmax_select_kernel, static_cast<const ArgmaxPart*>(parts), count, state,
                              tokens_out, max_steps);
}

cudaError_t set_state_launch(DecodeState* state, int token, int pos, int step, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    auto cfg = make_cfg(dim3(1), dim3(1), 0, s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, set_state_kernel, state, token, pos, step);
}

}  // namespace fb
