// INT4 group-128 GEMV for single-token decode (M = 1) on sm_100a.
//
// Replaces Fire's GEMV_int4_v1 / matmul_quant_kernel_cu
// (src/op/kernels/cuda/matmul_kernel.cu:230-314) for the .fire v2 layout:
//   qweight u8 [N, K/2] (even k in the low nibble), scales f32 [N, K/128],
//   zero points u8 [N, K/128], x f32 [K], y f32 [N],
//   y[n] = sum_k x[k] * (q[n,k] - z[n,g]) * s[n,g],  g = k / 128.
//
// Design (HBM-bound: 0.539 B per weight, the kernel must issue < ~2.2 ops/weight):
//  * Each lane streams 16-byte chunks (32 nibbles, always inside one group) with
//    L1-bypassing 128-bit loads; a warp owns a tile of R rows, so every x value read
//    from shared memory is reused R times.
//  * Dequantisation is integer-free: (w & (0xF << 4j)) | 0x4B000000 is the float
//    2^23 + q*16^j exactly (j <= 4; nibbles 5..7 are shifted down by 12 bits first),
//    and one packed FP32 add of -(2^23 + z*16^j) leaves (q - z)*16^j exactly. x is
//    staged pre-multiplied by 16^-j, so each packed FMA accumulates x*(q-z) exactly as
//    rounded products; the group scale multiplies each 32-value partial sum.
//  * __fadd2_rn/__ffma2_rn (sm_100 packed FP32) do two weights per instruction.
//  * x is staged once per CTA in shared memory, transposed ([8][K/32] float4) so that
//    lanes reading consecutive chunks hit consecutive 16-byte words (no bank conflicts).
//  * Optional RMSNorm prologue (the norm feeding q/k/v and gate/up), residual-add
//    epilogue (o/down) and SwiGLU epilogue (gate/up packed per tile), so the decode
//    layer needs no separate norm/add/swiglu launches.
//  * Programmatic dependent launch: weight prefetch to L2 is issued before waiting on
//    the producer of x.
#include "common.cuh"
#include "w4_gemv.h"

#include <cstdlib>
#include <cstring>
#include "w4_gemv_common.cuh"
#include "w4_gemv_spec.cuh"

namespace fb {

namespace {

using namespace w4;

struct Stage {
    uint4 w[kW4TileRows];
    float s[kW4TileRows];
    uint32_t z[kW4TileRows];
};

template <int R>
__device__ __forceinline__ void load_stage(Stage& st, const W4Args& a, int row0, int c, size_t row_bytes,
                                           int groups) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int row = min(row0 + r, a.N - 1);
        st.w[r] = ldg_stream(a.qw + static_cast<size_t>(row) * row_bytes + static_cast<size_t>(c) * 16);
        const size_t mi = static_cast<size_t>(row) * groups + (c >> 2);
        st.s[r] = __ldg(a.scales + mi);
        st.z[r] = __ldg(a.zeros + mi);
    }
}

template <int R, int EPI>
__global__ void __launch_bounds__(kThreads, 1) w4g128_gemv_kernel(const W4Args a) {
    extern __shared__ float4 xs[];
    __shared__ float red[32];
    const int K = a.K, N = a.N;
    const int chunks = K >> 5, groups = K >> 7;
    float* xsum = reinterpret_cast<float*>(xs + (K >> 2));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tiles = (N + R - 1) / R;
    const size_t row_bytes = static_cast<size_t>(K) >> 1;
    const uint32_t magic = a.magic;

    // Weights never depend on the previous kernel: start pulling this warp's first
    // tile into L2 before waiting for x.
    const int t_first = blockIdx.x + gridDim.x * warp;
    const int t_stride = gridDim.x * kWarps;
    if (a.prefetch && lane == 0 && t_first < tiles) {
        const int rows = min(R, N - t_first * R);
        prefetch_l2_bulk(a.qw + static_cast<size_t>(t_first) * R * row_bytes, static_cast<uint32_t>(rows * row_bytes));
    }
    pdl_wait();
    stage_x(a, xs, xsum, red);
    __syncthreads();
    pdl_launch_dependents();
    if (t_first >= tiles) return;

    // Work items of this warp: (tile, chunk-slot) in order; one item of look-ahead.
    const int per_tile = (chunks + 31) >> 5;  // chunk slots per lane per tile
    const int my_tiles = (tiles - t_first + t_stride - 1) / t_stride;
    const int items = my_tiles * per_tile;
    Stage cur, nxt;
    {
        const int c = lane;
        if (c < chunks) load_stage<R>(cur, a, t_first * R, c, row_bytes, groups);
    }
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;
    for (int it = 0; it < items; ++it) {
        const int tj = it / per_tile, slot = it - tj * per_tile;
        const int t = t_first + tj * t_stride;
        const int c = lane + 32 * slot;
        if (it + 1 < items) {
            const int tj1 = (it + 1) / per_tile, slot1 = it + 1 - tj1 * per_tile;
            const int c1 = lane + 32 * slot1;
            if (c1 < chunks) load_stage<R>(nxt, a, (t_first + tj1 * t_stride) * R, c1, row_bytes, groups);
        }
        if (c < chunks) {
            float4 xv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) xv[i] = xs[i * chunks + c];
            const float xc = xsum[c];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const float zf = __uint_as_float(cur.z[r] | 0x4B000000u) - 8388608.0f;
                acc[r] = fmaf(cur.s[r], chunk_dot(cur.w[r], xv, -zf * xc, magic), acc[r]);
            }
        }
        if (slot == per_tile - 1) {
            // tile complete: reduce across lanes and apply the epilogue
            const int row0 = t * R;
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);
            if constexpr (EPI == kW4Swiglu) {
                // Tile = R/2 gate rows then the matching R/2 up rows (packed at load time).
                // silu(g) * u as in src/op/kernels/cuda/swiglu_kernel.cu:11-12.
                if (lane < R / 2) {
                    float g = acc[0], u = acc[R / 2];
#pragma unroll
                    for (int j = 1; j < R / 2; ++j)
                        if (lane == j) { g = acc[j]; u = acc[R / 2 + j]; }
                    const float silu = g * 1.0f / (1.0f + expf(-g));
                    a.y[t * (R / 2) + lane] = silu * u;
                }
            } else {
                if (lane < R) {
                    float v = acc[0];
#pragma unroll
                    for (int j = 1; j < R; ++j)
                        if (lane == j) v = acc[j];
                    const int row = row0 + lane;
                    if (row < N) {
                        if constexpr (EPI == kW4Residual) v = a.residual[row] + v;
                        a.y[row] = v;
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        }
        cur = nxt;
    }
}

template <int R, int EPI>
cudaError_t launch_t(const W4Args& a, int num_sms, cudaStream_t stream, bool pdl) {
    auto kern = w4g128_gemv_kernel<R, EPI>;
    const int smem = a.K * 4 + (a.K / 32) * 4;  // x (pre-scaled) + per-chunk sums
    if (smem > 46 * 1024) {  // static shared memory also counts against the 48 KiB default
        // Opt in to exactly the dynamic shared memory this K needs (the limit counts
        // the kernel's static shared memory too).
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
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

cudaError_t w4g128_gemv_launch(const W4Args& a, int epi, int num_sms, cudaStream_t stream,
                               bool pdl) {
    // K-specialised kernels (w4_gemv_spec.cuh) cover the decode shapes; R = 4 rows per
    // lane group when there are enough tiles to fill every warp of the grid, else R = 2.
    // FIRE_B200_W4_PATH=mma selects the integer tensor-core kernel (w4_mma.cu) where it
    // applies (N % 16 == 0); the FP32 streaming kernels below are the default.
    static const bool mma = [] {
        const char* v = std::getenv("FIRE_B200_W4_PATH");
        return v != nullptr && std::strcmp(v, "mma") == 0;
    }();
    if (mma && w4_mma_supported(a)) return w4_mma_launch(a, epi, num_sms, stream, pdl);
    cudaError_t err = cudaSuccess;
    if (epi == kW4Swiglu) {
        if (a.N % kW4TileRows == 0 && a.N >= kW4TileRows && w4_spec_swiglu(a, num_sms, stream, pdl, &err))
            return err;
    } else {
        const int lpr = a.K >= 1024 ? 32 : 16;
        const int g = 32 / lpr;
        const long long tiles4 = (static_cast<long long>(a.N) + 4 * g - 1) / (4 * g);
        const int r = tiles4 >= static_cast<long long>(num_sms) * 12 ? 4 : 2;
        if (a.N >= r * g) {
            const bool done = epi == kW4Residual ? w4_spec_residual(a, r, num_sms, stream, pdl, &err)
                                                 : w4_spec_store(a, r, num_sms, stream, pdl, &err);
            if (done) return err;
        }
    }
    switch (epi) {
    case kW4Residual: return launch_t<kW4TileRows, kW4Residual>(a, num_sms, stream, pdl);
    case kW4Swiglu: return launch_t<kW4TileRows, kW4Swiglu>(a, num_sms, stream, pdl);
    default: return launch_t<kW4TileRows, kW4Store>(a, num_sms, stream, pdl);
    }
}

// ---------------------------------------------------------------------------
// Generic path: any group size, any byte alignment, any number of input rows.
// Same formula as matmul_quant_int4_fp32_naive (matmul_kernel.cu:202-227); one warp
// per output element, lanes stride over k, FP32 accumulation.
__global__ void w4_linear_generic_kernel(const float* __restrict__ x,
                                         const uint8_t* __restrict__ qw,
                                         const float* __restrict__ scales,
                                         const uint8_t* __restrict__ zeros, float* __restrict__ y,
                                         int rows, int N, int K, int group) {
    const int lane = threadIdx.x & 31;
    const long long warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    const long long total = static_cast<long long>(rows) * N;
    const int groups = K / group;
    for (long long o = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
         o < total; o += warps) {
        const int m = static_cast<int>(o / N), n = static_cast<int>(o % N);
        const uint8_t* qrow = qw + static_cast<size_t>(n) * (K / 2);
        const float* xr = x + static_cast<size_t>(m) * K;
        float sum = 0.0f;
        for (int k = lane; k < K; k += 32) {
            const uint8_t b = qrow[k >> 1];
            const int q = (k & 1) ? (b >> 4) : (b & 15);
            const size_t gi = static_cast<size_t>(n) * groups + k / group;
            sum = fmaf(xr[k], static_cast<float>(q - static_cast<int>(zeros[gi])) * scales[gi],
                       sum);
        }
        sum = warp_sum(sum);
        if (lane == 0) y[static_cast<size_t>(m) * N + n] = sum;
    }
}

cudaError_t w4_linear_generic_launch(const float* x, const uint8_t* qw, const float* scales,
                                     const uint8_t* zeros, float* y, int rows, int N, int K,
                                     int group, int num_sms, cudaStream_t stream) {
    const long long warps_needed = static_cast<long long>(rows) * N;
    long long blocks = (warps_needed + 7) / 8;
    const long long cap = static_cast<long long>(num_sms) * 8;
    if (blocks > cap) blocks = cap;
    w4_linear_generic_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        x, qw, scales, zeros, y, rows, N, K, group);
    return cudaGetLastError();
}

}  // namespace fb
