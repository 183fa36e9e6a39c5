// INT4 group-128 GEMV specialised on K (the decode shapes of Qwen3 and their
// tensor-parallel shards). Same arithmetic as the runtime-K kernel in w4_gemv.cu;
// with K a compile-time constant the row stride, group count and slot count are
// immediates, the per-slot loop is fully unrolled, and the address of every load is
// a per-tile base plus an immediate offset.
//
// Work split: LPR lanes share a row (LPR = 32, or 16 when a row has fewer than 32
// 16-byte chunks), so a warp covers G = 32/LPR lane groups of R rows each: a warp tile
// is G*R consecutive rows and a lane owns chunk ll + LPR*s of its R rows for slot
// s < SLOTS. Rows are visited word by word so only two float4 of x are live; every
// x value read from shared memory serves R rows. Loads run one slot ahead (across tile
// boundaries too) and the next tile's rows are prefetched into L2 when a tile starts.
#pragma once
#include "w4_gemv_common.cuh"

namespace fb {
namespace w4 {

template <int R>
struct SpecStage {
    uint4 w[R];
    float s[R];
    uint32_t z[R];
};

template <int LPR, int SLOTS, int R, int EPI>
__global__ void __launch_bounds__(kThreads, 1) w4_spec_kernel(const W4Args a) {
    constexpr int CHUNKS = LPR * SLOTS;  // 16-byte chunks per row
    constexpr int K = CHUNKS * 32;
    constexpr int ROW_BYTES = K / 2;
    constexpr int GROUPS = K / 128;
    constexpr int G = 32 / LPR;
    constexpr int WR = G * R;  // rows per warp tile
    extern __shared__ float4 xs[];
    __shared__ float red[32];
    float* xsum = reinterpret_cast<float*>(xs + K / 4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lg = lane / LPR, ll = lane % LPR;
    const int N = a.N;
    const int tiles = (N + WR - 1) / WR;
    const uint32_t magic = a.magic;
    const int t_first = blockIdx.x + gridDim.x * warp;
    const int t_stride = gridDim.x * kWarps;
    // the last tile is shifted back to end at row N (N >= WR); it writes only its own rows
    auto row0_of = [&](int t) { return min(t * WR, N - WR); };

    if (a.prefetch && lane == 0 && t_first < tiles)
        prefetch_l2_bulk(a.qw + static_cast<size_t>(row0_of(t_first)) * ROW_BYTES, WR * ROW_BYTES);
    pdl_wait();
    stage_x(a, xs, xsum, red);
    __syncthreads();
    pdl_launch_dependents();
    if (t_first >= tiles) return;

    auto load = [&](SpecStage<R>& st, int row0, int s) {
        const int c = ll + LPR * s;
        const size_t r = static_cast<size_t>(row0 + lg * R);
        const uint8_t* q = a.qw + r * ROW_BYTES + c * 16;
        const float* sp = a.scales + r * GROUPS + (c >> 2);
        const uint8_t* zp = a.zeros + r * GROUPS + (c >> 2);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            st.w[i] = ldg_stream(q + i * ROW_BYTES);
            st.s[i] = __ldg(sp + i * GROUPS);
            st.z[i] = __ldg(zp + i * GROUPS);
        }
    };
    auto compute = [&](const SpecStage<R>& st, int s, float2* acc) {
        const int c = ll + LPR * s;
        const float xc = xsum[c];
        const float2 nm = make_float2(-8388608.0f, -8388608.0f);
        float2 p[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const float zf = __uint_as_float(st.z[i] | 0x4B000000u) - 8388608.0f;
            p[i] = make_float2(-zf * xc, 0.f);
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float4 xa = xs[(2 * m) * CHUNKS + c], xb = xs[(2 * m + 1) * CHUNKS + c];
#pragma unroll
            for (int i = 0; i < R; ++i) {
                const uint32_t v = m == 0 ? st.w[i].x : m == 1 ? st.w[i].y : m == 2 ? st.w[i].z : st.w[i].w;
                const uint32_t t = v >> 12;
                const float2 d01 = __fadd2_rn(make_float2(nib<0xFu>(v, magic), nib<0xF0u>(v, magic)), nm);
                const float2 d23 = __fadd2_rn(make_float2(nib<0xF00u>(v, magic), nib<0xF000u>(v, magic)), nm);
                const float2 d45 = __fadd2_rn(make_float2(nib<0xF0000u>(v, magic), nib<0xF00u>(t, magic)), nm);
                const float2 d67 = __fadd2_rn(make_float2(nib<0xF000u>(t, magic), nib<0xF0000u>(t, magic)), nm);
                p[i] = __ffma2_rn(make_float2(xa.x, xa.y), d01, p[i]);
                p[i] = __ffma2_rn(make_float2(xa.z, xa.w), d23, p[i]);
                p[i] = __ffma2_rn(make_float2(xb.x, xb.y), d45, p[i]);
                p[i] = __ffma2_rn(make_float2(xb.z, xb.w), d67, p[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = __ffma2_rn(make_float2(st.s[i], st.s[i]), p[i], acc[i]);
    };

    SpecStage<R> b0, b1;
    int t = t_first;
    int row0 = row0_of(t);
    load(b0, row0, 0);
    while (true) {
        const int tn = t + t_stride;
        const bool has_next = tn < tiles;
        const int row0n = has_next ? row0_of(tn) : row0;
        if (a.prefetch && lane == 0 && has_next)
            prefetch_l2_bulk(a.qw + static_cast<size_t>(row0n) * ROW_BYTES, WR * ROW_BYTES);
        float2 acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int s = 0; s < SLOTS; ++s) {
            if ((s & 1) == 0) {
                if (s + 1 < SLOTS) load(b1, row0, s + 1);
                else if (has_next) load(b1, row0n, 0);
                compute(b0, s, acc);
            } else {
                if (s + 1 < SLOTS) load(b0, row0, s + 1);
                else if (has_next) load(b0, row0n, 0);
                compute(b1, s, acc);
            }
        }
        // reduce each row over its LPR lanes
        float v[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            float x = acc[i].x + acc[i].y;
#pragma unroll
            for (int o = LPR / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
            v[i] = x;
        }
        if constexpr (EPI == kW4Swiglu) {
            // tile = R/2 gate rows then the matching R/2 up rows (N % WR == 0, LPR == 32);
            // silu(g) * u as in src/op/kernels/cuda/swiglu_kernel.cu:11-12
            if (lane < R / 2) {
                float g = v[0], u = v[R / 2];
#pragma unroll
                for (int j = 1; j < R / 2; ++j)
                    if (lane == j) { g = v[j]; u = v[R / 2 + j]; }
                const float silu = g * 1.0f / (1.0f + expf(-g));
                a.y[t * (R / 2) + lane] = silu * u;
            }
        } else {
            if (ll < R) {
                float out = v[0];
#pragma unroll
                for (int j = 1; j < R; ++j)
                    if (ll == j) out = v[j];
                const int row = row0 + lg * R + ll;
                if (row >= t * WR) {  // rows before t*WR belong to the previous tile
                    if constexpr (EPI == kW4Residual) out = a.residual[row] + out;
                    a.y[row] = out;
                }
            }
        }
        if (!has_next) break;
        if constexpr ((SLOTS & 1) != 0) b0 = b1;  // odd slot count: the look-ahead landed in b1
        t = tn;
        row0 = row0n;
    }
}

template <int LPR, int SLOTS, int R, int EPI>
cudaError_t spec_launch(const W4Args& a, int num_sms, cudaStream_t stream, bool pdl) {
    constexpr int K = LPR * SLOTS * 32;
    constexpr int WR = (32 / LPR) * R;
    auto kern = w4_spec_kernel<LPR, SLOTS, R, EPI>;
    const int smem = K * 4 + (K / 32) * 4;
    if (smem > 46 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    const int tiles = (a.N + WR - 1) / WR;
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

// Dispatch over the specialised K values for one epilogue and R; returns false when K
// has no specialisation (the caller then uses the runtime-K kernel).
template <int R, int EPI>
bool spec_dispatch(const W4Args& a, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err) {
    switch (a.K) {
    case 1024: *err = spec_launch<32, 1, R, EPI>(a, num_sms, s, pdl); return true;
    case 2048: *err = spec_launch<32, 2, R, EPI>(a, num_sms, s, pdl); return true;
    case 3072: *err = spec_launch<32, 3, R, EPI>(a, num_sms, s, pdl); return true;
    case 4096: *err = spec_launch<32, 4, R, EPI>(a, num_sms, s, pdl); return true;
    case 6144: *err = spec_launch<32, 6, R, EPI>(a, num_sms, s, pdl); return true;
    case 12288: *err = spec_launch<32, 12, R, EPI>(a, num_sms, s, pdl); return true;
    case 512: *err = spec_launch<16, 1, R, EPI>(a, num_sms, s, pdl); return true;
    case 1536: *err = spec_launch<16, 3, R, EPI>(a, num_sms, s, pdl); return true;
    default: return false;
    }
}

}  // namespace w4

// Specialised launch for one epilogue (defined in w4_gemv_spec_*.cu). Returns false
// when no specialisation covers the shape.
bool w4_spec_store(const W4Args& a, int rows_per_lane, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err);
bool w4_spec_residual(const W4Args& a, int rows_per_lane, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err);
bool w4_spec_swiglu(const W4Args& a, int num_sms, cudaStream_t s, bool pdl, cudaError_t* err);

}  // namespace fb
