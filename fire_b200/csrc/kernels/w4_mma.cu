// INT4 group-128 GEMV (M = 1) on the tensor cores with exact integer products.
//
// Same contract as the streaming kernels in w4_gemv.cu / w4_gemv_spec.cuh
// (Fire's GEMV_int4_v1, src/op/kernels/cuda/matmul_kernel.cu:230-267):
//   y[n] = sum_g s[n,g] * sum_{k in g} x[k] * (q[n,k] - z[n,g]).
// The FP32 SIMT formulation costs ~2.5 instructions per weight, about what the issue
// rate allows at HBM speed; this one costs ~0.8:
//  * x is staged once per CTA as fixed point per 128-wide group: x_fix = rint(x * 2^e_g)
//    with |x_fix| < 2^26 (27 bits against the group maximum, finer than FP32's 24),
//    split into four signed base-128 digits, each an int8 column of the MMA B operand.
//  * the packed nibbles become the u8 A operand with one AND per four weights:
//    (w & 0x0F0F0F0F) holds the even nibbles of a word, ((w >> 4) & 0x0F0F0F0F) the odd
//    ones; the k order inside an MMA is permuted to match (a sum does not care) and the
//    digit layout in shared memory follows the same permutation.
//  * mma.sync m16n8k32 u8 x s8 -> s32 gives sum_k q_k * digit_k exactly per group; the
//    digits recombine in FP32, z * sum_k x_fix[k] is subtracted (exact integer sum), and
//    the group scale s * 2^-e_g is applied per group.
// A warp owns a 16-row tile and a share of its K groups; partial sums of a tile are
// combined in shared memory in a fixed order (deterministic). Weights stream with
// L1-bypassing 128-bit loads, one item of look-ahead, issued before the PDL wait.
#include "common.cuh"
#include "w4_gemv.h"

namespace fb {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;     // rows per MMA tile
constexpr int kMaxParts = 16;
static_assert(kTile % kW4TileRows == 0, "gate/up packing must tile the MMA rows");

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Geometry {
    int groups;     // K / 128
    int items;      // groups / GPI
    int nt;         // tiles per CTA
    int parts;      // K parts per tile
    int tiles;      // N / 16
};

// Stage x: residual sum / RMSNorm as the other GEMVs, then per group the fixed-point
// digits (shared memory [group][digit n][quad c][mma j][8 bytes]) and {sum x_fix, 2^-e}.
__device__ void stage_digits(const W4Args& a, unsigned char* xd, float2* xg, float* red) {
    const int K = a.K, groups = K >> 7;
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
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int g = warp; g < groups; g += nwarps) {
        const int k0 = g * 128 + 4 * lane;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = load_input(a.x, a.x_add, a.x_sum_out, k0 + e);
            if (a.norm_w != nullptr) v[e] = v[e] * a.norm_w[k0 + e] * scale;
        }
        float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        m = warp_max(m);
        // m in [2^ex, 2^(ex+1)): x * 2^(25-ex) has magnitude < 2^26
        const int ex = static_cast<int>((__float_as_uint(m) >> 23) & 0xFF) - 127;
        int sh = 25 - ex;
        if (m == 0.0f || sh > 126) sh = 126;
        const float up = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);     // 2^sh
        const float down = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);   // 2^-sh (sh <= 126)
        int fx[4];
        long long sum = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            fx[e] = __float2int_rn(v[e] * up);
            sum += fx[e];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) xg[g] = make_float2(static_cast<float>(sum), down);
        // k_local = 4*lane + e: quad c = lane/8, mma j = (lane/2)%4, p = 4*(lane%2) + e;
        // p even -> b0 byte p/2, p odd -> b1 byte p/2
        const int c = lane >> 3, j = (lane >> 1) & 3, hi = lane & 1;
        int r[4] = {fx[0], fx[1], fx[2], fx[3]};
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            int d[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                d[e] = ((r[e] + 64) & 127) - 64;
                r[e] = (r[e] - d[e]) >> 7;
            }
            unsigned char* slot = xd + (((static_cast<size_t>(g) * 4 + n) * 4 + c) * 4 + j) * 8;
            // e = 0, 2 -> b0 (even p); e = 1, 3 -> b1 (odd p); this lane owns bytes 2*hi, 2*hi+1
            const uint16_t b0 = static_cast<uint16_t>((d[0] & 0xFF) | ((d[2] & 0xFF) << 8));
            const uint16_t b1 = static_cast<uint16_t>((d[1] & 0xFF) | ((d[3] & 0xFF) << 8));
            *reinterpret_cast<uint16_t*>(slot + 2 * hi) = b0;
            *reinterpret_cast<uint16_t*>(slot + 4 + 2 * hi) = b1;
        }
    }
}

template <int GPI>
struct Item {
    uint4 w[2][GPI];     // rows g, g+8; one 16-byte chunk per group
    float s[2][GPI];
    uint32_t z[2][GPI];
};

template <int GPI, int EPI>
__global__ void __launch_bounds__(kThreads, 1) w4_mma_kernel(const W4Args a, const Geometry geo) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ float red[32];
    const int groups = geo.groups;
    unsigned char* xd = smem;                                                   // groups * 512
    float2* xg = reinterpret_cast<float2*>(smem + static_cast<size_t>(groups) * 512);
    float* part = reinterpret_cast<float*>(xg + groups);                        // [nt][parts][16]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, c = lane & 3;
    const size_t row_bytes = static_cast<size_t>(a.K) >> 1;
    const int tile0 = blockIdx.x * geo.nt;
    const int nt = min(geo.nt, geo.tiles - tile0);
    const int units = nt * geo.parts;
    // this warp's units u = warp, warp + 16, ...: tile u / parts, K part u % parts
    const int my_units = warp < units ? (units - warp + kWarps - 1) / kWarps : 0;
    auto part_range = [&](int p, int* i0, int* i1) {
        *i0 = (p * geo.items) / geo.parts;
        *i1 = ((p + 1) * geo.items) / geo.parts;
    };
    // flattened item sequence of this warp: (unit ordinal, item index)
    auto load_item = [&](Item<GPI>& it, int tile, int item) {
        const size_t r0 = static_cast<size_t>(tile) * kTile + gq;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const size_t row = r0 + h * 8;
            const uint8_t* q = a.qw + row * row_bytes;
#pragma unroll
            for (int gi = 0; gi < GPI; ++gi) {
                const int g = item * GPI + gi;
                it.w[h][gi] = ldg_stream(q + static_cast<size_t>(g) * 64 + c * 16);
                it.s[h][gi] = __ldg(a.scales + row * groups + g);
                it.z[h][gi] = __ldg(a.zeros + row * groups + g);
            }
        }
    };

    // first item (weights do not depend on the previous kernel)
    int u_ord = 0, it_idx = 0, it_end = 0, cur_tile = 0, cur_part = 0;
    Item<GPI> cur, nxt;
    if (my_units > 0) {
        const int u = warp;
        cur_tile = tile0 + u / geo.parts;
        cur_part = u % geo.parts;
        part_range(cur_part, &it_idx, &it_end);
        if (it_idx < it_end) load_item(cur, cur_tile, it_idx);
    }
    pdl_wait();
    stage_digits(a, xd, xg, red);
    for (int i = threadIdx.x; i < nt * geo.parts * kTile; i += kThreads) part[i] = 0.0f;
    __syncthreads();
    pdl_launch_dependents();

    // per-lane digit weights: quad c = 0 holds digit columns 0,1; c = 1 holds 2,3
    const float w_even = c == 0 ? 1.0f : 16384.0f;
    const float w_odd = c == 0 ? 128.0f : 2097152.0f;
    const float zmul = c == 0 ? 1.0f : 0.0f;
    const bool has_b = gq < 4;  // lanes holding digit n = gq
    float acc0 = 0.0f, acc1 = 0.0f;  // rows gq, gq+8 (this lane's digit share)
    while (u_ord < my_units) {
        // look-ahead: next item of this unit, or the first item of the next unit
        int n_ord = u_ord, n_idx = it_idx + 1, n_end = it_end, n_tile = cur_tile, n_part = cur_part;
        if (n_idx >= it_end) {
            n_ord = u_ord + 1;
            if (n_ord < my_units) {
                const int u = warp + n_ord * kWarps;
                n_tile = tile0 + u / geo.parts;
                n_part = u % geo.parts;
                part_range(n_part, &n_idx, &n_end);
            }
        }
        const bool more = n_ord < my_units && n_idx < n_end;
        if (more) load_item(nxt, n_tile, n_idx);
        if (it_idx < it_end) {
#pragma unroll
            for (int gi = 0; gi < GPI; ++gi) {
                const int g = it_idx * GPI + gi;
                uint4 b4[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
                if (has_b) {
                    const uint4* src = reinterpret_cast<const uint4*>(xd + ((static_cast<size_t>(g) * 4 + gq) * 4 + c) * 32);
                    b4[0] = src[0];
                    b4[1] = src[1];
                }
                const uint32_t bb[8] = {b4[0].x, b4[0].y, b4[0].z, b4[0].w, b4[1].x, b4[1].y, b4[1].z, b4[1].w};
                int d[4] = {0, 0, 0, 0};
                const uint32_t wg[4] = {cur.w[0][gi].x, cur.w[0][gi].y, cur.w[0][gi].z, cur.w[0][gi].w};
                const uint32_t wh[4] = {cur.w[1][gi].x, cur.w[1][gi].y, cur.w[1][gi].z, cur.w[1][gi].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t A[4] = {wg[j] & 0x0F0F0F0Fu, wh[j] & 0x0F0F0F0Fu, (wg[j] >> 4) & 0x0F0F0F0Fu,
                                           (wh[j] >> 4) & 0x0F0F0F0Fu};
                    mma_u8s8(d, A, bb[2 * j], bb[2 * j + 1]);
                }
                const float2 gxs = xg[g];
                const float z0 = __uint_as_float(cur.z[0][gi] | 0x4B000000u) - 8388608.0f;
                const float z1 = __uint_as_float(cur.z[1][gi] | 0x4B000000u) - 8388608.0f;
                const float f0 = fmaf(-zmul * z0, gxs.x, fmaf(static_cast<float>(d[1]), w_odd, static_cast<float>(d[0]) * w_even));
                const float f1 = fmaf(-zmul * z1, gxs.x, fmaf(static_cast<float>(d[3]), w_odd, static_cast<float>(d[2]) * w_even));
                acc0 = fmaf(cur.s[0][gi] * gxs.y, f0, acc0);
                acc1 = fmaf(cur.s[1][gi] * gxs.y, f1, acc1);
            }
        }
        if (n_ord != u_ord || !more) {
            // unit complete: combine the quad's digit shares, store the partial sums
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if (c == 0) {
                float* dst = part + ((cur_tile - tile0) * geo.parts + cur_part) * kTile;
                dst[gq] = acc0;
                dst[gq + 8] = acc1;
            }
            acc0 = acc1 = 0.0f;
            if (n_ord >= my_units) break;
        }
        u_ord = n_ord;
        it_idx = n_idx;
        it_end = n_end;
        cur_tile = n_tile;
        cur_part = n_part;
        cur = nxt;
    }
    __syncthreads();
    // fixed-order reduction over the K parts, then the epilogue
    if constexpr (EPI == kW4Swiglu) {
        // gate/up are packed per kW4TileRows rows: half gate rows, then the matching up rows
        constexpr int half = kW4TileRows / 2;
        for (int o = threadIdx.x; o < nt * kTile / 2; o += kThreads) {
            const int gr = kW4TileRows * (o / half) + o % half, ur = gr + half;
            const float* pg = part + (gr / kTile) * geo.parts * kTile + gr % kTile;
            const float* pu = part + (ur / kTile) * geo.parts * kTile + ur % kTile;
            float g = 0.0f, u = 0.0f;
            for (int p = 0; p < geo.parts; ++p) {
                g += pg[p * kTile];
                u += pu[p * kTile];
            }
            const float silu = g * 1.0f / (1.0f + expf(-g));  // swiglu_kernel.cu:11-12
            a.y[tile0 * (kTile / 2) + o] = silu * u;
        }
    } else {
        for (int i = threadIdx.x; i < nt * kTile; i += kThreads) {
            const int tl = i >> 4, r = i & 15;
            float v = 0.0f;
            for (int p = 0; p < geo.parts; ++p) v += part[(tl * geo.parts + p) * kTile + r];
            const int row = (tile0 + tl) * kTile + r;
            if constexpr (EPI == kW4Residual) v = a.residual[row] + v;
            a.y[row] = v;
        }
    }
}

int gcd(int x, int y) {
    while (y) {
        const int t = x % y;
        x = y;
        y = t;
    }
    return x;
}

template <int GPI, int EPI>
cudaError_t launch(const W4Args& a, int num_sms, cudaStream_t stream, bool pdl) {
    Geometry geo{};
    geo.groups = a.K / 128;
    geo.items = geo.groups / GPI;
    geo.tiles = a.N / kTile;
    geo.nt = (geo.tiles + num_sms - 1) / num_sms;
    int parts = kMaxParts / gcd(geo.nt, kMaxParts);
    while (parts > 1 && parts > geo.items) parts >>= 1;
    geo.parts = parts;
    const int grid = (geo.tiles + geo.nt - 1) / geo.nt;
    const size_t smem = static_cast<size_t>(geo.groups) * (512 + 8) +
                        static_cast<size_t>(geo.nt) * geo.parts * kTile * sizeof(float);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    auto kern = w4_mma_kernel<GPI, EPI>;
    if (smem > 46 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a, geo);
}

}  // namespace

bool w4_mma_supported(const W4Args& a) {
    return a.N >= kTile && a.N % kTile == 0 && a.K % 128 == 0 && a.K >= 128 && a.K <= 53248;
}

cudaError_t w4_mma_launch(const W4Args& a, int epi, int num_sms, cudaStream_t stream, bool pdl) {
    const bool two = (a.K % 256) == 0;
    switch (epi) {
    case kW4Residual:
        return two ? launch<2, kW4Residual>(a, num_sms, stream, pdl) : launch<1, kW4Residual>(a, num_sms, stream, pdl);
    case kW4Swiglu:
        return two ? launch<2, kW4Swiglu>(a, num_sms, stream, pdl) : launch<1, kW4Swiglu>(a, num_sms, stream, pdl);
    default:
        return two ? launch<2, kW4Store>(a, num_sms, stream, pdl) : launch<1, kW4Store>(a, num_sms, stream, pdl);
    }
}

}  // namespace fb
