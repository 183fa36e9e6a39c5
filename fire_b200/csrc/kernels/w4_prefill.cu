// INT4 group-128 Linear for many rows (prefill) on the tcgen05 tensor cores.
//
//   Y[M, N] = X[M, K] . W[N, K]^T with w = s * (q - z) formed in FP32 (tools/quant.py
//   dequantize_int4_groupwise order) and rounded once to FP16, and each row of X scaled by a
//   power of two 2^sh (sh chosen so the row's largest |x| lands in [2^14, 2^15)) and rounded
//   once to FP16; FP32 accumulation in tensor memory, then y = acc * 2^-sh (exact). Both
//   operands carry 11 significant bits, so the product's error is two FP16 roundings
//   (~4e-4 relative RMS), one tensor-core instruction per 16 K.
//
//   * CTA tile 128 (M) x 128 (N), K in stages of 64 (one 128-byte swizzle row), a 6-stage
//     shared-memory ring with full/empty mbarriers per stage; CTAs that share a W tile are
//     adjacent in launch order (blockIdx.x walks M), so W is read from HBM once;
//   * one thread streams the X tile (and, in the two-pass form, the W tile) with TMA
//     (128-byte swizzle, each CTA loading its own tiles);
//   * W, in the default two-pass form, is first dequantised into FP16 [N, K] scratch in HBM
//     by an elementwise kernel and streamed by TMA; in the one-pass form
//     (FIRE_B200_PREFILL_FUSED=1) eight more warps dequantise it into each stage straight
//     from the INT4 .fire rows or layer-stack items (no FP16 copy of W in HBM). Both give
//     the same bits. At M = 512 the two-pass form is faster: the one-pass form redoes the
//     dequantisation for every 128-row M tile and its dequantising warps, not the tensor
//     cores, set the pace;
//   * one thread issues tcgen05.mma.cta_group::1.kind::f16 (M128 N128 K16, four per stage)
//     from shared-memory descriptors into a 128-column FP32 TMEM accumulator and frees each
//     stage with tcgen05.commit;
//   * four warps read their 32 TMEM lanes with tcgen05.ld, scale and store FP32 rows.
// Weights whose dequantised magnitude can leave the FP16 range (|s| * max(z, 15 - z) > 65504)
// are refused: the kernel records error 4. Every wait is bounded (0.2 s of GPU time): on
// timeout the kernel records an error, stops issuing, still commits and drains what it issued
// and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "w4_prefill.h"

namespace fb {
namespace {

constexpr int kStages = 6;
constexpr int kTileA = kPrefillBM * kPrefillBK * 2;  // 16 KB of FP16 X
constexpr int kTileB = kPrefillBN * kPrefillBK * 2;  // 16 KB of FP16 W
constexpr int kStageBytes = kTileA + kTileB;
constexpr int kTmemCols = kPrefillBN;  // FP32 accumulator columns
constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* alignment */ + 256 /* barriers */;
constexpr float kF16Max = 65504.0f;

// instruction descriptor, kind::f16: D F32 (bits 4-5 = 1), A F16 (7-9 = 0), B F16 (10-12 = 0),
// both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t kIdesc =
    (1u << 4) | (static_cast<uint32_t>(kPrefillBN >> 3) << 17) | (static_cast<uint32_t>(kPrefillBM >> 4) << 24);

// where the stage's W tile comes from
constexpr int kSrcTma = 0;    // FP16 [N, K] in HBM, by TMA (two-pass form)
constexpr int kSrcRows = 1;   // .fire INT4 rows + scales + zero points, dequantised in the CTA
constexpr int kSrcItems = 2;  // layer-stack items, dequantised in the CTA
constexpr int kDequantWarps = 8;
constexpr int kPrefetch = 3;  // stages of nibbles in flight per dequantising thread
template <int kSrc>
constexpr int threads_for() { return kSrc == kSrcTma ? 128 : 128 + 32 * kDequantWarps; }

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned c) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(c) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(su32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}
// bounded wait that lets the thread be suspended (up to 20 us per try) until the phase
// completes: for waiters off the critical path, so they leave issue slots to the others
__device__ bool mbar_wait_idle(uint64_t* b, unsigned parity) {
    const unsigned long long t0 = gtime();
    for (;;) {
        unsigned ok;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
            : "=r"(ok)
            : "r"(su32(b)), "r"(parity), "r"(20000u)
            : "memory");
        if (ok) return true;
        if (gtime() - t0 > kWaitNs) return false;
    }
}
// bounded wait; false after kWaitNs
__device__ bool mbar_wait(uint64_t* b, unsigned parity) {
    const unsigned long long t0 = gtime();
    for (int i = 0;; ++i) {
        if (mbar_try(b, parity)) return true;
        if ((i & 63) == 63 && gtime() - t0 > kWaitNs) return false;
    }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            su32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
}
// shared-memory matrix descriptor, K-major, 128-byte swizzle: start >> 4 (bits 0-13),
// leading byte offset 16 B (unused for swizzled K-major), stride byte offset 1024 B (8 rows
// of 128 B) at bits 32-45, descriptor version 1 (bits 46-47), layout SWIZZLE_128B = 2 (bits 61-63)
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}


// weights of this group fit FP16 after dequantisation (|q - z| <= max(z, 15 - z))
__device__ __forceinline__ bool f16_safe(float sc, float zp) { return fabsf(sc) * fmaxf(zp, 15.0f - zp) <= kF16Max; }

// eight weights of one 32-bit word (even k in the low nibble) -> one 16-byte FP16 chunk.
// A byte permute puts each nibble q into the mantissa of 2^23, giving the float 2^23 + q
// (no integer-to-float conversion), so q - z is one exact packed add of -(2^23 + z); then
// s * (q - z) is one packed FP32 multiply (the same single rounding as s * (float(q) - z))
// and the pair is rounded once to FP16.
__device__ __forceinline__ uint4 dequant8_f16(uint32_t v, float sc, float zp) {
    const uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
    const float nz = -(8388608.0f + zp);  // exact: zp is an integer below 256
    const float2 off = make_float2(nz, nz), s2 = make_float2(sc, sc);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t sel = 0x7440u | static_cast<uint32_t>(j);  // bytes {x.b[j], 0, 0, 0x4B}
        const float2 q = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, sel)),
                                     __uint_as_float(__byte_perm(hi, 0x4B000000u, sel)));
        const float2 w = __fmul2_rn(__fadd2_rn(q, off), s2);
        const __half2 h = __floats2half2_rn(w.x, w.y);  // .x = lower k
        o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// INT4 source of the dequantising warps: half h (16 bytes, 32 weights) of row n's 64 K of
// stage kt, with its group's scale and zero point
template <int kSrc>
struct W4Src {
    const uint8_t* q;  // .fire qweight [N, K/2] or layer-stack items (16 rows x 256 K per 2208 bytes)
    const float* s;    // .fire scales [N, K/128]
    const uint8_t* z;  // .fire zero points [N, K/128]
    int K;
    __device__ __forceinline__ void load(int n, int kt, int h, uint4& w, float& sc, float& zp) const {
        if (kSrc == kSrcItems) {
            const int t = n >> 4, r = n & 15, it = kt >> 2, gi = (kt >> 1) & 1, half = kt & 1;
            const uint8_t* item = q + (static_cast<size_t>(t) * (K / 256) + it) * 2208;
            w = __ldg(reinterpret_cast<const uint4*>(item) + (((r >> 3) * 2 + gi) * 32 + 4 * (r & 7) + 2 * half + h));
            sc = __ldg(reinterpret_cast<const float*>(item + 2048) + r * 2 + gi);
            zp = static_cast<float>(__ldg(item + 2176 + r * 2 + gi));
        } else {
            w = __ldg(reinterpret_cast<const uint4*>(q + static_cast<size_t>(n) * (K / 2) + kt * 32) + h);
            const size_t g = static_cast<size_t>(n) * (K / 128) + (kt >> 1);
            sc = __ldg(s + g);
            zp = static_cast<float>(__ldg(z + g));
        }
    }
};

// One 128 x 128 output tile. Warp 0 lane 0: TMA producer; warp 1 lane 0: MMA issuer; warps
// 0-3: epilogue (warp w owns TMEM lanes, i.e. rows, 32w..32w+31); warps 4.. (dequantising
// forms): W rows n0 + (d & 127), half d >> 7 of each stage's 64 K, stored in the 128-byte
// swizzle layout TMA would have produced (16-byte chunk c of row r at chunk c ^ (r & 7)),
// published with a proxy fence (the MMA reads shared memory through the async proxy) and
// one arrival per warp on the stage's full barrier.
template <int kSrc>
__global__ void __launch_bounds__(threads_for<kSrc>(), 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const W4Src<kSrc> src, const float* __restrict__ rscale, float* y, int M, int N, int K, int* err) {
    constexpr bool kTmaB = kSrc == kSrcTma;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* failed = reinterpret_cast<int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kPrefillBM, n0 = blockIdx.y * kPrefillBN;
    const int KT = K / kPrefillBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], kTmaB ? 1 : 1 + kDequantWarps);  // producer (with its bytes) [+ dequant warps]
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
        if (kTmaB) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
    }
    if (warp == 1) {  // the whole warp allocates the accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (!kTmaB && warp >= 4) {
        const int d = threadIdx.x - 128, r = d & 127, h = d >> 7, n = n0 + r;
        uint4 w[kPrefetch];
        float sc[kPrefetch], zp[kPrefetch];
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i)
            if (i < KT) src.load(n, i, h, w[i], sc[i], zp[i]);
        uint8_t* const brow0 = smem + kTileA + r * 128;
        bool range_ok = true;
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % kStages;
            const uint4 cw = w[0];
            const float csc = sc[0], czp = zp[0];
#pragma unroll
            for (int i = 0; i + 1 < kPrefetch; ++i) {  // shift the prefetch window (register moves)
                w[i] = w[i + 1];
                sc[i] = sc[i + 1];
                zp[i] = zp[i + 1];
            }
            if (kt + kPrefetch < KT)
                src.load(n, kt + kPrefetch, h, w[kPrefetch - 1], sc[kPrefetch - 1], zp[kPrefetch - 1]);
            range_ok = range_ok && f16_safe(csc, czp);
            bool ok = true;
            if (kt >= kStages) ok = mbar_wait(&empty[s], static_cast<unsigned>((kt / kStages - 1) & 1));
            const bool all_ok = __all_sync(0xffffffffu, ok);
            if (!all_ok && lane == 0) {
                atomicExch(err, 3);
                *reinterpret_cast<volatile int*>(failed) = 1;
            }
            if (!all_ok || *reinterpret_cast<volatile int*>(failed)) break;
            uint8_t* brow = brow0 + s * kStageBytes;
            const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)  // k = 8c .. 8c+7 of the half are bytes 4c .. 4c+3
                *reinterpret_cast<uint4*>(brow + (((4 * h + c) ^ (r & 7)) << 4)) = dequant8_f16(wd[c], csc, czp);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&full[s])) : "memory");
        }
        if (!range_ok) atomicExch(err, 4);
    } else if (warp == 0 && lane == 0) {
        // producer: the X tile (and W tile) of K slice kt
        int issued = 0;
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % kStages;
            if (kt >= kStages && !mbar_wait(&empty[s], static_cast<unsigned>((kt / kStages - 1) & 1))) {
                atomicExch(err, 1);
                *reinterpret_cast<volatile int*>(failed) = 1;
                break;
            }
            if (*reinterpret_cast<volatile int*>(failed)) break;
            uint8_t* a = smem + s * kStageBytes;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&full[s])),
                         "r"(kTmaB ? kStageBytes : kTileA)
                         : "memory");
            tma_load_2d(a, &tma_a, kt * kPrefillBK, m0, &full[s]);
            if (kTmaB) tma_load_2d(a + kTileA, &tma_b, kt * kPrefillBK, n0, &full[s]);
            issued = kt + 1;
        }
        // drain: every issued copy lands before the CTA may exit (bounded; in the
        // dequantising forms a phase may also wait for arrivals a failure skipped)
        for (int kt = issued > kStages ? issued - kStages : 0; kt < issued; ++kt)
            mbar_wait(&full[kt % kStages], static_cast<unsigned>((kt / kStages) & 1));
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % kStages;
            if (!mbar_wait(&full[s], static_cast<unsigned>((kt / kStages) & 1))) {
                atomicExch(err, 2);
                *reinterpret_cast<volatile int*>(failed) = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a = su32(smem + s * kStageBytes), b = a + kTileA;
#pragma unroll
            for (int k = 0; k < kPrefillBK / 16; ++k)  // K16 per instruction: +32 bytes along the swizzled row
                umma_f16(tmem, desc_sw128(a + 32 * k), desc_sw128(b + 32 * k), (kt | k) != 0);
            umma_commit(&empty[s]);
        }
        umma_commit(done);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
    if (warp < 4) {
        const bool ok = mbar_wait_idle(done, 0) && *reinterpret_cast<volatile int*>(failed) == 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__all_sync(0xffffffffu, ok)) {
            const int row = m0 + warp * 32 + lane;
            const float rs = row < M ? __ldg(rscale + row) : 0.0f;
            float* dst = y + static_cast<size_t>(row) * N + n0;
#pragma unroll 1
            for (int c = 0; c < kPrefillBN / 32; ++c) {
                uint32_t r[32];
                const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(c * 32);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                      "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                      "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < M) {
                    float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        d4[j] = make_float4(__uint_as_float(r[4 * j]) * rs, __uint_as_float(r[4 * j + 1]) * rs,
                                            __uint_as_float(r[4 * j + 2]) * rs, __uint_as_float(r[4 * j + 3]) * rs);
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// W (INT4 group 128, .fire rows) -> FP16 [N, K]: one thread per 8 weights (one 32-bit word)
__global__ void dequant_rows_f16_kernel(const uint8_t* __restrict__ qw, const float* __restrict__ scales,
                                        const uint8_t* __restrict__ zeros, __half* __restrict__ out, int N, int K,
                                        int* err) {
    const long long total = static_cast<long long>(N) * (K / 8);
    const int groups = K / 128;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int n = static_cast<int>(i / (K / 8));
        const int k = static_cast<int>(i % (K / 8)) * 8;
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(qw + static_cast<size_t>(n) * (K / 2) + k / 2));
        const float s = __ldg(scales + static_cast<size_t>(n) * groups + k / 128);
        const float z = static_cast<float>(__ldg(zeros + static_cast<size_t>(n) * groups + k / 128));
        if (!f16_safe(s, z)) atomicExch(err, 4);
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(n) * K + k) = dequant8_f16(w, s, z);
    }
}

// W in the layer-stack item layout (16 rows x 256 K per 2208-byte item, see layer_stack.h)
// -> FP16 [N, K] in the items' row order; one thread per 8 weights
__global__ void dequant_items_f16_kernel(const uint8_t* __restrict__ items, __half* __restrict__ out, int N, int K,
                                         int* err) {
    const long long total = static_cast<long long>(N) * (K / 8);
    const int ipr = K / 256;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int n = static_cast<int>(i / (K / 8));
        const int k = static_cast<int>(i % (K / 8)) * 8;
        const int tile = n >> 4, r = n & 15, it = k >> 8, kl = k & 255;
        const int gi = kl >> 7, b = (kl & 127) >> 1;  // group in the item, byte in the row's 64-byte group
        const uint8_t* item = items + (static_cast<size_t>(tile) * ipr + it) * 2208;
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(
            item + (((r >> 3) * 2 + gi) * 32 + (r & 7) * 4 + (b >> 4)) * 16 + (b & 15)));
        const float s = __ldg(reinterpret_cast<const float*>(item + 2048) + r * 2 + gi);
        const float z = static_cast<float>(__ldg(item + 2176 + r * 2 + gi));
        if (!f16_safe(s, z)) atomicExch(err, 4);
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(n) * K + k) = dequant8_f16(w, s, z);
    }
}

// X FP32 [M, K] -> FP16 scaled per row by 2^sh, sh = 15 - e for the row's largest |x| =
// m * 2^e (m in [0.5, 1)), so that value lands in [2^14, 2^15): no overflow, and values down
// to 2^-29 of the row's largest stay normal. rscale[row] = 2^-sh (exact powers of two, made
// from the exponent bits). One CTA per row.
__global__ void x_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ x16, float* __restrict__ rscale,
                                int K) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * K);
    float mx = 0.0f;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = __ldg(xr + i);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
    // frexp exponent of a normal float: biased exponent - 126 (0 for a zero row)
    const int e = mx > 0.0f ? static_cast<int>((__float_as_uint(mx) >> 23) & 0xFF) - 126 : 0;
    const int sh = max(-126, min(126, 15 - e));
    const float up = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
    uint2* dst = reinterpret_cast<uint2*>(x16 + static_cast<size_t>(row) * K);
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = __ldg(xr + i);
        const __half2 a = __floats2half2_rn(v.x * up, v.y * up), b = __floats2half2_rn(v.z * up, v.w * up);
        dst[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
    }
    if (threadIdx.x == 0) rscale[row] = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D FP16 row-major [rows, K] map with a 64 x 128 box and 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, int rows, int K, int box_rows) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kPrefillBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// X in FP16 at the start of the workspace, the row scales after it
cudaError_t prepare_x(const float* x, int M, int K, void* workspace, __half** x16, float** rscale, cudaStream_t s) {
    *x16 = static_cast<__half*>(workspace);
    *rscale = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(static_cast<size_t>(M) * K * 2));
    x_to_f16_kernel<<<M, 256, 0, s>>>(x, *x16, *rscale, K);
    return cudaGetLastError();
}

template <int kSrc>
cudaError_t launch_tiles(const CUtensorMap& ma, const CUtensorMap& mb, const W4Src<kSrc>& src, const float* rscale,
                         float* y, int M, int N, int K, int* err, cudaStream_t s) {
    auto kern = prefill_kernel<kSrc>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    const dim3 grid(static_cast<unsigned>(M / kPrefillBM), static_cast<unsigned>(N / kPrefillBN));
    kern<<<grid, threads_for<kSrc>(), kSmemBytes, s>>>(ma, mb, src, rscale, y, M, N, K, err);
    return cudaGetLastError();
}

}  // namespace

bool prefill_supported(int M, int N, int K, int group) {
    return group == 128 && M >= kPrefillBM && N >= kPrefillBN && M % kPrefillBM == 0 && N % kPrefillBN == 0 &&
           K % 128 == 0 && K > 0;
}

size_t prefill_gemm_workspace_bytes(int M, int K) {
    return align256(static_cast<size_t>(M) * K * 2) + align256(static_cast<size_t>(M) * 4);
}

size_t prefill_workspace_bytes(int M, int N, int K) {
    return prefill_gemm_workspace_bytes(M, K) + align256(static_cast<size_t>(N) * K * 2);
}

cudaError_t prefill_dequant_rows_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K,
                                        void* w_f16, int* err, cudaStream_t s) {
    if (N <= 0 || K % 128 || err == nullptr || reinterpret_cast<uintptr_t>(w_f16) % 16 ||
        reinterpret_cast<uintptr_t>(qw) % 4)
        return cudaErrorInvalidValue;
    const long long w8 = static_cast<long long>(N) * K / 8;
    dequant_rows_f16_kernel<<<static_cast<int>(std::min<long long>((w8 + 255) / 256, 8192)), 256, 0, s>>>(
        qw, scales, zeros, static_cast<__half*>(w_f16), N, K, err);
    return cudaGetLastError();
}

cudaError_t prefill_dequant_items_launch(const uint8_t* items, int N, int K, void* w_f16, int* err, cudaStream_t s) {
    if (N % 16 || K % 256 || err == nullptr || reinterpret_cast<uintptr_t>(w_f16) % 16 ||
        reinterpret_cast<uintptr_t>(items) % 16)
        return cudaErrorInvalidValue;
    const long long w8 = static_cast<long long>(N) * K / 8;
    dequant_items_f16_kernel<<<static_cast<int>(std::min<long long>((w8 + 255) / 256, 8192)), 256, 0, s>>>(
        items, static_cast<__half*>(w_f16), N, K, err);
    return cudaGetLastError();
}

cudaError_t prefill_gemm_launch(const float* x, const void* w_f16, float* y, int M, int N, int K, void* workspace,
                                size_t workspace_bytes, int* err, cudaStream_t s) {
    if (!prefill_supported(M, N, K, 128) || workspace == nullptr || err == nullptr) return cudaErrorInvalidValue;
    if (workspace_bytes < prefill_gemm_workspace_bytes(M, K)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(workspace) |
         reinterpret_cast<uintptr_t>(w_f16)) % 16)
        return cudaErrorInvalidValue;
    __half* x16;
    float* rscale;
    cudaError_t e = prepare_x(x, M, K, workspace, &x16, &rscale, s);
    if (e != cudaSuccess) return e;
    CUtensorMap ma, mb;
    if (!make_map(&ma, x16, M, K, kPrefillBM) || !make_map(&mb, w_f16, N, K, kPrefillBN)) return cudaErrorNotSupported;
    return launch_tiles<kSrcTma>(ma, mb, W4Src<kSrcTma>{nullptr, nullptr, nullptr, K}, rscale, y, M, N, K, err, s);
}

bool prefill_one_pass() {
    static const bool one = [] {
        const char* v = std::getenv("FIRE_B200_PREFILL_FUSED");
        return v != nullptr && std::strcmp(v, "1") == 0;
    }();
    return one;
}

cudaError_t prefill_w4_fused_launch(const float* x, const uint8_t* w, const float* scales, const uint8_t* zeros,
                                    bool items, float* y, int M, int N, int K, void* workspace,
                                    size_t workspace_bytes, int* err, cudaStream_t s) {
    if (!prefill_supported(M, N, K, 128) || workspace == nullptr || err == nullptr || w == nullptr)
        return cudaErrorInvalidValue;
    if (items ? K % 256 != 0 : (scales == nullptr || zeros == nullptr)) return cudaErrorInvalidValue;
    if (workspace_bytes < prefill_gemm_workspace_bytes(M, K)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(workspace) |
         reinterpret_cast<uintptr_t>(w)) % 16)
        return cudaErrorInvalidValue;
    __half* x16;
    float* rscale;
    cudaError_t e = prepare_x(x, M, K, workspace, &x16, &rscale, s);
    if (e != cudaSuccess) return e;
    CUtensorMap ma;
    if (!make_map(&ma, x16, M, K, kPrefillBM)) return cudaErrorNotSupported;
    if (items)
        return launch_tiles<kSrcItems>(ma, ma, W4Src<kSrcItems>{w, nullptr, nullptr, K}, rscale, y, M, N, K, err, s);
    return launch_tiles<kSrcRows>(ma, ma, W4Src<kSrcRows>{w, scales, zeros, K}, rscale, y, M, N, K, err, s);
}

cudaError_t prefill_w4_launch(const float* x, const uint8_t* qw, const float* scales, const uint8_t* zeros, float* y,
                              int M, int N, int K, void* workspace, size_t workspace_bytes, int* err,
                              cudaStream_t s) {
    if (!prefill_supported(M, N, K, 128) || workspace == nullptr || err == nullptr) return cudaErrorInvalidValue;
    if (workspace_bytes < prefill_workspace_bytes(M, N, K)) return cudaErrorInvalidValue;
    const size_t gws = prefill_gemm_workspace_bytes(M, K);
    // the one-pass form reads 16-byte chunks of the rows; the two-pass form needs 4-byte alignment
    if (prefill_one_pass() && reinterpret_cast<uintptr_t>(qw) % 16 == 0)
        return prefill_w4_fused_launch(x, qw, scales, zeros, false, y, M, N, K, workspace, gws, err, s);
    void* wb = static_cast<char*>(workspace) + gws;
    cudaError_t e = prefill_dequant_rows_launch(qw, scales, zeros, N, K, wb, err, s);
    if (e != cudaSuccess) return e;
    return prefill_gemm_launch(x, wb, y, M, N, K, workspace, gws, err, s);
}

}  // namespace fb
