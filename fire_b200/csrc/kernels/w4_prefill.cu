// INT4 group-128 Linear for many rows (prefill) on the tcgen05 tensor cores.
//
//   1. dequantise W once into BF16 scratch: w = s * (q - z) in FP32 (tools/quant.py
//      dequantize_int4_groupwise order), one rounding to BF16; split X (FP32) into
//      x_hi = bf16(x) and x_lo = bf16(x - x_hi), so X enters with ~16 mantissa bits and
//      the product's error is W's one BF16 rounding. HBM-bound passes over N*K/2 + N*K*2
//      and M*K*8 bytes.
//   2. a BF16 GEMM, Y = X . W^T, FP32 accumulation in tensor memory:
//      * CTA tile 128 (M) x 128 (N), K in stages of 64 (one 128-byte swizzle row);
//      * one thread streams the x_hi, x_lo and W tiles with TMA (128-byte swizzle, each
//        CTA loading its own tiles) into a 4-stage shared-memory ring, full/empty mbarriers;
//      * one thread issues tcgen05.mma.cta_group::1.kind::f16 (M128 N128 K16: x_hi.W and
//        x_lo.W per 16 K, eight per stage) from shared-memory descriptors into a
//        128-column FP32 TMEM accumulator and frees each stage with tcgen05.commit;
//      * the four warps read their 32 TMEM lanes with tcgen05.ld and store FP32 rows.
// Dequantising inside the GEMM would cost ~2 instructions per weight against M MACs per
// weight, i.e. several times the MMA time at M = 512, so the dequantised tile is made once.
// Every wait is bounded (0.2 s of GPU time): on timeout the kernel records an error, stops
// issuing, still commits and drains what it issued and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "w4_prefill.h"

namespace fb {
namespace {

constexpr int kStages = 4;
constexpr int kTileA = kPrefillBM * kPrefillBK * 2;  // 16 KB (x_hi, then x_lo)
constexpr int kTileB = kPrefillBN * kPrefillBK * 2;  // 16 KB
constexpr int kStageBytes = 2 * kTileA + kTileB;
constexpr int kThreads = 128;
constexpr int kTmemCols = kPrefillBN;  // FP32 accumulator columns
constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* alignment */ + 256 /* barriers */;

// instruction descriptor, kind::f16: D F32 (bits 4-5 = 1), A BF16 (7-9 = 1), B BF16 (10-12 = 1),
// both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kPrefillBN >> 3) << 17) |
                            (static_cast<uint32_t>(kPrefillBM >> 4) << 24);

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
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
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

__global__ void __launch_bounds__(kThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_alo,
                        const __grid_constant__ CUtensorMap tma_b, float* y, int M, int N, int K, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* failed = reinterpret_cast<int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * kPrefillBM, n0 = blockIdx.x * kPrefillBN;
    const int KT = K / kPrefillBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_alo)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
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

    if (warp == 0 && lane == 0) {
        // producer: A tile rows m0.., B tile rows n0.., K slice kt
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
                         "r"(kStageBytes)
                         : "memory");
            tma_load_2d(a, &tma_a, kt * kPrefillBK, m0, &full[s]);
            tma_load_2d(a + kTileA, &tma_alo, kt * kPrefillBK, m0, &full[s]);
            tma_load_2d(a + 2 * kTileA, &tma_b, kt * kPrefillBK, n0, &full[s]);
            issued = kt + 1;
        }
        // drain: every issued stage lands before the CTA may exit
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
            const uint32_t a = su32(smem + s * kStageBytes), alo = a + kTileA, b = a + 2 * kTileA;
#pragma unroll
            for (int k = 0; k < kPrefillBK / 16; ++k) {  // K16 per instruction: +32 bytes along the swizzled row
                umma_bf16(tmem, desc_sw128(a + 32 * k), desc_sw128(b + 32 * k), (kt | k) != 0);
                umma_bf16(tmem, desc_sw128(alo + 32 * k), desc_sw128(b + 32 * k), 1);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(done);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
    // epilogue: warp w owns TMEM lanes (rows) 32w..32w+31
    const bool ok = mbar_wait(done, 0) && *reinterpret_cast<volatile int*>(failed) == 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (__all_sync(0xffffffffu, ok)) {
        const int row = m0 + warp * 32 + lane;
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
                    d4[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                        __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
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

// ---------------------------------------------------------------------------------
// Fused form: W is dequantised into shared memory inside the pipeline instead of through
// BF16 scratch in HBM. Eight more warps (the "dequant warps"; thread d <-> row n0 + (d & 127)
// of the W tile, half d >> 7 of its 64 K of the stage) read 16 bytes of nibbles per stage
// from the .fire rows or the layer-stack items, kPrefetch stages ahead in registers so the
// loads' latency hides behind the MMAs, form w = s * (q - z) in FP32 and round it once to
// BF16 exactly as dequant_w4_bf16_kernel does, and store four 16-byte chunks into the
// stage's B tile in the 128-byte-swizzle layout TMA would have produced (16-byte chunk c of
// row r at chunk c ^ (r & 7)). They publish the tile with a proxy fence (the MMA reads
// shared memory through the async proxy) and one arrival per warp on the stage's full
// barrier, next to the producer's transaction count for the two X tiles. Same products and
// accumulation order as the two-pass form, so the results are bit-identical; per stage the
// TMA moves 32 KB instead of 48 KB, and the separate dequantisation pass is gone.
constexpr int kDequantWarps = 8;
constexpr int kFusedThreads = 128 + 32 * kDequantWarps;  // warps 0-3 as above, then the dequant warps
constexpr int kPrefetch = 3;                              // stages of nibbles in flight per thread

template <bool kItems>
struct W4Src {
    const uint8_t* q;      // .fire qweight [N, K/2] or layer-stack items
    const float* s;        // .fire scales [N, K/128] (rows form)
    const uint8_t* z;      // .fire zero points [N, K/128] (rows form)
    int K;
    // half h (16 bytes, 32 weights) of this row's 64 K of stage kt, its scale and zero point
    __device__ __forceinline__ void load(int n, int kt, int h, uint4& w, float& sc, float& zp) const {
        if (kItems) {
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

template <bool kItems>
__global__ void __launch_bounds__(kFusedThreads, 1)
    prefill_w4_fused_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_alo,
                            const W4Src<kItems> src, float* y, int M, int N, int K, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    int* failed = reinterpret_cast<int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kPrefillBM, n0 = blockIdx.y * kPrefillBN;  // M tiles of one N tile run together
    const int KT = K / kPrefillBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1 + kDequantWarps);  // producer (with the X bytes) + the dequant warps
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_alo)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp >= 4) {
        // dequant warps: row n0 + (d & 127), half d >> 7, every stage
        const int d = threadIdx.x - 128, r = d & 127, h = d >> 7, n = n0 + r;
        uint4 w[kPrefetch];
        float sc[kPrefetch], zp[kPrefetch];
#pragma unroll
        for (int i = 0; i < kPrefetch; ++i)
            if (i < KT) src.load(n, i, h, w[i], sc[i], zp[i]);
        uint8_t* const brow0 = smem + 2 * kTileA + r * 128;
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
            if (kt + kPrefetch < KT) src.load(n, kt + kPrefetch, h, w[kPrefetch - 1], sc[kPrefetch - 1], zp[kPrefetch - 1]);
            bool ok = true;
            if (kt >= kStages) ok = mbar_wait(&empty[s], static_cast<unsigned>((kt / kStages - 1) & 1));
            const bool all_ok = __all_sync(0xffffffffu, ok);
            if (!all_ok && lane == 0) {
                atomicExch(err, 3);
                *reinterpret_cast<volatile int*>(failed) = 1;
            }
            if (!all_ok || *reinterpret_cast<volatile int*>(failed)) break;
            // 32 weights = 4 chunks of 8 (k = 8c .. 8c+7 are bytes 4c .. 4c+3 of the half)
            uint8_t* brow = brow0 + s * kStageBytes;
            const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t v = wd[c];
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float lo = csc * (static_cast<float>((v >> (8 * j)) & 0xF) - czp);
                    const float hi = csc * (static_cast<float>((v >> (8 * j + 4)) & 0xF) - czp);
                    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);  // .x = lower k
                    o[j] = *reinterpret_cast<const uint32_t*>(&b);
                }
                *reinterpret_cast<uint4*>(brow + (((4 * h + c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
            // visible to the tensor core's (async proxy) reads, then one arrival per warp
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&full[s])) : "memory");
        }
    } else if (warp == 0 && lane == 0) {
        // producer: the x_hi and x_lo tiles of rows m0.., K slice kt
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
                         "r"(2 * kTileA)
                         : "memory");
            tma_load_2d(a, &tma_a, kt * kPrefillBK, m0, &full[s]);
            tma_load_2d(a + kTileA, &tma_alo, kt * kPrefillBK, m0, &full[s]);
            issued = kt + 1;
        }
        // drain: every issued X copy lands before the CTA may exit (bounded)
        for (int kt = issued > kStages ? issued - kStages : 0; kt < issued; ++kt) {
            const int s = kt % kStages;
            const unsigned long long t0 = gtime();
            for (int i = 0;; ++i) {
                // the X bytes of stage kt are in once the barrier's transaction count is met;
                // the phase itself may also wait for dequant arrivals that a failure skipped
                if (mbar_try(&full[s], static_cast<unsigned>((kt / kStages) & 1))) break;
                if ((i & 63) == 63 && gtime() - t0 > kWaitNs) break;
            }
        }
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
            const uint32_t a = su32(smem + s * kStageBytes), alo = a + kTileA, b = a + 2 * kTileA;
#pragma unroll
            for (int k = 0; k < kPrefillBK / 16; ++k) {
                umma_bf16(tmem, desc_sw128(a + 32 * k), desc_sw128(b + 32 * k), (kt | k) != 0);
                umma_bf16(tmem, desc_sw128(alo + 32 * k), desc_sw128(b + 32 * k), 1);
            }
            umma_commit(&empty[s]);
        }
        umma_commit(done);
    }
    __syncwarp();
    if (warp < 4) {
        const bool ok = mbar_wait(done, 0) && *reinterpret_cast<volatile int*>(failed) == 0;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (__all_sync(0xffffffffu, ok)) {
            const int row = m0 + warp * 32 + lane;
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
                        d4[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                            __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
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

// W (INT4 group 128) -> BF16 [N, K]: one thread per 8 weights (one 32-bit word of nibbles)
__global__ void dequant_w4_bf16_kernel(const uint8_t* __restrict__ qw, const float* __restrict__ scales,
                                       const uint8_t* __restrict__ zeros, __nv_bfloat16* __restrict__ out, int N,
                                       int K) {
    const long long total = static_cast<long long>(N) * (K / 8);
    const int groups = K / 128;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int n = static_cast<int>(i / (K / 8));
        const int k = static_cast<int>(i % (K / 8)) * 8;
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(qw + static_cast<size_t>(n) * (K / 2) + k / 2));
        const float s = __ldg(scales + static_cast<size_t>(n) * groups + k / 128);
        const float z = static_cast<float>(__ldg(zeros + static_cast<size_t>(n) * groups + k / 128));
        uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = s * (static_cast<float>((w >> (8 * j)) & 0xF) - z);
            const float hi = s * (static_cast<float>((w >> (8 * j + 4)) & 0xF) - z);
            const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);  // .x = lower k
            packed[j] = *reinterpret_cast<const uint32_t*>(&b);
        }
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(n) * K + k) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

// W in the layer-stack item layout (16 rows x 256 K per 2208-byte item, see layer_stack.h)
// -> BF16 [N, K] in the items' row order; one thread per 8 weights
__global__ void dequant_items_bf16_kernel(const uint8_t* __restrict__ items, __nv_bfloat16* __restrict__ out, int N,
                                          int K) {
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
        uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = s * (static_cast<float>((w >> (8 * j)) & 0xF) - z);
            const float hi = s * (static_cast<float>((w >> (8 * j + 4)) & 0xF) - z);
            const __nv_bfloat162 bb = __floats2bfloat162_rn(lo, hi);
            packed[j] = *reinterpret_cast<const uint32_t*>(&bb);
        }
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(n) * K + k) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
}

// X FP32 -> x_hi = bf16(x), x_lo = bf16(x - x_hi), 8 elements per thread
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&p);
}
__global__ void split_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo, long long n8) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
        const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = pack_bf16(v[2 * j], v[2 * j + 1]);
            const __nv_bfloat162 hb = *reinterpret_cast<const __nv_bfloat162*>(&h[j]);
            l[j] = pack_bf16(v[2 * j] - __low2float(hb), v[2 * j + 1] - __high2float(hb));
        }
        reinterpret_cast<uint4*>(hi)[i] = make_uint4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<uint4*>(lo)[i] = make_uint4(l[0], l[1], l[2], l[3]);
    }
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

// 2-D BF16 row-major [rows, K] map with a 64 x 128 box and 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, int rows, int K, int box_rows) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kPrefillBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

bool prefill_supported(int M, int N, int K, int group) {
    return group == 128 && M >= kPrefillBM && N >= kPrefillBN && M % kPrefillBM == 0 && N % kPrefillBN == 0 &&
           K % 128 == 0 && K > 0;
}

size_t prefill_workspace_bytes(int M, int N, int K) {
    return 2 * align256(static_cast<size_t>(M) * K * 2) + align256(static_cast<size_t>(N) * K * 2);
}

size_t prefill_gemm_workspace_bytes(int M, int K) { return 2 * align256(static_cast<size_t>(M) * K * 2); }

cudaError_t prefill_dequant_rows_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K,
                                        void* w_bf16, cudaStream_t s) {
    if (N <= 0 || K % 128 || reinterpret_cast<uintptr_t>(w_bf16) % 16 || reinterpret_cast<uintptr_t>(qw) % 4)
        return cudaErrorInvalidValue;
    const long long w8 = static_cast<long long>(N) * K / 8;
    dequant_w4_bf16_kernel<<<static_cast<int>(std::min<long long>((w8 + 255) / 256, 8192)), 256, 0, s>>>(
        qw, scales, zeros, static_cast<__nv_bfloat16*>(w_bf16), N, K);
    return cudaGetLastError();
}

cudaError_t prefill_dequant_items_launch(const uint8_t* items, int N, int K, void* w_bf16, cudaStream_t s) {
    if (N % 16 || K % 256 || reinterpret_cast<uintptr_t>(w_bf16) % 16 || reinterpret_cast<uintptr_t>(items) % 16)
        return cudaErrorInvalidValue;
    const long long w8 = static_cast<long long>(N) * K / 8;
    dequant_items_bf16_kernel<<<static_cast<int>(std::min<long long>((w8 + 255) / 256, 8192)), 256, 0, s>>>(
        items, static_cast<__nv_bfloat16*>(w_bf16), N, K);
    return cudaGetLastError();
}

cudaError_t prefill_gemm_launch(const float* x, const void* w_bf16, float* y, int M, int N, int K, void* workspace,
                                size_t workspace_bytes, int* err, cudaStream_t s) {
    if (!prefill_supported(M, N, K, 128) || workspace == nullptr || err == nullptr) return cudaErrorInvalidValue;
    if (workspace_bytes < prefill_gemm_workspace_bytes(M, K)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(workspace) |
         reinterpret_cast<uintptr_t>(w_bf16)) % 16)
        return cudaErrorInvalidValue;
    const size_t xbytes = align256(static_cast<size_t>(M) * K * 2);
    __nv_bfloat16* xb = static_cast<__nv_bfloat16*>(workspace);
    __nv_bfloat16* xl = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(workspace) + xbytes);
    const long long n8 = static_cast<long long>(M) * K / 8;
    split_bf16_kernel<<<static_cast<int>(std::min<long long>((n8 + 255) / 256, 4096)), 256, 0, s>>>(x, xb, xl, n8);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap ma, malo, mb;
    if (!make_map(&ma, xb, M, K, kPrefillBM) || !make_map(&malo, xl, M, K, kPrefillBM) ||
        !make_map(&mb, w_bf16, N, K, kPrefillBN))
        return cudaErrorNotSupported;
    e = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    dim3 grid(static_cast<unsigned>(N / kPrefillBN), static_cast<unsigned>(M / kPrefillBM));
    prefill_gemm_kernel<<<grid, kThreads, kSmemBytes, s>>>(ma, malo, mb, y, M, N, K, err);
    return cudaGetLastError();
}

bool prefill_two_pass() {
    static const bool two = [] {
        const char* v = std::getenv("FIRE_B200_PREFILL_TWO_PASS");
        return v != nullptr && std::strcmp(v, "1") == 0;
    }();
    return two;
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
    const size_t xbytes = align256(static_cast<size_t>(M) * K * 2);
    __nv_bfloat16* xb = static_cast<__nv_bfloat16*>(workspace);
    __nv_bfloat16* xl = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(workspace) + xbytes);
    const long long n8 = static_cast<long long>(M) * K / 8;
    split_bf16_kernel<<<static_cast<int>(std::min<long long>((n8 + 255) / 256, 4096)), 256, 0, s>>>(x, xb, xl, n8);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap ma, malo;
    if (!make_map(&ma, xb, M, K, kPrefillBM) || !make_map(&malo, xl, M, K, kPrefillBM)) return cudaErrorNotSupported;
    const dim3 grid(static_cast<unsigned>(M / kPrefillBM), static_cast<unsigned>(N / kPrefillBN));
    if (items) {
        auto kern = prefill_w4_fused_kernel<true>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        kern<<<grid, kFusedThreads, kSmemBytes, s>>>(ma, malo, W4Src<true>{w, nullptr, nullptr, K}, y, M, N, K, err);
    } else {
        auto kern = prefill_w4_fused_kernel<false>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        kern<<<grid, kFusedThreads, kSmemBytes, s>>>(ma, malo, W4Src<false>{w, scales, zeros, K}, y, M, N, K, err);
    }
    return cudaGetLastError();
}

cudaError_t prefill_w4_launch(const float* x, const uint8_t* qw, const float* scales, const uint8_t* zeros, float* y,
                              int M, int N, int K, void* workspace, size_t workspace_bytes, int* err,
                              cudaStream_t s) {
    if (!prefill_supported(M, N, K, 128) || workspace == nullptr || err == nullptr) return cudaErrorInvalidValue;
    if (workspace_bytes < prefill_workspace_bytes(M, N, K)) return cudaErrorInvalidValue;
    const size_t gws = prefill_gemm_workspace_bytes(M, K);
    if (!prefill_two_pass())
        return prefill_w4_fused_launch(x, qw, scales, zeros, false, y, M, N, K, workspace, gws, err, s);
    void* wb = static_cast<char*>(workspace) + gws;
    cudaError_t e = prefill_dequant_rows_launch(qw, scales, zeros, N, K, wb, s);
    if (e != cudaSuccess) return e;
    return prefill_gemm_launch(x, wb, y, M, N, K, workspace, gws, err, s);
}

}  // namespace fb
