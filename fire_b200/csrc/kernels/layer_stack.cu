// Persistent Qwen3 layer-stack decode kernel (see layer_stack.h for the contract).
//
// Per layer (src/model/qwen.cpp:190-292):
//   phase 0  qkv   = W_qkv . rmsnorm(hidden, attn_norm)
//   phase 1  attention: q/k RMSNorm + RoPE, KV-cache write of this position, softmax(q.K)/sqrt(d) . V
//   phase 2  attn_res = hidden + W_o . attn_out
//   phase 3  act  = silu(W_gate . x) * (W_up . x),  x = rmsnorm(attn_res, ffn_norm)
//   phase 4  hidden = attn_res + W_down . act
//
// Work split. A GEMV phase is cut into units of 16 rows x (K / kparts); units of every
// phase of every layer are dealt to the CTAs round-robin in one running sequence, so
// each CTA streams about the same number of bytes per layer. An attention unit is one
// KV head x 128 keys. A CTA's items (2208-byte weight items, or 4 K or V rows) form one
// sequence in a fixed order that the producer and the consumers both derive from the
// step's position.
//
// INT4 math (as in w4_mma.cu): x is staged once per phase as fixed-point base-128
// digits; each item is four u8 x s8 m16n8k32 MMAs per 128-group with exact int32 sums,
// recombined in FP32 with the zero point and the group scale. An item's 16 row sums go
// to a shared-memory slot; the warp that completes a unit adds the slots in item order
// (deterministic) and applies the phase epilogue. Split-K units write global partials;
// the last one of a row tile (atomic ticket) adds them in K order.
//
// Synchronisation. Ring slots have "full" (TMA transaction count) and "empty" (one
// consumer-warp arrival) mbarriers. Phases wait on per-(layer, phase) counters that
// each CTA bumps once (a release reduction after a consumer barrier) when its units of
// that phase are done; readers take the counter with an acquire load.
// Every wait is bounded: on timeout the kernel records kStackErrTimeout in the decode
// state, stops issuing copies, keeps the barrier structure of its consumer warps
// intact (work is skipped, barriers are still met), waits for its copies in flight and
// returns.
#include "common.cuh"
#include "layer_stack.h"

namespace fb {
namespace {

constexpr int W = kStackConsumerWarps;
constexpr int kConsumers = W * 32;
// Every wait gives up after kWaitNs of GPU time (a healthy wait lasts microseconds);
// kSpinLimit is only a backstop on the number of polls.
constexpr unsigned long long kWaitNs = 200ull * 1000 * 1000;
constexpr int kSpinLimit = 1 << 26;
constexpr int kMaxG = kStackMaxGroup;

__device__ __forceinline__ uint32_t su32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// TMA bulk copy global -> this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// tensor-parallel exchange words: tag << 32 | float bits, one aligned 64-bit access each
// (single-copy atomic), relaxed at system scope: no fence, the tag is the validity
__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// true once `t0` lies more than kWaitNs in the past (checked every 64 polls)
__device__ __forceinline__ bool overdue(int i, unsigned long long t0) {
    return (i & 63) == 63 && gtime() - t0 > kWaitNs;
}
__device__ __forceinline__ void stamp(const StackArgs& a, int l, int p, int k) {
    if (a.trace != nullptr)
        a.trace[((static_cast<size_t>(blockIdx.x) * a.L + l) * kStackPhases + p) * kStackTraceSlots + k] = gtime();
}
__device__ __forceinline__ void record(const StackArgs& a, int l, int p, int k, unsigned long long v) {
    if (a.trace != nullptr)
        a.trace[((static_cast<size_t>(blockIdx.x) * a.L + l) * kStackPhases + p) * kStackTraceSlots + k] = v;
}
__device__ __forceinline__ bool state_failed(const DecodeState* st) {
    return *reinterpret_cast<const volatile int*>(&st->error) != 0;
}
__device__ __forceinline__ void record_timeout(DecodeState* st) { atomicCAS(&st->error, 0, kStackErrTimeout); }

// consumer-only named barrier (the producer warp never joins)
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Shared {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    uint8_t* x;       // digits [groups][4 digits][4 quads][4 mma][8 B], then float2 [groups]
    float* part;      // [units of the phase][ipu][16] per-item row sums
    int* ucnt;        // [max_units]
    float* xv;        // tensor parallel: the o / down row sums of the CTA's units [max_units][16]
    float* red;       // [32]
    int* misc;        // [0] failed flag, [2] attention "last" flag, [4..5] traced wait cycles (u64)
};

__device__ __forceinline__ Shared carve(const StackArgs& a, uint8_t* base) {
    Shared s;
    s.ring = base;
    s.full = reinterpret_cast<uint64_t*>(base + a.off_bar);
    s.empty = s.full + a.ring_slots;
    s.x = base + a.off_x;
    s.part = reinterpret_cast<float*>(base + a.off_part);
    s.ucnt = reinterpret_cast<int*>(base + a.off_ucnt);
    s.xv = reinterpret_cast<float*>(base + a.off_xv);
    s.red = reinterpret_cast<float*>(base + a.off_misc);
    s.misc = reinterpret_cast<int*>(base + a.off_misc + 32 * sizeof(float));
    return s;
}

// ---------------------------------------------------------------------------------
// Schedule shared by the producer and the consumers.
struct Sched {
    int grid, n, nch, att_units, layer_units;
    __device__ int units(const StackArgs& a, int p) const { return p == 1 ? att_units : a.ph[p].units; }
    __device__ int prefix(const StackArgs& a, int p) const {
        int s = 0;
        for (int q = 0; q < p; ++q) s += units(a, q);
        return s;
    }
    // this CTA's units of (l, p): u = first + k * grid, k < count
    __device__ void mine(const StackArgs& a, int l, int p, int* first, int* count) const {
        const int U = units(a, p);
        const long long rot = (static_cast<long long>(l) * layer_units + prefix(a, p)) % grid;
        const int r = static_cast<int>((blockIdx.x + grid - rot) % grid);
        *first = r;
        *count = r < U ? (U - 1 - r) / grid + 1 : 0;
    }
    __device__ int att_items(int c) const {  // K (or V) items of attention chunk c
        const int T = min(kStackChunk, n - c * kStackChunk);
        return (T + 3) >> 2;
    }
};

__device__ __forceinline__ Sched make_sched(const StackArgs& a, int pos) {
    Sched s;
    s.grid = a.grid;
    s.n = pos + 1;
    s.nch = (s.n + kStackChunk - 1) / kStackChunk;
    s.att_units = a.kv_heads * s.nch;
    s.layer_units = s.att_units;
    for (int p = 0; p < kStackPhases; ++p)
        if (p != 1) s.layer_units += a.ph[p].units;
    return s;
}

__device__ __forceinline__ const uint8_t* phase_items(const StackLayer& L, int p) {
    return p == 0 ? L.qkv : (p == 2 ? L.o : (p == 3 ? L.gu : L.down));
}

// ---------------------------------------------------------------------------------
// Producer: the producer warp streams the CTA's item sequence into the ring, one unit
// per step: lane j issues item j of the unit (a single issuing thread caps the copy
// rate far below HBM speed). Steps are separated by __syncwarp, so no lane runs more
// than one step (<= 32 items) ahead of another; with >= 32 slots the parity of a
// slot's "empty" barrier cannot alias.
struct RingCursor {
    int slot = 0;          // slot of item `seq`
    unsigned parity = 0;   // its phase parity ((seq / S) & 1)
    unsigned seq = 0;
};

__device__ void producer(const StackArgs& a, const Shared& sh, const Sched& sc, int pos) {
    const int S = a.ring_slots;
    const int lane = threadIdx.x & 31;
    RingCursor cur;
    bool ok = true;
    // this lane's item of the step: slot and parity of seq + lane (lane < 32 <= S)
    auto lane_slot = [&](int* slot, unsigned* parity) {
        int sl = cur.slot + lane;
        unsigned par = cur.parity;
        if (sl >= S) {
            sl -= S;
            par ^= 1u;
        }
        *slot = sl;
        *parity = par;
    };
    // wait until the consumer of the previous item in `slot` released it
    unsigned long long waited = 0;
    auto acquire = [&](unsigned seq, int slot, unsigned parity) -> bool {
        if (seq < static_cast<unsigned>(S)) return true;
        uint64_t* b = &sh.empty[slot];
        const long long c0 = a.trace != nullptr ? clock64() : 0;
        const unsigned long long t0 = gtime();
        for (int i = 0; i < kSpinLimit; ++i) {
            if (mbar_try(b, parity ^ 1u)) {
                if (a.trace != nullptr) waited += clock64() - c0;
                return true;
            }
            if ((i & 255) == 255 && state_failed(a.state)) return false;
            if (overdue(i, t0)) break;
        }
        record_timeout(a.state);
        return false;
    };
    auto advance = [&](int m) {
        cur.seq += static_cast<unsigned>(m);
        cur.slot += m;
        while (cur.slot >= S) {
            cur.slot -= S;
            cur.parity ^= 1u;
        }
        if (lane == 0) *reinterpret_cast<volatile unsigned*>(&sh.misc[6]) = cur.seq;  // for the L2 prefetcher
    };
    const size_t kv_stride = static_cast<size_t>(a.kv_dim);
    for (int l = 0; l < a.L && ok; ++l) {
        const StackLayer& Ly = a.layers[l];
        for (int p = 0; p < kStackPhases && ok; ++p) {
            int first, count;
            sc.mine(a, l, p, &first, &count);
            if (p == 1) {
                const size_t layer_off = static_cast<size_t>(l) * a.capacity * kv_stride;
                for (int k = 0; k < count && ok; ++k) {
                    const int u = first + k * sc.grid;
                    const int c = u / a.kv_heads, h = u % a.kv_heads;
                    const int t0 = c * kStackChunk, ni = sc.att_items(c);  // ni <= 32
                    for (int half = 0; half < 2 && ok; ++half) {
                        const float* base = (half ? a.vcache : a.kcache) + layer_off + static_cast<size_t>(h) * 128;
                        bool mine_ok = true;
                        if (lane < ni) {
                            int slot;
                            unsigned parity;
                            lane_slot(&slot, &parity);
                            mine_ok = acquire(cur.seq + lane, slot, parity);
                            if (mine_ok) {
                                uint8_t* dst = sh.ring + static_cast<size_t>(slot) * kItemBytes;
                                // rows t < pos only: row pos is produced in this step (from qkv)
                                const int t = t0 + 4 * lane;
                                const int rows = max(0, min(4, pos - t));
                                mbar_expect_tx(&sh.full[slot], static_cast<unsigned>(rows) * 512u);
                                for (int r = 0; r < rows; ++r)
                                    bulk_load(dst + r * 512, base + static_cast<size_t>(t + r) * kv_stride, 512u,
                                              &sh.full[slot]);
                            }
                        }
                        ok = !__any_sync(0xffffffffu, !mine_ok);
                        advance(ni);
                    }
                }
            } else {
                const StackPhase& ph = a.ph[p];
                const uint8_t* items = phase_items(Ly, p);
                for (int k = 0; k < count && ok; ++k) {
                    const int u = first + k * sc.grid;
                    const int tile = u / ph.kparts, kp = u % ph.kparts;
                    const uint8_t* unit = items + (static_cast<size_t>(tile) * ph.ipr + static_cast<size_t>(kp) * ph.ipu) * kItemBytes;
                    // the unit's items in steps of at most 32 (one per lane)
                    for (int j0 = 0; j0 < ph.ipu && ok; j0 += 32) {
                        const int m = min(32, ph.ipu - j0);
                        bool mine_ok = true;
                        if (lane < m) {
                            int slot;
                            unsigned parity;
                            lane_slot(&slot, &parity);
                            mine_ok = acquire(cur.seq + lane, slot, parity);
                            if (mine_ok) {
                                mbar_expect_tx(&sh.full[slot], kItemBytes);
                                bulk_load(sh.ring + static_cast<size_t>(slot) * kItemBytes,
                                          unit + static_cast<size_t>(j0 + lane) * kItemBytes, kItemBytes, &sh.full[slot]);
                            }
                        }
                        ok = !__any_sync(0xffffffffu, !mine_ok);
                        advance(m);
                    }
                }
            }
            if (count > 0 && lane == 0) {
                stamp(a, l, p, 4);
                record(a, l, p, 6, waited);
            }
            waited = 0;
        }
    }
    // every issued copy must land before the CTA may exit: lane 0 walks back over the
    // last min(seq, S) items (slot and parity of each use)
    if (lane == 0) {
        int slot = cur.slot;
        unsigned parity = cur.parity;
        const unsigned n = cur.seq < static_cast<unsigned>(S) ? cur.seq : static_cast<unsigned>(S);
        for (unsigned i = 0; i < n; ++i) {
            if (--slot < 0) {
                slot = S - 1;
                parity ^= 1u;
            }
            const unsigned long long t0 = gtime();
            for (int it = 0; it < kSpinLimit; ++it)
                if (mbar_try(&sh.full[slot], parity) || overdue(it, t0)) break;
        }
    }
}

// ---------------------------------------------------------------------------------
// L2 prefetcher: walks the producer's item sequence kStackPrefetchAhead items ahead of
// the ring and asks L2 to fetch each item (weights: one 2208-byte item per lane; K/V:
// one 512-byte row per lane), so phases that stall on latency keep HBM busy and the ring
// refills from L2. Prefetches carry no completion, so this warp never blocks the others.
__device__ __forceinline__ void prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ void prefetcher(const StackArgs& a, const Shared& sh, const Sched& sc, int pos) {
    const int lane = threadIdx.x & 31;
    unsigned seq = 0;
    // wait (bounded) until the ring producer is within reach of item `upto`
    auto throttle = [&](unsigned upto) -> bool {
        const unsigned long long t0 = gtime();
        for (int i = 0; i < kSpinLimit; ++i) {
            const unsigned prod = *reinterpret_cast<volatile unsigned*>(&sh.misc[6]);
            if (prod + kStackPrefetchAhead >= upto) return true;
            if (*reinterpret_cast<volatile int*>(&sh.misc[0]) != 0 || overdue(i, t0)) return false;
            __nanosleep(200);
        }
        return false;
    };
    const size_t kv_stride = static_cast<size_t>(a.kv_dim);
    for (int l = 0; l < a.L; ++l) {
        const StackLayer& Ly = a.layers[l];
        for (int p = 0; p < kStackPhases; ++p) {
            int first, count;
            sc.mine(a, l, p, &first, &count);
            if (p == 1) {
                const size_t layer_off = static_cast<size_t>(l) * a.capacity * kv_stride;
                for (int k = 0; k < count; ++k) {
                    const int u = first + k * sc.grid;
                    const int c = u / a.kv_heads, h = u % a.kv_heads;
                    const int t0 = c * kStackChunk, ni = sc.att_items(c);
                    const int rows = min(kStackChunk, pos - t0);  // rows t < pos
                    for (int half = 0; half < 2; ++half) {
                        if (!throttle(seq + ni)) return;
                        const float* base = (half ? a.vcache : a.kcache) + layer_off + static_cast<size_t>(h) * 128;
                        for (int r = lane; r < rows; r += 32) prefetch_l2(base + static_cast<size_t>(t0 + r) * kv_stride, 512u);
                        seq += ni;
                    }
                }
            } else {
                const StackPhase& ph = a.ph[p];
                const uint8_t* items = phase_items(Ly, p);
                for (int k = 0; k < count; ++k) {
                    if (!throttle(seq + ph.ipu)) return;
                    const int u = first + k * sc.grid;
                    const int tile = u / ph.kparts, kp = u % ph.kparts;
                    const uint8_t* unit =
                        items + (static_cast<size_t>(tile) * ph.ipr + static_cast<size_t>(kp) * ph.ipu) * kItemBytes;
                    for (int j = lane; j < ph.ipu; j += 32) prefetch_l2(unit + static_cast<size_t>(j) * kItemBytes, kItemBytes);
                    seq += ph.ipu;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------
// Consumer helpers
__device__ __forceinline__ bool failed(const Shared& sh) {
    return *reinterpret_cast<volatile int*>(&sh.misc[0]) != 0;
}
__device__ __forceinline__ void mark_failed(const Shared& sh) { *reinterpret_cast<volatile int*>(&sh.misc[0]) = 1; }

// all lanes of a warp wait for ring item `seq` (each lane observes the barrier phase, so
// the TMA-written bytes are visible to all); the result is warp-uniform; false if the
// kernel is failing
struct Slot {
    int index;
    unsigned parity;
};
__device__ __forceinline__ Slot slot_of(unsigned seq, int S) {
    const unsigned q = seq / static_cast<unsigned>(S);
    return Slot{static_cast<int>(seq - q * static_cast<unsigned>(S)), q & 1u};
}

__device__ bool wait_item(const StackArgs& a, const Shared& sh, Slot sl, long long& waited) {
    const unsigned parity = sl.parity;
    uint64_t* b = &sh.full[sl.index];
    // (try_wait may itself block for a while, so the traced time starts before it)
    const long long c0 = a.trace != nullptr ? clock64() : 0;
    if (__all_sync(0xffffffffu, mbar_try(b, parity))) {  // common case: already landed
        if (a.trace != nullptr) waited += clock64() - c0;
        return true;
    }
    if (__any_sync(0xffffffffu, failed(sh))) return false;
    const unsigned long long t0 = gtime();
    bool ok = false;
    for (int i = 0; i < kSpinLimit; ++i) {
        if (mbar_try(b, parity)) {
            ok = true;
            break;
        }
        if ((i & 255) == 255 && state_failed(a.state)) break;
        if (overdue(i, t0)) break;
    }
    if (a.trace != nullptr) waited += clock64() - c0;
    if (__all_sync(0xffffffffu, ok)) return true;
    if ((threadIdx.x & 31) == 0) {
        if (!state_failed(a.state)) record_timeout(a.state);
        mark_failed(sh);
    }
    return false;
}
__device__ __forceinline__ void release_item(const Shared& sh, Slot sl) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sh.empty[sl.index]);
}

// thread 0 of the consumers waits until `target` CTAs finished (l, p); then all consumers sync
__device__ void wait_phase(const StackArgs& a, const Shared& sh, int l, int p, unsigned target) {
    if (threadIdx.x == 0 && !failed(sh)) {
        const unsigned* ctr = a.sync + l * kStackPhases + p;
        bool ok = false;
        const unsigned long long t0 = gtime();
        for (int i = 0; i < kSpinLimit; ++i) {
            if (ld_acquire(ctr) >= target) { ok = true; break; }
            if ((i & 63) == 63 && state_failed(a.state)) break;
            if (overdue(i, t0)) break;
            __nanosleep(32);
        }
        if (!ok) {
            if (!state_failed(a.state)) record_timeout(a.state);
            mark_failed(sh);
        }
    }
    cbar();
}
// one thread publishes the phase after a consumer barrier: a release reduction orders
// every store the CTA made before the barrier ahead of the counter update
__device__ __forceinline__ void signal_phase(const StackArgs& a, int l, int p) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync + l * kStackPhases + p) : "memory");
}

// Tensor parallel: the value of an exchange word of layer l (see StackArgs); a wait that
// runs out marks the kernel failed and yields 0
__device__ __forceinline__ unsigned xtag(unsigned tag_base, int l) { return tag_base + static_cast<unsigned>(l) + 1u; }
__device__ float word_wait(const StackArgs& a, const Shared& sh, const unsigned long long* p, unsigned tag) {
    unsigned long long w = ld_word_sys(p);
    if (static_cast<unsigned>(w >> 32) == tag) return __uint_as_float(static_cast<unsigned>(w));
    const unsigned long long t0 = gtime();
    for (int i = 0; i < kSpinLimit; ++i) {
        w = ld_word_sys(p);
        if (static_cast<unsigned>(w >> 32) == tag) return __uint_as_float(static_cast<unsigned>(w));
        if ((i & 63) == 63 && (failed(sh) || state_failed(a.state))) break;
        if (overdue(i, t0)) {
            if (!state_failed(a.state)) record_timeout(a.state);
            break;
        }
    }
    mark_failed(sh);
    return 0.0f;
}
// (p_0 + p_1 + ... + p_{tp-1}) of elements e0..e0+3 from this rank's exchange words `ll`
// [tp][n], added in rank order. The words of kWordRanks ranks are loaded together (one
// round trip per kWordRanks ranks, not one per word); a word still holding an older tag
// is then polled alone.
constexpr int kWordRanks = 2;
__device__ float4 word_sum4(const StackArgs& a, const Shared& sh, const unsigned long long* ll, int n, int e0,
                            unsigned tag) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < a.tp; r0 += kWordRanks) {
        const int nr = min(kWordRanks, a.tp - r0);
        unsigned long long w[kWordRanks][4];
#pragma unroll
        for (int j = 0; j < kWordRanks; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c)
                w[j][c] = j < nr ? ld_word_sys(ll + static_cast<size_t>(r0 + j) * n + e0 + c) : 0ull;
#pragma unroll
        for (int j = 0; j < kWordRanks; ++j) {
            if (j >= nr) break;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float v = static_cast<unsigned>(w[j][c] >> 32) == tag
                                    ? __uint_as_float(static_cast<unsigned>(w[j][c]))
                                    : word_wait(a, sh, ll + static_cast<size_t>(r0 + j) * n + e0 + c, tag);
                s[c] = r0 + j == 0 ? v : s[c] + v;
            }
        }
    }
    return make_float4(s[0], s[1], s[2], s[3]);
}

__device__ float csum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    cbar();
    if (lane == 0) red[warp] = v;
    cbar();
    return warp_sum(lane < W ? red[lane] : 0.0f);
}

// Stage x as fixed-point digits per 128-group (w4_mma.cu layout). With an RMSNorm the
// digits hold x * w; the scalar 1/rms multiplies the row sums in the epilogue (the same
// product, reassociated), so no block-wide reduction sits between the input and the
// first MMA: each warp leaves its sum of squares in red[warp].
// `own`: a unit has exactly W items and warp w consumes item w of every unit, so it
// stages only the groups of those items (2 per K part) and needs no barrier after.
// Otherwise warp w stages groups w, w + W, ... and the consumers sync afterwards.
constexpr int kStageRegs = 8;

__device__ __forceinline__ void store_digits(const float (&v)[4], int g, const Shared& sh, int groups) {
    const int lane = threadIdx.x & 31;
    uint8_t* xd = sh.x;
    float2* xg = reinterpret_cast<float2*>(sh.x + static_cast<size_t>(groups) * 512);
    // group max of |v| (non-negative floats order like their bit patterns)
    const uint32_t mb = max(max(__float_as_uint(fabsf(v[0])), __float_as_uint(fabsf(v[1]))),
                            max(__float_as_uint(fabsf(v[2])), __float_as_uint(fabsf(v[3]))));
    const uint32_t gm = __reduce_max_sync(0xffffffffu, mb);
    // max in [2^ex, 2^(ex+1)): x * 2^(25-ex) has magnitude < 2^26
    const int ex = static_cast<int>((gm >> 23) & 0xFF) - 127;
    int sh_ = 25 - ex;
    if (gm == 0 || sh_ > 126) sh_ = 126;
    const float up = __uint_as_float(static_cast<uint32_t>(127 + sh_) << 23);
    const float down = __uint_as_float(static_cast<uint32_t>(127 - sh_) << 23);
    int fx[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) fx[e] = __float2int_rn(v[e] * up);
    // exact integer group sum: |lane sum| < 2^28, reduced as 15 high + 13 low bits
    const int ls = (fx[0] + fx[1]) + (fx[2] + fx[3]);
    const int shi = __reduce_add_sync(0xffffffffu, ls >> 13);
    const int slo = __reduce_add_sync(0xffffffffu, ls & 0x1FFF);
    if (lane == 0) xg[g] = make_float2(fmaf(static_cast<float>(shi), 8192.0f, static_cast<float>(slo)), down);
    // digits = bit fields of the two's complement: bits 0-6, 7-13, 14-20 (unsigned,
    // 0..127) and the arithmetic shift by 21 (signed, -32..31); x = d0 + 2^7 d1 + 2^14 d2 + 2^21 d3
    const int c = lane >> 3, j = (lane >> 1) & 3, hi = lane & 1;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
        int d[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) d[e] = n < 3 ? (fx[e] >> (7 * n)) & 127 : fx[e] >> 21;
        uint8_t* slot = xd + (((static_cast<size_t>(g) * 4 + n) * 4 + c) * 4 + j) * 8;
        *reinterpret_cast<uint16_t*>(slot + 2 * hi) = static_cast<uint16_t>(__byte_perm(d[0], d[2], 0x0040));
        *reinterpret_cast<uint16_t*>(slot + 4 + 2 * hi) = static_cast<uint16_t>(__byte_perm(d[1], d[3], 0x0040));
    }
}

// Tensor parallel (parts != nullptr): the input is x + (p_0 + p_1 + ... ) over the ranks'
// partials `parts` [tp][k] (this rank's exchange words, waited for by tag), the same sum on
// every rank; of
// the `writers` CTAs taking part in the phase, the one of rank `writer` = g mod writers
// also stores group g of the sum to `keep`.
__device__ void stage_x(const StackArgs& a, const float* x, const float* norm_w, const StackPhase& ph, bool own,
                        const Shared& sh, const unsigned long long* parts, unsigned tag, float* keep, int writer,
                        int writers) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int groups = ph.k >> 7;
    const int mine = own ? 2 * ph.kparts : (groups - warp + W - 1) / W;  // groups this warp stages
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* w4 = reinterpret_cast<const float4*>(norm_w);
    // own: warp w consumes item w of every unit, i.e. groups 2(kp*W + w) + {0, 1}
    auto group_of = [&](int i) { return own ? 2 * ((i >> 1) * W + warp) + (i & 1) : warp + i * W; };
    float ss = 0.0f;
    for (int b0 = 0; b0 < mine; b0 += kStageRegs) {
        float4 v[kStageRegs];
#pragma unroll
        for (int i = 0; i < kStageRegs; ++i)
            v[i] = b0 + i < mine ? __ldcg(x4 + group_of(b0 + i) * 32 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (parts != nullptr) {
#pragma unroll
            for (int i = 0; i < kStageRegs; ++i) {
                if (b0 + i < mine) {
                    const int idx = group_of(b0 + i) * 32 + lane;
                    const float4 sm = word_sum4(a, sh, parts, ph.k, 4 * idx, tag);
                    v[i] = make_float4(v[i].x + sm.x, v[i].y + sm.y, v[i].z + sm.z, v[i].w + sm.w);
                    if (group_of(b0 + i) % writers == writer) reinterpret_cast<float4*>(keep)[idx] = v[i];
                }
            }
        }
        if (norm_w != nullptr) {
#pragma unroll
            for (int i = 0; i < kStageRegs; ++i) {
                if (b0 + i < mine) {
                    ss = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, ss))));
                    const float4 w = __ldg(w4 + group_of(b0 + i) * 32 + lane);
                    v[i] = make_float4(v[i].x * w.x, v[i].y * w.y, v[i].z * w.z, v[i].w * w.w);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kStageRegs; ++i) {
            if (b0 + i < mine) {
                const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
                store_digits(e, group_of(b0 + i), sh, groups);
            }
        }
    }
    if (norm_w != nullptr) {
        ss = warp_sum(ss);
        if (lane == 0) sh.red[warp] = ss;
    }
}

// Row sums of one item (16 rows x 256 K) against the staged digits; lanes with c == 0
// return rows gq (first) and gq + 8 (second).
struct ItemRegs {
    uint4 wv[2][2];  // [row half][group]: this lane's 16-byte chunk
    float2 s0, s1;   // scales of rows gq, gq + 8 (both groups)
    uint32_t z0, z1; // zero points of rows gq, gq + 8 (group 0 low byte)
};

__device__ __forceinline__ ItemRegs load_item(const uint8_t* item) {
    const int lane = threadIdx.x & 31, gq = lane >> 2;
    ItemRegs r;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
            r.wv[h][gi] = reinterpret_cast<const uint4*>(item)[(h * 2 + gi) * 32 + lane];
    r.s0 = *reinterpret_cast<const float2*>(item + kItemScaleOff + gq * 8);
    r.s1 = *reinterpret_cast<const float2*>(item + kItemScaleOff + (gq + 8) * 8);
    r.z0 = *reinterpret_cast<const uint16_t*>(item + kItemZeroOff + gq * 2);
    r.z1 = *reinterpret_cast<const uint16_t*>(item + kItemZeroOff + (gq + 8) * 2);
    return r;
}

// Accumulate one item (16 rows x 256 K) against the staged digits into this lane's
// share of rows gq (acc0) and gq + 8 (acc1); the quad's four lanes are added later.
// Lane c of a quad holds digit columns 2c, 2c+1 of the MMA result: c = 0 digits 0/1,
// c = 1 digits 2/3 (weight 128^2), c >= 2 the unused zero columns.
// The B operand (x digits) and the float2 {sum, 2^-e} of the two 128-groups of an item.
struct Digits {
    uint4 b[2][2];  // [group][2 x 16 bytes]: digit column gq (lanes gq < 4), quad c
    float2 gx[2];
};

__device__ __forceinline__ Digits load_digits(const Shared& sh, int groups, int g0) {
    const int lane = threadIdx.x & 31, gq = lane >> 2, c = lane & 3;
    const float2* xg = reinterpret_cast<const float2*>(sh.x + static_cast<size_t>(groups) * 512);
    Digits d;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        d.b[gi][0] = d.b[gi][1] = make_uint4(0, 0, 0, 0);
        if (gq < 4) {
            const uint4* src =
                reinterpret_cast<const uint4*>(sh.x + ((static_cast<size_t>(g0 + gi) * 4 + gq) * 4 + c) * 32);
            d.b[gi][0] = src[0];
            d.b[gi][1] = src[1];
        }
        d.gx[gi] = xg[g0 + gi];
    }
    return d;
}

// Accumulate one item (16 rows x 256 K) against its groups' digits into this lane's
// share of rows gq (acc0) and gq + 8 (acc1); the quad's four lanes are added later.
// Lane c of a quad holds digit columns 2c, 2c+1 of the MMA result: c = 0 digits 0/1,
// c = 1 digits 2/3 (weight 128^2), c >= 2 the unused zero columns.
__device__ __forceinline__ void item_accumulate(const ItemRegs& it, const Digits& dg, float& acc0, float& acc1) {
    const int lane = threadIdx.x & 31, c = lane & 3;
    const auto& wv = it.wv;
    const float cw = c == 0 ? 1.0f : 16384.0f;
    const float zmul = c == 0 ? -1.0f : 0.0f;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        const uint4* b4 = dg.b[gi];
        const uint32_t wg[4] = {wv[0][gi].x, wv[0][gi].y, wv[0][gi].z, wv[0][gi].w};
        const uint32_t wh[4] = {wv[1][gi].x, wv[1][gi].y, wv[1][gi].z, wv[1][gi].w};
        int da[4] = {0, 0, 0, 0}, db[4] = {0, 0, 0, 0};
        constexpr uint32_t m = 0x0F0F0F0Fu;
        mma_u8s8(da, wg[0] & m, wh[0] & m, (wg[0] >> 4) & m, (wh[0] >> 4) & m, b4[0].x, b4[0].y);
        mma_u8s8(db, wg[1] & m, wh[1] & m, (wg[1] >> 4) & m, (wh[1] >> 4) & m, b4[0].z, b4[0].w);
        mma_u8s8(da, wg[2] & m, wh[2] & m, (wg[2] >> 4) & m, (wh[2] >> 4) & m, b4[1].x, b4[1].y);
        mma_u8s8(db, wg[3] & m, wh[3] & m, (wg[3] >> 4) & m, (wh[3] >> 4) & m, b4[1].z, b4[1].w);
        // d_even + 128 d_odd: exact in int32 (|column sum| <= 128 * 15 * 127), one rounding to float
        const int t0 = (da[0] + db[0]) + 128 * (da[1] + db[1]);
        const int t1 = (da[2] + db[2]) + 128 * (da[3] + db[3]);
        const float2 gx = dg.gx[gi];
        // zero point as float: 2^23 + z, minus 2^23
        const float zf0 = __uint_as_float(__byte_perm(it.z0, 0x4B000000u, 0x7540 + gi)) - 8388608.0f;
        const float zf1 = __uint_as_float(__byte_perm(it.z1, 0x4B000000u, 0x7540 + gi)) - 8388608.0f;
        const float f0 = fmaf(zmul * zf0, gx.x, static_cast<float>(t0) * cw);
        const float f1 = fmaf(zmul * zf1, gx.x, static_cast<float>(t1) * cw);
        acc0 = fmaf((gi ? it.s0.y : it.s0.x) * gx.y, f0, acc0);
        acc1 = fmaf((gi ? it.s1.y : it.s1.x) * gx.y, f1, acc1);
    }
}

// Epilogue of one finished row tile; lane r < 16 holds the full sum of row tile*16 + r.
// The residual input of a phase's rows (hidden for o, attn_res for down); it is final
// before the phase starts, so it is read ahead of the epilogue.
template <bool kTp>
__device__ __forceinline__ const float* phase_residual(const StackArgs& a, int p) {
    if (kTp) return nullptr;  // added to the reduced sums when the next phase stages them
    return p == 2 ? a.hidden_buf : (p == 4 ? a.attn_res : nullptr);
}

template <bool kTp>
__device__ __forceinline__ void tile_epilogue(const StackArgs& a, int p, int tile, float v, float res) {
    const int lane = threadIdx.x & 31;
    const float up = __shfl_down_sync(0xffffffffu, v, 8);
    if (lane >= 16) return;
    const int row = tile * 16 + lane;
    if (p == 0) {
        a.qkv[row] = v;
    } else if (p == 2) {
        if (kTp) {  // row-parallel partial sums to every rank (the residual is added when staging)
            for (int r = 0; r < a.tp; ++r) a.xo[r][static_cast<size_t>(a.rank) * a.hidden + row] = v;
        } else {
            a.attn_res[row] = res + v;  // residual (qwen.cpp:262)
        }
    } else if (p == 3) {
        if (lane < 8) {
            const float silu = v * 1.0f / (1.0f + expf(-v));  // swiglu_kernel.cu:11-12
            a.act[tile * 8 + lane] = silu * up;
        }
    } else if (kTp) {
        for (int r = 0; r < a.tp; ++r) a.xdown[r][static_cast<size_t>(a.rank) * a.hidden + row] = v;
    } else {
        a.hidden_buf[row] = res + v;  // residual (qwen.cpp:291)
    }
}

// Finish unit k of this CTA's units in phase p (one warp): add its item partial sums in
// item order and apply the epilogue; split-K partials meet through a per-tile ticket.
template <bool kTp>
__device__ void finish_unit(const StackArgs& a, const Shared& sh, const Sched& sc, int p, int first, int k,
                            float scale, float res) {
    const int lane = threadIdx.x & 31;
    const StackPhase& ph = a.ph[p];
    const int u = first + k * sc.grid;
    const int tile = u / ph.kparts, kp = u % ph.kparts;
    float v = 0.0f;
    if (lane < 16) {
        const float* pp = sh.part + static_cast<size_t>(k) * ph.ipu * 16 + lane;
        float v4[4] = {0.f, 0.f, 0.f, 0.f};  // four chains, combined in a fixed order
        int j = 0;
        for (; j + 4 <= ph.ipu; j += 4) {
#pragma unroll
            for (int q = 0; q < 4; ++q) v4[q] += pp[(j + q) * 16];
        }
        for (; j < ph.ipu; ++j) v4[0] += pp[j * 16];
        v = ((v4[0] + v4[1]) + (v4[2] + v4[3])) * scale;
    }
    if (kTp && (p == 2 || p == 4)) {  // sent to every rank after the local signal (kparts == 1)
        if (lane < 16) sh.xv[k * 16 + lane] = v;
    } else if (ph.kparts == 1) {
        tile_epilogue<kTp>(a, p, tile, v, res);
    } else {
        if (lane < 16) a.kpart[static_cast<size_t>(kp) * ph.n + tile * 16 + lane] = v;
        __threadfence();
        __syncwarp();
        unsigned* ticket = a.sync + a.L * kStackPhases + a.kv_heads + tile;
        int last = 0;
        if (lane == 0) last = atomicAdd(ticket, 1u) == static_cast<unsigned>(ph.kparts - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
            v = 0.0f;
            if (lane < 16)
                for (int q = 0; q < ph.kparts; ++q) v += __ldcg(a.kpart + static_cast<size_t>(q) * ph.n + tile * 16 + lane);
            tile_epilogue<kTp>(a, p, tile, v, res);
            if (lane == 0) *ticket = 0u;
        }
    }
}

template <bool kTp>
__device__ void gemv_phase(const StackArgs& a, const Shared& sh, const Sched& sc, int l, int p, int first, int count,
                           unsigned seq_base, unsigned tag_base) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const StackPhase& ph = a.ph[p];
    const int groups = ph.k >> 7;
    const int total = count * ph.ipu;
    long long waited = 0;
    // residual rows of the unit this warp finishes first (k = warp), read ahead
    const float* resid = phase_residual<kTp>(a, p);
    float res0 = 0.0f;
    if (resid != nullptr && warp < count && lane < 16)
        res0 = __ldcg(resid + ((first + warp * sc.grid) / ph.kparts) * 16 + lane);
    // this warp's items s = warp, warp + W, ...: unit k, item j, ring slot and parity all
    // advance incrementally (no division per item; W < ring slots)
    const int S = a.ring_slots;
    int k = warp / ph.ipu, j = warp % ph.ipu;
    Slot sl = slot_of(seq_base + static_cast<unsigned>(warp), S);
    int kp = ph.kparts == 1 ? 0 : (first + k * sc.grid) % ph.kparts;
    // with one K part and W items per unit, every item of this warp uses the same two
    // groups: their digits stay in registers for the phase
    const bool fixed = ph.kparts == 1 && ph.ipu == W;
    Digits dg{};
    if (fixed && warp < total) dg = load_digits(sh, groups, 2 * j);
    for (int s = warp; s < total; s += W) {
        if (wait_item(a, sh, sl, waited)) {
            const ItemRegs it = load_item(sh.ring + static_cast<size_t>(sl.index) * kItemBytes);
            release_item(sh, sl);
            if (!fixed) dg = load_digits(sh, groups, 2 * (kp * ph.ipu + j));
            float acc0 = 0.0f, acc1 = 0.0f;
            item_accumulate(it, dg, acc0, acc1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if ((lane & 3) == 0) {
                float* dst = sh.part + (static_cast<size_t>(k) * ph.ipu + j) * 16;
                dst[lane >> 2] = acc0;
                dst[(lane >> 2) + 8] = acc1;
            }
        }
        j += W;
        bool new_unit = false;
        while (j >= ph.ipu) {
            j -= ph.ipu;
            ++k;
            new_unit = true;
        }
        if (new_unit && ph.kparts > 1) kp = (first + k * sc.grid) % ph.kparts;
        sl.index += W;
        if (sl.index >= S) {
            sl.index -= S;
            sl.parity ^= 1u;
        }
    }
    if (a.trace != nullptr && lane == 0 && waited > 0)
        atomicAdd(reinterpret_cast<unsigned long long*>(sh.misc + 4), static_cast<unsigned long long>(waited));
    if (threadIdx.x == 0) stamp(a, l, p, 7);
    // all items of the phase are in: finish the units in parallel, then one thread
    // publishes the phase (barrier, then fence + counter: every epilogue store of this
    // CTA is ordered before the counter update)
    cbar();
    if (!failed(sh)) {
        // RMSNorm scale 1/sqrt(mean(x^2) + eps) (rmsnorm_kernel.cu), warp sums added in order
        float scale = 1.0f;
        if (p == 0 || p == 3) {
            float ss = 0.0f;
            for (int w = 0; w < W; ++w) ss += sh.red[w];
            scale = 1.0f / sqrtf(ss / static_cast<float>(ph.k) + a.eps);
        }
        for (int k = warp; k < count; k += W) {
            float res = res0;
            if (k != warp && resid != nullptr && lane < 16)
                res = __ldcg(resid + ((first + k * sc.grid) / ph.kparts) * 16 + lane);
            finish_unit<kTp>(a, sh, sc, p, first, k, scale, res);
        }
    }
    cbar();
    if (threadIdx.x == 0 && !failed(sh)) {
        signal_phase(a, l, p);
        stamp(a, l, p, 3);
        unsigned long long* w = reinterpret_cast<unsigned long long*>(sh.misc + 4);
        record(a, l, p, 5, *w);
        *w = 0;
    }
    if (kTp && (p == 2 || p == 4) && !failed(sh)) {
        // the CTA's rows to every rank's exchange block, tagged, after the local signal: no
        // release follows them (a reader checks each word's tag), so nothing waits for NVLink
        const unsigned tag = xtag(tag_base, l);
        unsigned long long* const* dst = p == 2 ? a.xo : a.xdown;
        for (int i = threadIdx.x; i < count * 16; i += kConsumers) {
            const int row = (first + (i >> 4) * sc.grid) * 16 + (i & 15);
            const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(sh.xv[i]);
            for (int r = 0; r < a.tp; ++r) st_word_sys(dst[r] + static_cast<size_t>(a.rank) * a.hidden + row, w);
        }
    }
}

// One attention unit (G q heads per KV head): KV head h, keys [128c, 128c + T); all consumer warps.
template <int G>
__device__ void attention_unit(const StackArgs& a, const Shared& sh, const Sched& sc, int l, int pos, int c, int h,
                               unsigned base, bool traced) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto mark = [&](int k) {
        if (traced && tid == 0) stamp(a, l, 1, k);
    };
    const int t0 = c * kStackChunk;
    const int T = min(kStackChunk, sc.n - t0);
    const int ni = (T + 3) >> 2;
    const bool holds = c == sc.nch - 1;
    float* qs = reinterpret_cast<float*>(sh.x);  // [G][128]
    float* kp = qs + G * 128;                     // [128] this position's rotated k
    float* vp = kp + 128;                         // [128] and v
    float* wml = vp + 128;                        // [W][G][2] per-warp softmax max / sum
    float* wf = wml + 2 * W * kMaxG;              // [W][G] merge factors exp(m_w - M)
    float* ml = wf + W * kMaxG;                   // [G][2] merge scratch
    float* vpart = ml + 2 * kMaxG;                // [W][G][128]
    float* wc = vpart + W * G * 128;              // [G][max_chunks]
    const bool dead = failed(sh);
    const float* srow = a.rope_sin + static_cast<size_t>(pos) * 64;
    const float* crow = a.rope_cos + static_cast<size_t>(pos) * 64;
    const StackLayer& Ly = a.layers[l];
    // q/k RMSNorm + RoPE (qwen.cpp:222-240); the KV write of this position (kv_cache.cpp:31-73)
    if (!dead && warp < G) {
        const float4 r4 = __ldcg(reinterpret_cast<const float4*>(a.qkv + static_cast<size_t>(h * G + warp) * 128) + lane);
        float v[4] = {r4.x, r4.y, r4.z, r4.w};
        head_norm_rope(v, Ly.q_norm, srow, crow, a.eps);
        reinterpret_cast<float4*>(qs + warp * 128)[lane] = make_float4(v[0], v[1], v[2], v[3]);
    } else if (!dead && warp == G && holds) {
        const float4 k4 = __ldcg(reinterpret_cast<const float4*>(a.qkv + a.q_dim + static_cast<size_t>(h) * 128) + lane);
        const float4 v4 =
            __ldcg(reinterpret_cast<const float4*>(a.qkv + a.q_dim + a.kv_dim + static_cast<size_t>(h) * 128) + lane);
        float kv[4] = {k4.x, k4.y, k4.z, k4.w};
        head_norm_rope(kv, Ly.k_norm, srow, crow, a.eps);
        const float4 kr = make_float4(kv[0], kv[1], kv[2], kv[3]);
        reinterpret_cast<float4*>(kp)[lane] = kr;
        reinterpret_cast<float4*>(vp)[lane] = v4;
        const size_t row = (static_cast<size_t>(l) * a.capacity + pos) * a.kv_dim + static_cast<size_t>(h) * 128;
        reinterpret_cast<float4*>(a.kcache + row)[lane] = kr;
        reinterpret_cast<float4*>(a.vcache + row)[lane] = v4;
    }
    cbar();
    mark(2);
    // Each warp takes items i = warp, warp + W (ni <= 32, so at most two): scores of its
    // keys, a local softmax (max m, sum l) and the unnormalised P.V over its keys, all
    // in registers; the warps' (m, l, o) are merged below (flash-decoding merge).
    // Scores: lanes 8*kk..8*kk+7 hold key kk of an item, float4 sub + 8m of its row.
    const int kk = lane >> 3, sub = lane & 7;
    const int n_keys = sc.n;
    long long waited = 0;
    float scv[2][G];
#pragma unroll
    for (int it = 0; it < 2; ++it)
#pragma unroll
        for (int g = 0; g < G; ++g) scv[it][g] = -INFINITY;
    bool have[2] = {false, false};
    const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int i = warp + it * W;
        if (i >= ni) break;
        const Slot sl = slot_of(base + static_cast<unsigned>(i), a.ring_slots);
        if (!wait_item(a, sh, sl, waited)) break;
        have[it] = true;
        const int t = t0 + 4 * i + kk;
        const float4* src = t == pos ? reinterpret_cast<const float4*>(kp)
                                     : reinterpret_cast<const float4*>(sh.ring + static_cast<size_t>(sl.index) * kItemBytes) + kk * 32;
        float4 kf[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) kf[m] = t < n_keys ? src[sub + 8 * m] : make_float4(0.f, 0.f, 0.f, 0.f);
        release_item(sh, sl);
        // all heads advance together (independent chains)
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; ++g) dot[g] = 0.0f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 q = q4[g * 32 + sub + 8 * m];
                dot[g] = fmaf(q.x, kf[m].x, dot[g]);
                dot[g] = fmaf(q.y, kf[m].y, dot[g]);
                dot[g] = fmaf(q.z, kf[m].z, dot[g]);
                dot[g] = fmaf(q.w, kf[m].w, dot[g]);
            }
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
#pragma unroll
            for (int g = 0; g < G; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], o);
#pragma unroll
        for (int g = 0; g < G; ++g) scv[it][g] = t < n_keys ? dot[g] * a.scale : -INFINITY;
    }
    mark(10);
    // local softmax over this warp's keys (each key is replicated on its 8 lanes)
    float wm[G], wl[G];
#pragma unroll
    for (int g = 0; g < G; ++g) wm[g] = fmaxf(scv[0][g], scv[1][g]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int g = 0; g < G; ++g) wm[g] = fmaxf(wm[g], __shfl_xor_sync(0xffffffffu, wm[g], o));
#pragma unroll
    for (int g = 0; g < G; ++g) {
        wl[g] = 0.0f;
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const float e = have[it] ? expf(scv[it][g] - wm[g]) : 0.0f;
            scv[it][g] = e;
            wl[g] += sub == 0 ? e : 0.0f;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int g = 0; g < G; ++g) wl[g] += __shfl_xor_sync(0xffffffffu, wl[g], o);
    mark(11);
    // unnormalised P.V: lane owns dims 4*lane..4*lane+3 of every head
    float4 acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        if (!have[it]) break;
        const int i = warp + it * W;
        const Slot sl = slot_of(base + static_cast<unsigned>(ni + i), a.ring_slots);
        if (!wait_item(a, sh, sl, waited)) break;
        const float4* rows = reinterpret_cast<const float4*>(sh.ring + static_cast<size_t>(sl.index) * kItemBytes);
        float4 vv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int t = t0 + 4 * i + q;
            vv[q] = t == pos ? reinterpret_cast<const float4*>(vp)[lane]
                             : (t < n_keys ? rows[q * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f));
        }
        release_item(sh, sl);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float pr[G];
#pragma unroll
            for (int g = 0; g < G; ++g) pr[g] = __shfl_sync(0xffffffffu, scv[it][g], q * 8);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                acc[g].x = fmaf(pr[g], vv[q].x, acc[g].x);
                acc[g].y = fmaf(pr[g], vv[q].y, acc[g].y);
                acc[g].z = fmaf(pr[g], vv[q].z, acc[g].z);
                acc[g].w = fmaf(pr[g], vv[q].w, acc[g].w);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        reinterpret_cast<float4*>(vpart + (warp * G + g) * 128)[lane] = acc[g];
        if (lane == 0) {
            wml[(warp * G + g) * 2] = wm[g];
            wml[(warp * G + g) * 2 + 1] = wl[g];
        }
    }
    if (a.trace != nullptr && lane == 0 && waited > 0)
        atomicAdd(reinterpret_cast<unsigned long long*>(sh.misc + 4), static_cast<unsigned long long>(waited));
    mark(12);
    cbar();
    // this chunk's partial output: merge the warps' (m, l, o) in warp order. Thread
    // (w, g) turns warp w's max into its factor exp(m_w - M_g).
    const int hq0 = h * G;
    if (!failed(sh) && tid < W * G) {
        const int w = tid / G, g = tid % G;
        float M = -INFINITY;
#pragma unroll 4
        for (int v = 0; v < W; ++v) M = fmaxf(M, wml[(v * G + g) * 2]);
        const float mw = wml[(w * G + g) * 2];
        wf[w * G + g] = mw == -INFINITY ? 0.0f : expf(mw - M);
        if (w == 0) ml[2 * g] = M;
    }
    cbar();
    if (!failed(sh)) {
        for (int j = tid; j < G * 128; j += kConsumers) {
            const int g = j >> 7, d = j & 127;
            float o = 0.0f;
#pragma unroll 4
            for (int w = 0; w < W; ++w) o = fmaf(vpart[(w * G + g) * 128 + d], wf[w * G + g], o);
            a.attn_part[(static_cast<size_t>(hq0 + g) * a.max_chunks + c) * 128 + d] = o;
            if (d == 0) {
                float Lsum = 0.0f;
                for (int w = 0; w < W; ++w) Lsum = fmaf(wml[(w * G + g) * 2 + 1], wf[w * G + g], Lsum);
                float* dst = a.attn_ml + (static_cast<size_t>(hq0 + g) * a.max_chunks + c) * 2;
                dst[0] = ml[2 * g];
                dst[1] = Lsum;
            }
        }
    }
    // publish the chunk: barrier, then one fence + ticket (the consumers' stores above
    // are ordered before it); the last chunk of the head fences again before reading
    cbar();
    mark(7);
    unsigned* ticket = a.sync + a.L * kStackPhases + h;
    if (tid == 0) {
        int last = 0;
        if (!failed(sh)) {
            __threadfence();
            last = atomicAdd(ticket, 1u) == static_cast<unsigned>(sc.nch - 1);
            if (last) __threadfence();
        }
        sh.misc[2] = last;
    }
    cbar();
    mark(8);
    if (sh.misc[2]) {
        // the last chunk of this head combines all chunks (flash-decoding merge)
        for (int g = warp; g < G; g += W) {
            const float* pm = a.attn_ml + static_cast<size_t>(hq0 + g) * a.max_chunks * 2;
            float M = -INFINITY;
            for (int cc = lane; cc < sc.nch; cc += 32) M = fmaxf(M, __ldcg(pm + 2 * cc));
            M = warp_max(M);
            float S = 0.0f;
            for (int cc = lane; cc < sc.nch; cc += 32) {
                const float f = expf(__ldcg(pm + 2 * cc) - M);
                wc[g * a.max_chunks + cc] = f;
                S += __ldcg(pm + 2 * cc + 1) * f;
            }
            S = warp_sum(S);
            if (lane == 0) ml[2 * g + 1] = S;
        }
        cbar();
        for (int j = tid; j < G * 128; j += kConsumers) {
            const int g = j >> 7, d = j & 127;
            const float* pp = a.attn_part + static_cast<size_t>(hq0 + g) * a.max_chunks * 128 + d;
            float o = 0.0f;
            for (int cc = 0; cc < sc.nch; ++cc) o = fmaf(__ldcg(pp + static_cast<size_t>(cc) * 128), wc[g * a.max_chunks + cc], o);
            a.attn_out[static_cast<size_t>(hq0 + g) * 128 + d] = o / ml[2 * g + 1];
        }
        if (tid == 0) *ticket = 0u;
    }
    cbar();
    mark(9);
}

template <int G, bool kTp>
__device__ void consumer(const StackArgs& a, const Shared& sh, const Sched& sc, int pos, unsigned tag_base,
                         bool stall) {
    const int tid = threadIdx.x;
    unsigned seq = 0;
    for (int l = 0; l < a.L; ++l) {
        const StackLayer& Ly = a.layers[l];
        for (int p = 0; p < kStackPhases; ++p) {
            int first, count;
            sc.mine(a, l, p, &first, &count);
            if (count == 0) continue;
            if (tid == 0) stamp(a, l, p, 0);
            // input dependency: the phase before (layer 0's input comes from an earlier launch)
            if (l > 0 || p > 0) {
                const int lp = p == 0 ? l - 1 : l, pp = p == 0 ? kStackPhases - 1 : p - 1;
                const unsigned extra = stall && l == 0 && p == 2 ? 1u : 0u;  // failure injection
                wait_phase(a, sh, lp, pp, static_cast<unsigned>(min(sc.grid, sc.units(a, pp))) + extra);
            } else {
                cbar();
            }
            if (tid == 0) stamp(a, l, p, 1);
            if (p == 1) {
                for (int k = 0; k < count; ++k) {
                    const int u = first + k * sc.grid;
                    const int c = u / a.kv_heads, h = u % a.kv_heads;
                    attention_unit<G>(a, sh, sc, l, pos, c, h, seq, k == 0);
                    seq += static_cast<unsigned>(2 * sc.att_items(c));
                }
                if (tid == 0 && !failed(sh)) {
                    signal_phase(a, l, 1);
                    stamp(a, l, 1, 3);
                    unsigned long long* w = reinterpret_cast<unsigned long long*>(sh.misc + 4);
                    record(a, l, 1, 5, *w);
                    *w = 0;
                }
                continue;
            }
            const StackPhase& ph = a.ph[p];
            const bool own = ph.ipu == W;
            if (!failed(sh)) {
                const float* x = p == 0 ? a.hidden_buf : (p == 2 ? a.attn_out : (p == 3 ? a.attn_res : a.act));
                const float* nw = p == 0 ? Ly.attn_norm : (p == 3 ? Ly.ffn_norm : nullptr);
                // tensor parallel: attn_res = hidden + sum(o partials) (qwen.cpp:262) and
                // hidden = attn_res + sum(down partials) (qwen.cpp:291), formed here
                const unsigned long long* parts = nullptr;
                unsigned tag = 0;
                float* keep = nullptr;
                if (kTp && p == 3) {
                    x = a.hidden_buf;
                    parts = a.xo[a.rank];
                    tag = xtag(tag_base, l);
                    keep = a.attn_res;
                } else if (kTp && p == 0 && l > 0) {
                    x = a.attn_res;
                    parts = a.xdown[a.rank];
                    tag = xtag(tag_base, l - 1);
                    keep = a.hidden_buf;
                }
                stage_x(a, x, nw, ph, own, sh, parts, tag, keep, first, min(sc.grid, ph.units));
            }
            if (own)
                __syncwarp();
            else
                cbar();
            if (tid == 0) stamp(a, l, p, 2);
            gemv_phase<kTp>(a, sh, sc, l, p, first, count, seq, tag_base);
            seq += static_cast<unsigned>(count * ph.ipu);
        }
    }
    if (kTp) {
        // the final residual stream for the LM head: hidden = attn_res + sum(down partials)
        // of the last layer, group g by CTA g mod grid (warp w: g = blockIdx + w grid); the
        // local wait orders the attn_res write-back of the last gate/up staging
        wait_phase(a, sh, a.L - 1, 4, static_cast<unsigned>(min(sc.grid, sc.units(a, 4))));
        const int lane = tid & 31, warp = tid >> 5;
        const int g = static_cast<int>(blockIdx.x) + warp * sc.grid;
        if (!failed(sh) && g < (a.hidden >> 7)) {
            const int idx = g * 32 + lane;
            const float4 sm = word_sum4(a, sh, a.xdown[a.rank], a.hidden, 4 * idx, xtag(tag_base, a.L - 1));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(a.attn_res) + idx);
            reinterpret_cast<float4*>(a.hidden_buf)[idx] = make_float4(b.x + sm.x, b.y + sm.y, b.z + sm.z, b.w + sm.w);
        }
    }
}

template <int G, bool kTp>
__global__ void __launch_bounds__(kStackThreads, 1) stack_kernel(const StackArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const Shared sh = carve(a, smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.ring_slots; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        for (int i = 0; i < 8; ++i) sh.misc[i] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    pdl_wait();
    const int pos = a.state->pos;
    const bool bad = pos < 0 || pos >= a.capacity || state_failed(a.state);
    if (bad && blockIdx.x == 0 && threadIdx.x == 0 && !state_failed(a.state)) a.state->error = 1;
    __syncthreads();
    if (bad) {
        if (kTp && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(a.epoch, 1u);
        return;
    }
    const Sched sc = make_sched(a, pos);
    const bool stall = a.stall != nullptr && *reinterpret_cast<const volatile int*>(a.stall) != 0;
    // tensor parallel: this launch's exchange tags (see StackArgs)
    const unsigned ep = kTp ? *reinterpret_cast<const volatile unsigned*>(a.epoch) : 0u;
    if (warp == W) {
        producer(a, sh, sc, pos);
    } else if (warp == W + 1) {
        prefetcher(a, sh, sc, pos);
    } else {
        consumer<G, kTp>(a, sh, sc, pos, (ep + 1u) * static_cast<unsigned>(a.L + 1), stall);
        // every CTA read the epoch at its start, and CTA 0 gets here only after all ranks
        // finished the last layer
        if (kTp && blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(a.epoch) = ep + 1u;
    }
    pdl_launch_dependents();
}

__global__ void stack_pack_kernel(const uint8_t* __restrict__ qw, const float* __restrict__ scales,
                                  const uint8_t* __restrict__ zeros, int N, int K, int mode, uint8_t* __restrict__ out) {
    const int ipr = K / kItemK, groups = K / 128;
    const long long total = static_cast<long long>(N / kItemRows) * ipr * (kItemBytes / 16);
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long item = i / (kItemBytes / 16);
        const int ch = static_cast<int>(i % (kItemBytes / 16));
        const int tile = static_cast<int>(item / ipr), it = static_cast<int>(item % ipr);
        auto src_row = [&](int r) -> size_t {
            if (mode == kPackGateUp)
                return r < 8 ? static_cast<size_t>(tile) * 8 + r : static_cast<size_t>(N / 2) + static_cast<size_t>(tile) * 8 + (r - 8);
            return static_cast<size_t>(tile) * 16 + r;
        };
        uint8_t* dst = out + static_cast<size_t>(item) * kItemBytes + static_cast<size_t>(ch) * 16;
        if (ch < 128) {
            // chunk (h, gi, lane = 4*gq + c): row 8h + gq, group 2*it + gi, bytes 16c..16c+15
            const int h = ch >> 6, gi = (ch >> 5) & 1, ln = ch & 31, gq = ln >> 2, c = ln & 3;
            const size_t row = src_row(8 * h + gq);
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(
                qw + row * static_cast<size_t>(K / 2) + static_cast<size_t>(2 * it + gi) * 64 + c * 16);
        } else if (ch < 136) {
            float v[4];
            for (int e = 0; e < 4; ++e) {
                const int f = (ch - 128) * 4 + e;
                v[e] = scales[src_row(f >> 1) * groups + 2 * it + (f & 1)];
            }
            *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
            uint32_t w[4];
            for (int q = 0; q < 4; ++q) {
                uint32_t word = 0;
                for (int e = 0; e < 4; ++e) {
                    const int b = (ch - 136) * 16 + q * 4 + e;
                    word |= static_cast<uint32_t>(zeros[src_row(b >> 1) * groups + 2 * it + (b & 1)]) << (8 * e);
                }
                w[q] = word;
            }
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

int align_up(int v, int a) { return (v + a - 1) / a * a; }

}  // namespace

size_t stack_items_bytes(int N, int K) {
    return static_cast<size_t>(N / kItemRows) * (K / kItemK) * kItemBytes;
}

cudaError_t stack_pack_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K, int mode,
                              uint8_t* out, cudaStream_t s) {
    if (N <= 0 || K <= 0 || N % kItemRows || K % kItemK)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(qw) | reinterpret_cast<uintptr_t>(out)) % 16) return cudaErrorInvalidValue;
    const long long total = static_cast<long long>(N / kItemRows) * (K / kItemK) * (kItemBytes / 16);
    const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 1 << 16));
    stack_pack_kernel<<<grid, 256, 0, s>>>(qw, scales, zeros, N, K, mode, out);
    return cudaGetLastError();
}

size_t stack_sync_words(const StackArgs& a) {
    int tiles = 0;
    for (int p = 0; p < kStackPhases; ++p)
        if (p != 1) tiles = std::max(tiles, a.ph[p].tiles);
    return static_cast<size_t>(a.L) * kStackPhases + a.kv_heads + tiles;
}

size_t stack_exchange_bytes(int tp, int hidden, int L) {
    (void)L;
    return 2 * static_cast<size_t>(tp) * hidden * 8 + 16;
}

void stack_bind_exchange(StackArgs* a, int tp, int rank, void* const* base) {
    a->tp = tp;
    a->rank = rank;
    const size_t part = static_cast<size_t>(tp) * a->hidden * 8;
    for (int r = 0; r < kStackMaxTp; ++r) {
        uint8_t* b = r < tp ? static_cast<uint8_t*>(base[r]) : nullptr;
        a->xo[r] = b ? reinterpret_cast<unsigned long long*>(b) : nullptr;
        a->xdown[r] = b ? reinterpret_cast<unsigned long long*>(b + part) : nullptr;
    }
    a->epoch = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(base[rank]) + 2 * part);
}

size_t stack_kpart_floats(const StackArgs& a) {
    size_t m = 0;
    for (int p = 0; p < kStackPhases; ++p)
        if (p != 1 && a.ph[p].kparts > 1) m = std::max(m, static_cast<size_t>(a.ph[p].kparts) * a.ph[p].n);
    return m;
}

bool stack_plan(StackArgs* a, int grid) {
    const int G = a->kv_heads > 0 ? a->q_heads / a->kv_heads : 0;
    if (a->L <= 0 || a->kv_heads <= 0 || a->q_heads % a->kv_heads) return false;
    if (G != 1 && G != 2 && G != 4 && G != 5 && G != 8) return false;  // instantiated group sizes
    if (a->q_dim != a->q_heads * 128 || a->kv_dim != a->kv_heads * 128) return false;
    if (a->inter % 8 || grid <= 0) return false;
    if (a->hidden > W * kStageRegs * 128) return false;  // the RMSNorm'ed input is staged in one batch
    const int nk[kStackPhases][2] = {{a->q_dim + 2 * a->kv_dim, a->hidden}, {0, 0}, {a->hidden, a->q_dim},
                                     {2 * a->inter, a->hidden}, {a->hidden, a->inter}};
    int max_k = 0, max_units = 0, max_part = 0;
    for (int p = 0; p < kStackPhases; ++p) {
        StackPhase& ph = a->ph[p];
        ph = StackPhase{};
        if (p == 1) continue;
        ph.n = nk[p][0];
        ph.k = nk[p][1];
        if (ph.n % kItemRows || ph.k % kItemK || ph.k <= 0) return false;
        ph.tiles = ph.n / kItemRows;
        ph.ipr = ph.k / kItemK;
        // K split only when a whole row tile exceeds 64 items (split-K partials cost a
        // ticket round trip; rotation already balances the bytes per CTA over a layer)
        ph.kparts = 1;
        while (ph.ipr / ph.kparts > 64 || ph.ipr % ph.kparts) ++ph.kparts;
        ph.ipu = ph.ipr / ph.kparts;
        ph.units = ph.tiles * ph.kparts;
        max_k = std::max(max_k, ph.k);
        max_units = std::max(max_units, (ph.units + grid - 1) / grid);
        max_part = std::max(max_part, ((ph.units + grid - 1) / grid) * ph.ipu * 16);
    }
    a->grid = grid;
    a->max_units = max_units;
    a->part_floats = max_part;  // one 16-row slot per item of every unit of a phase
    a->max_chunks = (a->capacity + kStackChunk - 1) / kStackChunk;
    const int digits = (max_k / 128) * (512 + 8);
    const int att = (G * 128 + 256 + 3 * W * kStackMaxGroup + 2 * kStackMaxGroup + W * G * 128 + G * a->max_chunks) * 4;
    const int xbytes = align_up(std::max(digits, att), 128);
    const int part = align_up(a->part_floats * 4, 16);
    const int ucnt = align_up(max_units * 4, 16);
    const int xv = align_up(max_units * 16 * 4, 16);
    // tensor parallel: o and down leave whole row sums (no split-K ticket) for the exchange
    if (a->tp > 1 && (a->ph[2].kparts != 1 || a->ph[4].kparts != 1)) return false;
    const int misc = 32 * 4 + 32;
    const int fixed = xbytes + part + ucnt + xv + misc + 256;
    const int budget = 227 * 1024;
    int slots = (budget - fixed) / (kItemBytes + 16);
    slots = std::min(slots, 128);
    if (slots < 32) return false;  // the producer issues up to 32 items per step
    a->ring_slots = slots;
    int off = align_up(slots * kItemBytes, 128);
    a->off_bar = off;
    off = align_up(off + slots * 16, 128);
    a->off_x = off;
    off += xbytes;
    a->off_part = off;
    off += part;
    a->off_ucnt = off;
    off += ucnt;
    a->off_xv = off;
    off += xv;
    a->off_misc = off;
    off += misc;
    a->smem_bytes = align_up(off, 128);
    return a->smem_bytes <= budget;
}

cudaError_t stack_launch(const StackArgs& a, cudaStream_t s, bool cooperative) {
    void (*kern)(const StackArgs) = nullptr;
    switch (a.q_heads / a.kv_heads) {
    case 1: kern = a.tp > 1 ? stack_kernel<1, true> : stack_kernel<1, false>; break;
    case 2: kern = a.tp > 1 ? stack_kernel<2, true> : stack_kernel<2, false>; break;
    case 4: kern = a.tp > 1 ? stack_kernel<4, true> : stack_kernel<4, false>; break;
    case 5: kern = a.tp > 1 ? stack_kernel<5, true> : stack_kernel<5, false>; break;
    case 8: kern = a.tp > 1 ? stack_kernel<8, true> : stack_kernel<8, false>; break;
    default: return cudaErrorInvalidValue;
    }
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, a.smem_bytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.grid));
    cfg.blockDim = dim3(kStackThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(a.smem_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace fb
