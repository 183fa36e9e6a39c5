// Persistent decode kernel for the whole Qwen3 layer stack: the per-layer sequence of
// Fire's Qwen3Model::forward (src/model/qwen.cpp:190-292) as one launch per GPU, on one GPU
// or on each rank of a tensor-parallel group (o/down reductions exchanged inside the
// kernel through NVLink peer memory, see StackArgs).
//
// Every INT4 projection is stored as "items" of 16 rows x 256 K (2208 bytes) in the
// order the kernel reads them. One CTA runs per SM: a producer warp streams every item
// the CTA will consume in this step (all layers, all phases, plus the attention K/V
// rows) into a shared-memory ring with TMA bulk copies (a second warp walks the same
// sequence further ahead with L2 bulk prefetches), while 16 consumer warps run the
// phases qkv -> attention -> o -> gate/up -> down of each layer. A phase waits on a
// device-wide counter of the CTAs that finished the phase it depends on; the weight
// stream does not wait, so HBM stays busy across phase boundaries.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode_state.h"

namespace fb {

constexpr int kItemRows = 16;
constexpr int kItemK = 256;
// weights 16 rows x 2 groups x 64 bytes (MMA fragment order) | scales f32 [16][2] | zeros u8 [16][2]
constexpr int kItemBytes = 2208;
constexpr int kItemScaleOff = 2048;
constexpr int kItemZeroOff = 2176;
constexpr int kStackPhases = 5;  // 0 qkv, 1 attention, 2 o, 3 gate/up, 4 down
constexpr int kStackConsumerWarps = 16;
// consumer warps, the ring producer warp and the L2 prefetch warp
constexpr int kStackThreads = (kStackConsumerWarps + 2) * 32;
constexpr int kStackPrefetchAhead = 150;  // items the L2 prefetcher runs ahead of the ring
constexpr int kStackChunk = 128;  // keys per attention unit
constexpr int kStackMaxGroup = 8;  // q heads per KV head
constexpr int kStackErrTimeout = 3;  // DecodeState::error when a bounded wait gave up
constexpr int kStackTraceSlots = 13;
constexpr int kStackMaxTp = 8;

enum StackPackMode : int { kPackRows = 0, kPackGateUp = 1 };

// Bytes of the item layout of an [N, K] matrix (N % 16 == 0, K % 256 == 0).
size_t stack_items_bytes(int N, int K);
// Repack an INT4 group-128 matrix (qweight u8 [N, K/2], scales f32 [N, K/128],
// zero points u8 [N, K/128]) into items. kPackGateUp: source rows [0, N/2) are gate
// rows and [N/2, N) the matching up rows; item row tile t then holds gate rows
// 8t..8t+7 followed by up rows 8t..8t+7.
cudaError_t stack_pack_launch(const uint8_t* qw, const float* scales, const uint8_t* zeros, int N, int K,
                              int mode, uint8_t* out, cudaStream_t s);

struct StackLayer {
    const float* attn_norm;
    const float* ffn_norm;
    const float* q_norm;
    const float* k_norm;
    const uint8_t* qkv;   // [q | k | v] rows x hidden
    const uint8_t* o;     // hidden x q_dim
    const uint8_t* gu;    // kPackGateUp, 2*inter x hidden
    const uint8_t* down;  // hidden x inter
};

struct StackPhase {  // GEMV phase geometry, identical in every layer
    int n, k;
    int tiles;   // n / 16
    int ipr;     // items per row tile (k / 256)
    int kparts;  // K splits (their partial sums are added in a fixed order)
    int ipu;     // items per unit (ipr / kparts)
    int units;   // tiles * kparts
};

struct StackArgs {
    const StackLayer* layers;  // device array [L]
    int L;
    int hidden, q_dim, kv_dim, inter;
    int q_heads, kv_heads;
    float eps, scale;
    DecodeState* state;
    float* hidden_buf;  // residual stream in / out
    float* attn_res;    // hidden + o projection
    float* qkv;
    float* attn_out;
    float* act;
    float* kcache;  // [L][capacity][kv_dim]
    float* vcache;
    int capacity;
    int max_chunks;  // ceil(capacity / kStackChunk)
    const float* rope_sin;  // [capacity][64]
    const float* rope_cos;
    float* attn_part;  // [q_heads][max_chunks][128]
    float* attn_ml;    // [q_heads][max_chunks][2]
    float* kpart;      // split-K partial sums [kparts][n]
    unsigned* sync;    // phase counters, attention and tile tickets: zero before each launch
    // Tensor parallel (tp > 1; Fire's new src/model tensor-parallel layer). o and down are
    // row-parallel: each rank leaves partial row sums that every rank adds up, in rank
    // order, while staging the next phase's input. Rank r owns an exchange block (layout
    // in stack_exchange_bytes) mapped into every rank: xo[r] / xdown[r] are its o / down
    // partials [tp][hidden] as 64-bit words (tag << 32 | float bits). A CTA stores its rows'
    // partials into every rank's block with plain relaxed stores after its local phase
    // signal; a reader polls each word until the tag is this launch's tag for the layer,
    // (epoch + 1) * (L + 1) + layer + 1, with epoch = this rank's completed launches.
    int tp, rank;
    unsigned long long* xo[kStackMaxTp];
    unsigned long long* xdown[kStackMaxTp];
    unsigned* epoch;
    // optional timeline [grid][L][kStackPhases][kStackTraceSlots] of %globaltimer stamps:
    // 0 phase entered, 1 input dependency met, 2 input staged, 3 the CTA's last unit
    // done, 4 the producer issued the phase's last item (0 where the CTA had no units);
    // then SM cycles: 5 consumer warps waiting for ring items (summed over warps),
    // 6 the producer waiting for free slots; attention only (first unit of the CTA),
    // stamps: 2 q/k prepared, 7 chunk partial written, 8 ticket taken, 9 merge done,
    // and warp 0's own progress: 10 scores done, 11 local softmax done, 12 P.V done;
    // GEMV phases: 7 warp 0's last item done (before the phase's finish step)
    unsigned long long* trace;
    // failure injection for tests (nullptr in normal use): while *stall != 0, layer 0's o
    // phase waits for one CTA more than the grid has, so that bounded wait runs out and
    // the launch fails with kStackErrTimeout (a flag that nothing sets)
    const int* stall;
    StackPhase ph[kStackPhases];  // index 1 (attention) unused
    // shared-memory plan (filled by stack_plan)
    int grid;
    int ring_slots;
    int max_units;    // GEMV units one CTA owns in one phase, at most
    int part_floats;  // floats of the per-item partial sums of one phase (max over phases)
    int off_bar, off_x, off_part, off_ucnt, off_xv, off_misc;
    int smem_bytes;
};

size_t stack_sync_words(const StackArgs& a);
// Exchange block of one rank: o partials [tp][hidden] and down partials [tp][hidden] as
// tagged 64-bit words, then the epoch word.
size_t stack_exchange_bytes(int tp, int hidden, int L);
// Point a's exchange fields at the blocks `base[r]` (rank r's block as mapped here).
void stack_bind_exchange(StackArgs* a, int tp, int rank, void* const* base);
size_t stack_kpart_floats(const StackArgs& a);
// Fill the phase geometry and the shared-memory plan for `grid` CTAs; false when the
// shapes are outside what the kernel handles (the per-op kernels then run instead).
bool stack_plan(StackArgs* a, int grid);
cudaError_t stack_launch(const StackArgs& a, cudaStream_t s, bool cooperative);

}  // namespace fb
