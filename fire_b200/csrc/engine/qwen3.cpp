#include "engine/qwen3.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <chrono>
#include <thread>
#include <unordered_map>

#include "device_info.h"
#include "fire_b200.h"
#include "kernels/dense_gemv.h"
#include "kernels/ops.h"
#include "kernels/prefill_ops.h"
#include "kernels/w4_gemv.h"
#include "kernels/w4_prefill.h"

namespace fb {

namespace {

#define FB_CK(expr)                                                 \
    do {                                                            \
        const cudaError_t e_ = (expr);                              \
        if (e_ != cudaSuccess) return static_cast<int>(e_);         \
    } while (0)
#define FB_RC(expr)                     \
    do {                                \
        const int r_ = (expr);          \
        if (r_ != 0) return r_;         \
    } while (0)

size_t esize(int dt) { return dt == kSrcF32 ? 4 : (dt == kSrcBF16 ? 2 : 1); }
size_t pad256(size_t b) { return (b + 255) / 256 * 256; }

class Sources {
  public:
    explicit Sources(const std::vector<TensorSrc>& v) {
        for (const auto& t : v) m_[t.name] = &t;
    }
    const TensorSrc* get(const std::string& n) const {
        auto it = m_.find(n);
        return it == m_.end() ? nullptr : it->second;
    }
    bool has(const std::string& n) const { return m_.count(n) != 0; }

  private:
    std::unordered_map<std::string, const TensorSrc*> m_;
};

bool is(const TensorSrc* t, int dt, std::vector<int64_t> shape) {
    return t != nullptr && t->data != nullptr && t->dtype == dt && t->shape == shape;
}

int copy2d(void* dst, size_t dpitch, const TensorSrc* src, size_t src_off, size_t spitch, size_t width,
           size_t height, cudaStream_t s) {
    const char* p = static_cast<const char*>(src->data) + src_off;
    const cudaMemcpyKind kind = src->on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (height == 0 || width == 0) return 0;
    if (dpitch == width && spitch == width)
        return static_cast<int>(cudaMemcpyAsync(dst, p, width * height, kind, s));
    return static_cast<int>(cudaMemcpy2DAsync(dst, dpitch, p, spitch, width, height, kind, s));
}

}  // namespace

Qwen3Engine::~Qwen3Engine() {
    if (graph_fwd_) cudaGraphExecDestroy(graph_fwd_);
    if (graph_step_) cudaGraphExecDestroy(graph_step_);
    if (host_state_) cudaFreeHost(host_state_);
    if (host_seen_) cudaFreeHost(host_seen_);
    if (steps_done_) cudaEventDestroy(steps_done_);
    for (int r = 0; r < kStackMaxTp; ++r)
        if (xchg_peer_[r] && xchg_peer_[r] != xchg_) cudaIpcCloseMemHandle(xchg_peer_[r]);
    if (xchg_) cudaFree(xchg_);
    if (comm_ && nccl().ok) {
        if (aborted_)
            nccl().CommAbort(comm_);
        else
            nccl().CommDestroy(comm_);
    }
}

// Tensor parallel with the layer stack: allocate this rank's exchange block, share its
// IPC handle with every rank over NCCL (all-gather of the 64-byte handles) and map the
// peers' blocks. The kernel stores partial sums and bumps counters in those mappings
// (NVLink peer memory).
int Qwen3Engine::setup_exchange(std::string* err) {
    auto fail = [&](int code, const std::string& m) {
        if (err) *err = m;
        return code;
    };
    const size_t bytes = stack_exchange_bytes(tp_, d_.hidden, d_.layers);
    FB_CK(cudaMalloc(&xchg_, bytes));
    FB_CK(cudaMemset(xchg_, 0, bytes));
    cudaIpcMemHandle_t mine;
    FB_CK(cudaIpcGetMemHandle(&mine, xchg_));
    constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
    void* dh = nullptr;
    FB_CK(cudaMalloc(&dh, kH * tp_));
    std::vector<cudaIpcMemHandle_t> all(tp_);
    cudaStream_t s;
    int rc = static_cast<int>(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    if (!rc) rc = static_cast<int>(cudaMemcpyAsync(static_cast<char*>(dh) + kH * rank_, &mine, kH, cudaMemcpyHostToDevice, s));
    if (!rc && nccl().AllGather(static_cast<char*>(dh) + kH * rank_, dh, kH, kNcclUint8, comm_, s) != 0)
        rc = FIRE_B200_ERR_STATE;
    if (!rc) rc = static_cast<int>(cudaMemcpyAsync(all.data(), dh, kH * tp_, cudaMemcpyDeviceToHost, s));
    if (!rc) rc = static_cast<int>(cudaStreamSynchronize(s));
    cudaStreamDestroy(s);
    cudaFree(dh);
    if (rc) return fail(rc, "exchange handle all-gather failed");
    for (int r = 0; r < tp_; ++r) {
        if (r == rank_) {
            xchg_peer_[r] = xchg_;
            continue;
        }
        const cudaError_t e = cudaIpcOpenMemHandle(&xchg_peer_[r], all[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(static_cast<int>(e), std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    }
    return 0;
}

int Qwen3Engine::create(const Qwen3Dims& d, const std::vector<TensorSrc>& tensors, const EngineOptions& opt,
                        std::unique_ptr<Qwen3Engine>* out, std::string* err) {
    auto fail = [&](int code, const std::string& m) {
        if (err) *err = m;
        return code;
    };
    if (d.vocab <= 0 || d.hidden <= 0 || d.inter <= 0 || d.layers <= 0 || d.q_heads <= 0 || d.kv_heads <= 0 ||
        d.q_heads % d.kv_heads || d.max_seq <= 0 || !(d.eps > 0.f) || !(d.theta > 0.f))
        return fail(FIRE_B200_ERR_INVALID, "invalid Qwen3 profile");
    if (d.head_dim != 128) return fail(FIRE_B200_ERR_UNSUPPORTED, "the decode engine needs head_dim 128");
    const int t = opt.tp_size;
    if (t < 1 || opt.tp_rank < 0 || opt.tp_rank >= t) return fail(FIRE_B200_ERR_INVALID, "bad tensor-parallel rank");
    if (d.q_heads % t || d.kv_heads % t || d.inter % t || d.vocab % t)
        return fail(FIRE_B200_ERR_UNSUPPORTED, "heads, FFN width and vocab must divide by the TP size");
    if (d.hidden % 128 || (d.inter / t) % 128 || d.hidden > 53248 || d.inter / t > 53248)
        return fail(FIRE_B200_ERR_UNSUPPORTED, "hidden and FFN shard must be multiples of the 128 group");
    if (t > 1 && (opt.nccl_id == nullptr || !nccl().ok))
        return fail(FIRE_B200_ERR_UNSUPPORTED, "tensor parallel needs NCCL: " + nccl().error);

    std::unique_ptr<Qwen3Engine> e(new Qwen3Engine());
    e->d_ = d;
    e->opt_ = opt;
    e->tp_ = t;
    e->rank_ = opt.tp_rank;
    FB_CK(cudaGetDevice(&e->device_));
    FB_RC(device_sms(&e->sms_));
    e->hq_ = d.q_heads / t;
    e->hkv_ = d.kv_heads / t;
    e->q_ = e->hq_ * 128;
    e->kv_ = e->hkv_ * 128;
    e->f_ = d.inter / t;
    e->v_ = d.vocab / t;
    e->v_off_ = e->rank_ * e->v_;
    if (t > 1) {
        const int nr = nccl_comm_init_rank(&e->comm_, t, opt.nccl_id, e->rank_);
        if (nr != 0) return fail(FIRE_B200_ERR_STATE, std::string("ncclCommInitRank: ") + nccl().GetErrorString(nr));
    }
    // the persistent layer-stack kernel serves the step when the shapes fit, also under
    // tensor parallelism up to kStackMaxTp ranks (FIRE_B200_LAYER_STACK=0 selects the per-op
    // kernels; FIRE_B200_TP_STACK=0 only under tensor parallelism). Every rank reaches the
    // same decision: it depends only on the shapes and the environment given to all ranks.
    {
        const char* env = std::getenv("FIRE_B200_LAYER_STACK");
        const char* tp_env = std::getenv("FIRE_B200_TP_STACK");
        const bool tp_ok = t == 1 || (t <= kStackMaxTp && (tp_env == nullptr || std::strcmp(tp_env, "0") != 0));
        if ((env == nullptr || std::strcmp(env, "0") != 0) && tp_ok) {
            StackArgs probe = e->stack_template(d.max_seq);
            e->stack_ = stack_plan(&probe, e->sms_);
            const char* tr = std::getenv("FIRE_B200_STACK_TRACE");
            e->stack_trace_on_ = e->stack_ && tr != nullptr && std::strcmp(tr, "1") == 0;
            // failure injection for tests: the first step after prepare (and every step
            // until reset) fails in a bounded wait of the layer-stack kernel
            const char* st = std::getenv("FIRE_B200_FAULT_STALL");
            e->stall_on_ = e->stack_ && st != nullptr && std::strcmp(st, "1") == 0;
        }
        if (e->stack_ && t > 1) {
            const int xr = e->setup_exchange(err);
            if (xr != 0) return xr;
        }
    }
    e->weight_arena_.reset(new DeviceArena(e->device_));
    e->runtime_arena_.reset(new DeviceArena(e->device_));
    const int rc = e->import_weights(tensors, err);
    if (rc != 0) return rc;
    *out = std::move(e);
    return 0;
}

int Qwen3Engine::import_weights(const std::vector<TensorSrc>& tensors, std::string* err) {
    auto fail = [&](int code, const std::string& m) {
        if (err) *err = m;
        return code;
    };
    const Sources S(tensors);
    const int H = d_.hidden, F = d_.inter, Q = d_.q_heads * 128, KV = d_.kv_heads * 128, V = d_.vocab;
    const int L = d_.layers;

    // --- validate (Qwen3Loader::load_weights rules, src/model/qwen_loader.cpp:123-223)
    const TensorSrc* emb = S.get("tok_embeddings.weight");
    if (!(is(emb, kSrcF32, {V, H}) || is(emb, kSrcBF16, {V, H})))
        return fail(FIRE_B200_ERR_INVALID, "tok_embeddings.weight must be FP32 or BF16 [vocab, hidden]");
    auto w4_ok = [&](const std::string& base, int n, int k) {
        return is(S.get(base + ".qweight"), kSrcU8, {n, k / 2}) && is(S.get(base + ".scales"), kSrcF32, {n, k / 128}) &&
               is(S.get(base + ".zero_points"), kSrcU8, {n, k / 128});
    };
    for (int l = 0; l < L; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        if (!is(S.get(p + "attention_norm.weight"), kSrcF32, {H}) || !is(S.get(p + "ffn_norm.weight"), kSrcF32, {H}) ||
            !is(S.get(p + "attention.q_norm.weight"), kSrcF32, {128}) ||
            !is(S.get(p + "attention.k_norm.weight"), kSrcF32, {128}))
            return fail(FIRE_B200_ERR_INVALID, "bad norm weights in layer " + std::to_string(l));
        const std::pair<std::string, std::pair<int, int>> mats[] = {
            {"attention.wq", {Q, H}}, {"attention.wk", {KV, H}}, {"attention.wv", {KV, H}}, {"attention.wo", {H, Q}},
            {"feed_forward.w1", {F, H}}, {"feed_forward.w2", {H, F}}, {"feed_forward.w3", {F, H}}};
        for (const auto& m : mats) {
            if (S.has(p + m.first + ".weight"))
                return fail(FIRE_B200_ERR_UNSUPPORTED,
                            "plain FP32 projections are not on the INT4 decode path: " + p + m.first);
            if (!w4_ok(p + m.first, m.second.first, m.second.second))
                return fail(FIRE_B200_ERR_INVALID, "bad INT4 group-128 triplet: " + p + m.first);
        }
    }
    if (!is(S.get("norm.weight"), kSrcF32, {H})) return fail(FIRE_B200_ERR_INVALID, "bad norm.weight");
    const TensorSrc* head = S.get("output.weight");
    if (head != nullptr) {
        if (!(is(head, kSrcF32, {V, H}) || is(head, kSrcBF16, {V, H})))
            return fail(FIRE_B200_ERR_INVALID, "output.weight must be FP32 or BF16 [vocab, hidden]");
        head_kind_ = head->dtype == kSrcBF16 ? 1 : 0;
    } else if (w4_ok("output", V, H)) {
        head_kind_ = 2;
    } else {
        return fail(FIRE_B200_ERR_INVALID, "missing LM head (output.weight or output.qweight triplet)");
    }

    // --- sizes and one reservation
    auto w4_bytes = [](int n, int k) {
        return pad256(size_t(n) * k / 2) + pad256(size_t(n) * (k / 128) * 4) + pad256(size_t(n) * (k / 128));
    };
    size_t total = pad256(size_t(V) * H * esize(emb->dtype)) + pad256(size_t(H) * 4);
    auto mat_bytes = [&](int n, int k) { return stack_ ? pad256(stack_items_bytes(n, k)) : w4_bytes(n, k); };
    const size_t per_layer = mat_bytes(q_ + 2 * kv_, H) + mat_bytes(H, q_) + mat_bytes(2 * f_, H) + mat_bytes(H, f_) +
                             2 * pad256(size_t(H) * 4) + 2 * pad256(512);
    total += per_layer * L;
    if (stack_) total += pad256(size_t(L) * sizeof(StackLayer));
    total += head_kind_ == 2 ? w4_bytes(v_, H) : pad256(size_t(v_) * H * (head_kind_ == 1 ? 2 : 4));
    FB_RC(weight_arena_->reserve(total + 4096));
    weight_bytes_ = total;

    // Device-resident sources may still be in the making on the caller's streams (e.g. a
    // framework's kernels that filled them, queued on its own stream). The copies below run
    // on a private non-blocking stream, which is not ordered after any of those, so wait for
    // the device first.
    bool any_device = false;
    for (const auto& t : tensors) any_device = any_device || t.on_device;
    if (any_device) FB_CK(cudaDeviceSynchronize());
    cudaStream_t s;
    FB_CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    auto alloc = [&](size_t b) { return weight_arena_->alloc(b); };
    int rc = 0;
    auto whole = [&](const TensorSrc* src, size_t bytes) -> void* {
        void* p = alloc(bytes);
        if (!p) { rc = FIRE_B200_ERR_NOMEM; return nullptr; }
        if (!rc) rc = copy2d(p, bytes, src, 0, bytes, bytes, 1, s);
        return p;
    };
    auto w4_alloc = [&](W4Mat& m, int n, int k) {
        m.n = n;
        m.k = k;
        m.qw = static_cast<uint8_t*>(alloc(size_t(n) * k / 2));
        m.s = static_cast<float*>(alloc(size_t(n) * (k / 128) * 4));
        m.z = static_cast<uint8_t*>(alloc(size_t(n) * (k / 128)));
        if (!m.qw || !m.s || !m.z) rc = FIRE_B200_ERR_NOMEM;
    };
    // Copy rows of a global [N, K] INT4 matrix (qweight/scales/zero_points), columns
    // [c0, c0+kk) of K (group aligned), into `m`: source rows r0 + b*block + r go to
    // destination rows dst_row + b*dst_stride + r, for r < block and b < rows/block.
    // block == dst_stride == 1 is a plain row copy; block 2 / stride 4 interleaves
    // gate and up rows per GEMV tile.
    auto w4_copy = [&](W4Mat& m, const std::string& base, int K, int r0, int rows, int c0, int kk, int dst_row,
                       int block, int dst_stride) {
        const TensorSrc* q = S.get(base + ".qweight");
        const TensorSrc* sc = S.get(base + ".scales");
        const TensorSrc* z = S.get(base + ".zero_points");
        const size_t qrow = size_t(K) / 2, grow = size_t(K) / 128;
        const size_t dq = size_t(m.k) / 2, dg = size_t(m.k) / 128;
        const size_t wq = size_t(kk) / 2, wg = size_t(kk) / 128;
        const int nblocks = rows / block;
        for (int r = 0; r < block && !rc; ++r) {
            const size_t sr = size_t(r0) + r, dr = size_t(dst_row) + r;
            rc = copy2d(m.qw + dr * dq, dq * dst_stride, q, sr * qrow + c0 / 2, qrow * block, wq, nblocks, s);
            if (!rc)
                rc = copy2d(reinterpret_cast<char*>(m.s) + dr * dg * 4, dg * 4 * dst_stride, sc,
                            (sr * grow + c0 / 128) * 4, grow * 4 * block, wg * 4, nblocks, s);
            if (!rc)
                rc = copy2d(m.z + dr * dg, dg * dst_stride, z, sr * grow + c0 / 128, grow * block, wg, nblocks, s);
        }
    };

    // layer-stack layout: each matrix is uploaded in the .fire layout to a scratch
    // matrix, then repacked into items in the arena
    W4Mat tmp{};
    if (stack_) {
        const size_t elems = std::max({size_t(q_ + 2 * kv_) * H, size_t(H) * q_, size_t(2 * f_) * H, size_t(H) * f_});
        void *tq = nullptr, *ts = nullptr, *tz = nullptr;
        if (cudaMalloc(&tq, elems / 2) != cudaSuccess || cudaMalloc(&ts, elems / 128 * 4) != cudaSuccess ||
            cudaMalloc(&tz, elems / 128) != cudaSuccess) {
            cudaFree(tq);
            cudaFree(ts);
            cudaFree(tz);
            cudaStreamDestroy(s);
            return fail(FIRE_B200_ERR_NOMEM, "no room for the repack scratch matrix");
        }
        tmp.qw = static_cast<uint8_t*>(tq);
        tmp.s = static_cast<float*>(ts);
        tmp.z = static_cast<uint8_t*>(tz);
    }
    auto pack = [&](uint8_t** out, int n, int k, int mode) {
        *out = static_cast<uint8_t*>(alloc(stack_items_bytes(n, k)));
        if (!*out) rc = FIRE_B200_ERR_NOMEM;
        if (!rc) rc = static_cast<int>(stack_pack_launch(tmp.qw, tmp.s, tmp.z, n, k, mode, *out, s));
    };
    auto as_tmp = [&](int n, int k) -> W4Mat& {
        tmp.n = n;
        tmp.k = k;
        return tmp;
    };

    emb_bf16_ = emb->dtype == kSrcBF16;
    embedding_ = whole(emb, size_t(V) * H * esize(emb->dtype));
    final_norm_ = static_cast<float*>(whole(S.get("norm.weight"), size_t(H) * 4));
    layers_.resize(L);
    const int half = kW4TileRows / 2;
    for (int l = 0; l < L && !rc; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        Layer& y = layers_[l];
        y.attn_norm = static_cast<float*>(whole(S.get(p + "attention_norm.weight"), size_t(H) * 4));
        y.ffn_norm = static_cast<float*>(whole(S.get(p + "ffn_norm.weight"), size_t(H) * 4));
        y.q_norm = static_cast<float*>(whole(S.get(p + "attention.q_norm.weight"), 512));
        y.k_norm = static_cast<float*>(whole(S.get(p + "attention.k_norm.weight"), 512));
        if (stack_) {
            y.qkv.n = q_ + 2 * kv_, y.qkv.k = H;
            y.o.n = H, y.o.k = q_;
            y.gu.n = 2 * f_, y.gu.k = H;
            y.down.n = H, y.down.k = f_;
            W4Mat& a = as_tmp(q_ + 2 * kv_, H);
            w4_copy(a, p + "attention.wq", H, rank_ * q_, q_, 0, H, 0, 1, 1);
            if (!rc) w4_copy(a, p + "attention.wk", H, rank_ * kv_, kv_, 0, H, q_, 1, 1);
            if (!rc) w4_copy(a, p + "attention.wv", H, rank_ * kv_, kv_, 0, H, q_ + kv_, 1, 1);
            if (!rc) pack(&y.qkv_items, q_ + 2 * kv_, H, kPackRows);
            if (!rc) w4_copy(as_tmp(H, q_), p + "attention.wo", Q, 0, H, rank_ * q_, q_, 0, 1, 1);
            if (!rc) pack(&y.o_items, H, q_, kPackRows);
            // gate rows then up rows; the repack interleaves them per item row tile
            if (!rc) w4_copy(as_tmp(2 * f_, H), p + "feed_forward.w1", H, rank_ * f_, f_, 0, H, 0, 1, 1);
            if (!rc) w4_copy(tmp, p + "feed_forward.w3", H, rank_ * f_, f_, 0, H, f_, 1, 1);
            if (!rc) pack(&y.gu_items, 2 * f_, H, kPackGateUp);
            if (!rc) w4_copy(as_tmp(H, f_), p + "feed_forward.w2", F, 0, H, rank_ * f_, f_, 0, 1, 1);
            if (!rc) pack(&y.down_items, H, f_, kPackRows);
            continue;
        }
        // q/k/v: this rank's heads, concatenated
        w4_alloc(y.qkv, q_ + 2 * kv_, H);
        if (!rc) w4_copy(y.qkv, p + "attention.wq", H, rank_ * q_, q_, 0, H, 0, 1, 1);
        if (!rc) w4_copy(y.qkv, p + "attention.wk", H, rank_ * kv_, kv_, 0, H, q_, 1, 1);
        if (!rc) w4_copy(y.qkv, p + "attention.wv", H, rank_ * kv_, kv_, 0, H, q_ + kv_, 1, 1);
        // o: all rows, this rank's K slice (row parallel)
        w4_alloc(y.o, H, q_);
        if (!rc) w4_copy(y.o, p + "attention.wo", Q, 0, H, rank_ * q_, q_, 0, 1, 1);
        // gate/up: this rank's FFN rows, interleaved per GEMV tile (half gate, half up)
        w4_alloc(y.gu, 2 * f_, H);
        if (!rc) w4_copy(y.gu, p + "feed_forward.w1", H, rank_ * f_, f_, 0, H, 0, half, kW4TileRows);
        if (!rc) w4_copy(y.gu, p + "feed_forward.w3", H, rank_ * f_, f_, 0, H, half, half, kW4TileRows);
        // down: all rows, this rank's K slice
        w4_alloc(y.down, H, f_);
        if (!rc) w4_copy(y.down, p + "feed_forward.w2", F, 0, H, rank_ * f_, f_, 0, 1, 1);
    }
    if (!rc) {
        if (head_kind_ == 2) {
            w4_alloc(head_w4_, v_, H);
            if (!rc) w4_copy(head_w4_, "output", H, v_off_, v_, 0, H, 0, 1, 1);
        } else {
            const size_t rb = size_t(H) * (head_kind_ == 1 ? 2 : 4);
            head_dense_ = alloc(size_t(v_) * rb);
            if (!head_dense_) rc = FIRE_B200_ERR_NOMEM;
            if (!rc) rc = copy2d(head_dense_, rb, head, size_t(v_off_) * rb, rb, rb, v_, s);
        }
    }
    std::vector<StackLayer> host_layers;
    if (!rc && stack_) {
        for (const auto& y : layers_)
            host_layers.push_back(StackLayer{y.attn_norm, y.ffn_norm, y.q_norm, y.k_norm, y.qkv_items, y.o_items,
                                             y.gu_items, y.down_items});
        stack_layers_ = static_cast<StackLayer*>(alloc(size_t(L) * sizeof(StackLayer)));
        if (!stack_layers_) rc = FIRE_B200_ERR_NOMEM;
        if (!rc)
            rc = static_cast<int>(cudaMemcpyAsync(stack_layers_, host_layers.data(), size_t(L) * sizeof(StackLayer),
                                                  cudaMemcpyHostToDevice, s));
    }
    const cudaError_t se = cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    if (tmp.qw) {
        cudaFree(tmp.qw);
        cudaFree(tmp.s);
        cudaFree(tmp.z);
    }
    if (rc) return fail(rc, rc == FIRE_B200_ERR_NOMEM ? "device weight reservation exhausted" : "weight upload failed");
    if (se != cudaSuccess) return static_cast<int>(se);

    // bytes one decode step reads (weights, norms, one embedding row)
    auto w4b = [](const W4Mat& m) { return size_t(m.n) * m.k / 2 + size_t(m.n) * (m.k / 128) * 5; };
    size_t b = size_t(H) * esize(emb->dtype) + size_t(H) * 4;
    for (const auto& y : layers_) b += w4b(y.qkv) + w4b(y.o) + w4b(y.gu) + w4b(y.down) + size_t(2 * H + 256) * 4;
    b += head_kind_ == 2 ? w4b(head_w4_) : size_t(v_) * H * (head_kind_ == 1 ? 2 : 4);
    step_weight_bytes_ = b;
    return 0;
}

int Qwen3Engine::prepare(int capacity) {
    if (capacity <= 0 || capacity > d_.max_seq) return FIRE_B200_ERR_INVALID;
    if (graph_fwd_) { cudaGraphExecDestroy(graph_fwd_); graph_fwd_ = nullptr; }
    if (graph_step_) { cudaGraphExecDestroy(graph_step_); graph_step_ = nullptr; }
    runtime_arena_.reset(new DeviceArena(device_));
    capacity_ = capacity;
    length_ = 0;
    max_chunks_ = (capacity + kAttnChunk - 1) / kAttnChunk;
    const int H = d_.hidden;
    const size_t kv_elems = size_t(d_.layers) * capacity * kv_;
    const size_t attn_ws = attention_workspace_bytes(hq_, hkv_, 128, capacity);
    const size_t am_ws = argmax_workspace_bytes(kMaxSms);
    StackArgs sa{};
    size_t stack_bytes = 0;
    if (stack_) {
        sa = stack_template(capacity);
        if (!stack_plan(&sa, sms_)) return FIRE_B200_ERR_UNSUPPORTED;
        stack_trace_words_ = stack_trace_on_ ? size_t(sa.grid) * d_.layers * kStackPhases * kStackTraceSlots : 0;
        stack_bytes = 256 + pad256(stack_trace_words_ * 8) + pad256(stack_sync_words(sa) * 4) + pad256(stack_kpart_floats(sa) * 4 + 4) +
                      pad256(size_t(hq_) * sa.max_chunks * 128 * 4) + pad256(size_t(hq_) * sa.max_chunks * 2 * 4) + 1024;
    }
    size_t total = 0;
    const size_t sizes[] = {256, size_t(H) * 4 * 5, size_t(q_ + 2 * kv_) * 4, size_t(q_) * 8, size_t(f_) * 4,
                            size_t(v_) * 4, size_t(d_.vocab) * 4, kv_elems * 8, size_t(capacity) * 64 * 8,
                            attn_ws, am_ws, 256, 256 * size_t(tp_), size_t(capacity) * 4, stack_bytes};
    for (size_t sz : sizes) total += pad256(sz) + 256;
    FB_RC(runtime_arena_->reserve(total));
    auto A = [&](size_t b) { return runtime_arena_->alloc(b); };
    state_ = static_cast<DecodeState*>(A(sizeof(DecodeState)));
    hidden_ = static_cast<float*>(A(size_t(H) * 4));
    attn_res_ = static_cast<float*>(A(size_t(H) * 4));
    o_part_ = static_cast<float*>(A(size_t(H) * 4));
    down_part_ = static_cast<float*>(A(size_t(H) * 4));
    qkv_ = static_cast<float*>(A(size_t(q_ + 2 * kv_) * 4));
    q_rot_ = static_cast<float*>(A(size_t(q_) * 4));
    attn_out_ = static_cast<float*>(A(size_t(q_) * 4));
    act_ = static_cast<float*>(A(size_t(f_) * 4));
    logits_ = static_cast<float*>(A(size_t(v_) * 4));
    logits_full_ = tp_ > 1 ? static_cast<float*>(A(size_t(d_.vocab) * 4)) : logits_;
    kcache_ = static_cast<float*>(A(kv_elems * 4));
    vcache_ = static_cast<float*>(A(kv_elems * 4));
    rope_sin_ = static_cast<float*>(A(size_t(capacity) * 64 * 4));
    rope_cos_ = static_cast<float*>(A(size_t(capacity) * 64 * 4));
    attn_ws_ = A(attn_ws);
    argmax_ws_ = A(am_ws);
    best_local_ = A(kArgmaxPairBytes);
    best_all_ = A(kArgmaxPairBytes * tp_);
    tokens_buf_ = static_cast<int32_t*>(A(size_t(capacity) * 4));
    if (!state_ || !hidden_ || !attn_res_ || !o_part_ || !down_part_ || !qkv_ || !q_rot_ || !attn_out_ || !act_ ||
        !logits_ || !logits_full_ || !kcache_ || !vcache_ || !rope_sin_ || !rope_cos_ || !attn_ws_ || !argmax_ws_ ||
        !best_local_ || !best_all_ || !tokens_buf_)
        return FIRE_B200_ERR_NOMEM;
    if (stack_) {
        stack_sync_bytes_ = stack_sync_words(sa) * 4;
        stack_sync_ = static_cast<unsigned*>(A(stack_sync_bytes_));
        sa.kpart = static_cast<float*>(A(stack_kpart_floats(sa) * 4 + 4));
        sa.attn_part = static_cast<float*>(A(size_t(hq_) * sa.max_chunks * 128 * 4));
        sa.attn_ml = static_cast<float*>(A(size_t(hq_) * sa.max_chunks * 2 * 4));
        if (!stack_sync_ || !sa.kpart || !sa.attn_part || !sa.attn_ml) return FIRE_B200_ERR_NOMEM;
        sa.layers = stack_layers_;
        sa.state = state_;
        sa.hidden_buf = hidden_;
        sa.attn_res = attn_res_;
        sa.qkv = qkv_;
        sa.attn_out = attn_out_;
        sa.act = act_;
        sa.kcache = kcache_;
        sa.vcache = vcache_;
        sa.rope_sin = rope_sin_;
        sa.rope_cos = rope_cos_;
        sa.sync = stack_sync_;
        if (tp_ > 1) stack_bind_exchange(&sa, tp_, rank_, xchg_peer_);
        sa.trace = nullptr;
        sa.stall = nullptr;
        if (stall_on_) {
            stall_ = static_cast<int*>(A(sizeof(int)));
            if (!stall_) return FIRE_B200_ERR_NOMEM;
            FB_CK(cudaMemset(stall_, 0, sizeof(int)));  // armed below, after the checking step
            sa.stall = stall_;
        }
        if (stack_trace_words_) {
            sa.trace = static_cast<unsigned long long*>(A(stack_trace_words_ * 8));
            if (!sa.trace) return FIRE_B200_ERR_NOMEM;
        }
        stack_args_ = sa;
    }
    if (!host_state_) FB_CK(cudaMallocHost(reinterpret_cast<void**>(&host_state_), sizeof(DecodeState)));
    if (!host_seen_) FB_CK(cudaMallocHost(reinterpret_cast<void**>(&host_seen_), sizeof(DecodeState)));
    if (!steps_done_) FB_CK(cudaEventCreateWithFlags(&steps_done_, cudaEventDisableTiming));
    *host_seen_ = DecodeState{0, 0, 0, 0};

    cudaStream_t s;
    FB_CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    FB_CK(cudaMemsetAsync(state_, 0, sizeof(DecodeState), s));
    FB_CK(cudaMemsetAsync(attn_ws_, 0, attn_ws, s));
    FB_CK(cudaMemsetAsync(argmax_ws_, 0, am_ws, s));
    FB_CK(cudaMemsetAsync(kcache_, 0, kv_elems * 4, s));
    FB_CK(cudaMemsetAsync(vcache_, 0, kv_elems * 4, s));
    // RoPE caches for positions 0..capacity-1 (Qwen3Model::prepare, src/model/qwen.cpp:143-149)
    FB_CK(rope_cache_launch(128, capacity, d_.theta, rope_sin_, rope_cos_, sms_, s));
    // one eager step: sets kernel attributes and checks every launch before capture
    int rc = enqueue_step(s, true);
    if (rc == 0) rc = static_cast<int>(cudaStreamSynchronize(s));
    if (rc == 0) rc = static_cast<int>(cudaMemsetAsync(state_, 0, sizeof(DecodeState), s));
    if (rc == 0) rc = static_cast<int>(cudaStreamSynchronize(s));
    cudaStreamDestroy(s);
    if (rc) return rc;
    if (opt_.use_graph) {
        FB_RC(capture(false, &graph_fwd_));
        FB_RC(capture(true, &graph_step_));
    }
    if (stall_) {
        const int one = 1;
        FB_CK(cudaMemcpy(stall_, &one, sizeof(int), cudaMemcpyHostToDevice));
    }
    return 0;
}

// The layer-stack kernel is always launched cooperative, captured or not: its CTAs wait on
// one another, so all of them must be resident at once, which only the cooperative launch
// guarantees. A runtime that refuses it makes prepare() fail (the kernel is never run as a
// plain launch).
int Qwen3Engine::capture(bool sample, cudaGraphExec_t* exec) {
    cudaStream_t cs;
    FB_CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    int rc = e == cudaSuccess ? 0 : static_cast<int>(e);
    if (!rc) {
        rc = enqueue_step(cs, sample);
        e = cudaStreamEndCapture(cs, &g);
        if (!rc && e != cudaSuccess) rc = static_cast<int>(e);
    }
    if (!rc) {
        e = cudaGraphInstantiate(exec, g, 0);
        if (e != cudaSuccess) rc = static_cast<int>(e);
    }
    if (g) cudaGraphDestroy(g);
    cudaStreamDestroy(cs);
    return rc;
}

int Qwen3Engine::enqueue_step(cudaStream_t s, bool sample) {
    const bool pdl = opt_.pdl;
    const int H = d_.hidden;
    auto allreduce = [&](float* buf) -> int {
        const int r = nccl().AllReduce(buf, buf, size_t(H), kNcclFloat32, 0, comm_, s);
        return r == 0 ? 0 : FIRE_B200_ERR_STATE;
    };
    auto mat = [this](W4Args& a, const W4Mat& m) {
        a.err = &state_->error;
        a.qw = m.qw;
        a.scales = m.s;
        a.zeros = m.z;
        a.N = m.n;
        a.K = m.k;
    };
    FB_CK(embedding_launch(nullptr, 1, state_, embedding_, emb_bf16_, d_.vocab, H, hidden_, s, pdl));
    if (stack_) {
        FB_CK(cudaMemsetAsync(stack_sync_, 0, stack_sync_bytes_, s));
        if (stack_args_.trace) FB_CK(cudaMemsetAsync(stack_args_.trace, 0, stack_trace_words_ * 8, s));
        const cudaError_t e = stack_launch(stack_args_, s, true);
        if (e == cudaErrorCooperativeLaunchTooLarge || e == cudaErrorNotSupported) {
            (void)cudaGetLastError();
            return FIRE_B200_ERR_UNSUPPORTED;  // co-residency of the CTAs cannot be guaranteed
        }
        FB_CK(e);
    }
    for (int l = 0; l < (stack_ ? 0 : d_.layers); ++l) {
        const Layer& L = layers_[l];
        const size_t kv_layer = size_t(l) * capacity_ * kv_;
        // q/k/v = W_qkv . rmsnorm(h)   (qwen.cpp:196-217)
        W4Args a{};
        if (tp_ > 1 && l > 0) {
            a.x = attn_res_;
            a.x_add = down_part_;
            a.x_sum_out = hidden_;
        } else {
            a.x = hidden_;
        }
        a.norm_w = L.attn_norm;
        a.eps = d_.eps;
        mat(a, L.qkv);
        a.y = qkv_;
        a.prefetch = 1;
        FB_CK(w4g128_gemv_launch(a, kW4Store, sms_, s, pdl));
        // q_norm / k_norm, RoPE, KV write (qwen.cpp:222-240) fused into attention (qwen.cpp:242-247)
        AttnArgs at{};
        at.q = nullptr;
        at.qkv = qkv_;
        at.q_norm = L.q_norm;
        at.k_norm = L.k_norm;
        at.rope_sin = rope_sin_;
        at.rope_cos = rope_cos_;
        at.eps = d_.eps;
        at.key_cache = kcache_ + kv_layer;
        at.value_cache = vcache_ + kv_layer;
        at.out = attn_out_;
        at.tickets = static_cast<unsigned*>(attn_ws_);
        at.part_ml = reinterpret_cast<float*>(static_cast<char*>(attn_ws_) + 256);
        at.part = at.part_ml + size_t(hq_) * max_chunks_ * 2;
        at.state = state_;
        at.q_heads = hq_;
        at.kv_heads = hkv_;
        at.hd = 128;
        at.capacity = capacity_;
        at.max_chunks = max_chunks_;
        at.scale = 1.0f / sqrtf(128.0f);
        FB_CK(attention_launch(at, s, pdl));
        // o projection + residual (qwen.cpp:249-262)
        W4Args o{};
        o.x = attn_out_;
        mat(o, L.o);
        o.prefetch = 1;
        if (tp_ == 1) {
            o.y = attn_res_;
            o.residual = hidden_;
            FB_CK(w4g128_gemv_launch(o, kW4Residual, sms_, s, pdl));
        } else {
            o.y = o_part_;
            FB_CK(w4g128_gemv_launch(o, kW4Store, sms_, s, pdl));
            FB_RC(allreduce(o_part_));
        }
        // gate/up . rmsnorm(attn_res), SwiGLU (qwen.cpp:264-281)
        W4Args g{};
        if (tp_ == 1) {
            g.x = attn_res_;
        } else {
            g.x = hidden_;
            g.x_add = o_part_;
            g.x_sum_out = attn_res_;
        }
        g.norm_w = L.ffn_norm;
        g.eps = d_.eps;
        mat(g, L.gu);
        g.y = act_;
        g.prefetch = 1;
        FB_CK(w4g128_gemv_launch(g, kW4Swiglu, sms_, s, pdl));
        // down + residual (qwen.cpp:282-291)
        W4Args dn{};
        dn.x = act_;
        mat(dn, L.down);
        dn.prefetch = 1;
        if (tp_ == 1) {
            dn.y = hidden_;
            dn.residual = attn_res_;
            FB_CK(w4g128_gemv_launch(dn, kW4Residual, sms_, s, pdl));
        } else {
            dn.y = down_part_;
            FB_CK(w4g128_gemv_launch(dn, kW4Store, sms_, s, pdl));
            FB_RC(allreduce(down_part_));
        }
    }
    // final norm + LM head (qwen.cpp:294-301); the layer stack leaves the reduced
    // residual stream in hidden_ at every TP size, the per-op path leaves its last
    // all-reduced down partial to add here
    const bool add_down = tp_ > 1 && !stack_;
    const float* hx = add_down ? attn_res_ : hidden_;
    const float* hadd = add_down ? down_part_ : nullptr;
    float* hsum = add_down ? hidden_ : nullptr;
    if (head_kind_ == 2) {
        W4Args h{};
        h.x = hx;
        h.x_add = hadd;
        h.x_sum_out = hsum;
        h.norm_w = final_norm_;
        h.eps = d_.eps;
        mat(h, head_w4_);
        h.y = logits_;
        h.prefetch = 1;
        FB_CK(w4g128_gemv_launch(h, kW4Store, sms_, s, pdl));
    } else {
        DenseArgs h{};
        h.x = hx;
        h.x_add = hadd;
        h.x_sum_out = hsum;
        h.norm_w = final_norm_;
        h.eps = d_.eps;
        h.w = head_dense_;
        h.scale = 1.0f;
        h.y = logits_;
        h.N = v_;
        h.K = H;
        h.prefetch = 1;
        FB_CK(dense_gemv_launch(h, head_kind_ == 1, sms_, s, pdl));
    }
    const int am_sms = sms_ < kMaxSms ? sms_ : kMaxSms;
    if (sample) {
        if (tp_ == 1) {
            FB_CK(argmax_launch(logits_, v_, argmax_ws_, am_sms, nullptr, state_, tokens_buf_, capacity_, s, pdl));
        } else {
            FB_CK(argmax_launch(logits_, v_, argmax_ws_, am_sms, nullptr, nullptr, nullptr, 0, s, pdl, v_off_,
                                best_local_));
            const int r = nccl().AllGather(best_local_, best_all_, kArgmaxPairBytes, kNcclUint8, comm_, s);
            if (r != 0) return FIRE_B200_ERR_STATE;
            FB_CK(argmax_select_launch(best_all_, tp_, state_, tokens_buf_, capacity_, s, pdl));
        }
    } else if (tp_ > 1) {
        const int r = nccl().AllGather(logits_, logits_full_, size_t(v_), kNcclFloat32, comm_, s);
        if (r != 0) return FIRE_B200_ERR_STATE;
    }
    return 0;
}

int Qwen3Engine::launch_step(cudaStream_t s, bool sample) {
    cudaGraphExec_t g = sample ? graph_step_ : graph_fwd_;
    if (g) return static_cast<int>(cudaGraphLaunch(g, s));
    return enqueue_step(s, sample);
}

int Qwen3Engine::kernels_per_step() const {
    if (stack_) return 4 + (tp_ > 1 ? 1 : 0);  // embedding, layer stack, LM head, argmax (+ rank select)
    return 5 * d_.layers + 3 + (tp_ > 1 ? 1 : 0);
}

int Qwen3Engine::time_layer_stack(int reps, float* ms_out, cudaStream_t s) {
    if (!stack_ || capacity_ == 0) return FIRE_B200_ERR_STATE;
    if (reps <= 0 || ms_out == nullptr || length_ >= capacity_) return FIRE_B200_ERR_INVALID;
    FB_CK(set_state_launch(state_, 0, length_, 0, s, false));
    cudaEvent_t e0, e1;
    FB_CK(cudaEventCreate(&e0));
    FB_CK(cudaEventCreate(&e1));
    int rc = 0;
    for (int i = 0; i <= reps && rc == 0; ++i) {  // launch 0 warms up
        if (i == 1) rc = static_cast<int>(cudaEventRecord(e0, s));
        if (!rc) rc = static_cast<int>(cudaMemsetAsync(stack_sync_, 0, stack_sync_bytes_, s));
        if (!rc) rc = static_cast<int>(stack_launch(stack_args_, s, true));
    }
    if (!rc) rc = static_cast<int>(cudaEventRecord(e1, s));
    if (!rc) rc = static_cast<int>(cudaEventSynchronize(e1));
    float ms = 0.0f;
    if (!rc) rc = static_cast<int>(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc) return rc;
    *ms_out = ms / static_cast<float>(reps);
    return 0;
}

int64_t Qwen3Engine::stack_trace(uint64_t* host_out, int64_t capacity_words) const {
    if (!stack_args_.trace || !stack_trace_words_) return 0;
    const int64_t n = static_cast<int64_t>(stack_trace_words_);
    if (host_out && capacity_words > 0) {
        const size_t m = static_cast<size_t>(capacity_words < n ? capacity_words : n);
        if (cudaDeviceSynchronize() != cudaSuccess) return -1;
        if (cudaMemcpy(host_out, stack_args_.trace, m * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    }
    return n;
}

StackArgs Qwen3Engine::stack_template(int capacity) const {
    StackArgs a{};
    a.L = d_.layers;
    a.hidden = d_.hidden;
    a.q_dim = q_;
    a.kv_dim = kv_;
    a.inter = f_;
    a.q_heads = hq_;
    a.kv_heads = hkv_;
    a.tp = tp_;
    a.rank = rank_;
    a.eps = d_.eps;
    a.scale = 1.0f / sqrtf(128.0f);
    a.capacity = capacity;
    return a;
}

int Qwen3Engine::forward(int token, int pos, float* logits_out, cudaStream_t s) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    FB_RC(refuse());
    if (token < 0 || token >= d_.vocab) return FIRE_B200_ERR_INVALID;
    if (pos != length_ || pos < 0 || pos >= capacity_) return FIRE_B200_ERR_STATE;
    FB_CK(set_state_launch(state_, token, pos, 0, s, false));
    FB_RC(launch_step(s, false));
    if (logits_out != nullptr && logits_out != logits())
        FB_CK(cudaMemcpyAsync(logits_out, logits(), size_t(d_.vocab) * 4, cudaMemcpyDeviceToDevice, s));
    FB_RC(mark_steps(s));
    ++length_;  // KVCache::commit (src/model/kv_cache.cpp:76-83)
    return 0;
}

int Qwen3Engine::mark_steps(cudaStream_t s) {
    FB_CK(cudaMemcpyAsync(host_seen_, state_, sizeof(DecodeState), cudaMemcpyDeviceToHost, s));
    FB_CK(cudaEventRecord(steps_done_, s));
    return 0;
}

int Qwen3Engine::refuse() const {
    if (aborted_) return FIRE_B200_ERR_TIMEOUT;
    // the mirror holds the state after the last step group that has completed (a copy
    // still in flight shows the earlier value; status() waits for it)
    const int err = *reinterpret_cast<const volatile int32_t*>(&host_seen_->error);
    return err != 0 ? FIRE_B200_ERR_DEVICE : 0;
}

int Qwen3Engine::wait_event(cudaEvent_t ev) {
    if (tp_ == 1 || comm_ == nullptr) return static_cast<int>(cudaEventSynchronize(ev));
    // Tensor parallel: a peer that stopped answering leaves this rank's collective (or its
    // exchange polls) unfinished; wait with a deadline, watching the communicator, and
    // abort it when the deadline passes (ncclCommAbort ends its kernels).
    const long long limit_ms = opt_.deadline_ms > 0 ? opt_.deadline_ms : 30000;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return 0;
        if (q != cudaErrorNotReady) return static_cast<int>(q);
        int async_err = 0;
        if (nccl().CommGetAsyncError(comm_, &async_err) == 0 && async_err != 0 && async_err != kNcclInProgress) {
            nccl().CommAbort(comm_);
            comm_ = nullptr;
            aborted_ = true;
            return FIRE_B200_ERR_TIMEOUT;
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0);
        if (ms.count() > limit_ms) {
            nccl().CommAbort(comm_);
            comm_ = nullptr;
            aborted_ = true;
            return FIRE_B200_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int Qwen3Engine::status(int* device_error) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    if (aborted_) return FIRE_B200_ERR_TIMEOUT;
    FB_RC(wait_event(steps_done_));
    const int err = host_seen_->error;
    if (device_error) *device_error = err;
    return err != 0 ? FIRE_B200_ERR_DEVICE : 0;
}

int Qwen3Engine::abort() {
    if (comm_ != nullptr && nccl().ok) {
        nccl().CommAbort(comm_);
        comm_ = nullptr;
        aborted_ = true;
    }
    return 0;
}

int Qwen3Engine::kv_export(int length, float* key, float* value, cudaStream_t s) const {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    if (!key || !value || length < 0 || length > length_) return FIRE_B200_ERR_INVALID;
    const size_t row = size_t(kv_) * 4, part = size_t(length) * row;
    for (int l = 0; l < d_.layers; ++l) {
        const size_t src = size_t(l) * capacity_ * kv_;
        FB_CK(cudaMemcpyAsync(reinterpret_cast<char*>(key) + l * part, kcache_ + src, part, cudaMemcpyDefault, s));
        FB_CK(cudaMemcpyAsync(reinterpret_cast<char*>(value) + l * part, vcache_ + src, part, cudaMemcpyDefault, s));
    }
    FB_CK(cudaStreamSynchronize(s));
    return 0;
}

int Qwen3Engine::kv_import(int length, const float* key, const float* value, cudaStream_t s) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    FB_RC(refuse());
    if (!key || !value || length < 0 || length > capacity_) return FIRE_B200_ERR_INVALID;
    const size_t row = size_t(kv_) * 4, part = size_t(length) * row;
    for (int l = 0; l < d_.layers; ++l) {
        const size_t dst = size_t(l) * capacity_ * kv_;
        FB_CK(cudaMemcpyAsync(kcache_ + dst, reinterpret_cast<const char*>(key) + l * part, part, cudaMemcpyDefault, s));
        FB_CK(cudaMemcpyAsync(vcache_ + dst, reinterpret_cast<const char*>(value) + l * part, part, cudaMemcpyDefault, s));
    }
    FB_CK(cudaStreamSynchronize(s));
    length_ = length;
    return 0;
}

namespace {
constexpr int kPrefillChunk = 2048;   // prompt rows per batched step (one pass of W per layer up to here)
constexpr int kPrefillMinRows = 64;   // below this the per-token path is as fast
}  // namespace

int Qwen3Engine::prefill_buffers() {
    if (prefill_arena_) return 0;
    const size_t C = kPrefillChunk, H = d_.hidden;
    const size_t qkv = size_t(q_ + 2 * kv_), maxk = std::max({size_t(H), size_t(q_), size_t(f_)});
    // FP16 copy of the largest matrix, used by the two-pass form
    const size_t maxw =
        !prefill_one_pass() ? std::max({qkv * H, size_t(H) * q_, size_t(2 * f_) * H, size_t(H) * f_}) * 2 : 256;
    pf_gemm_ws_bytes_ = prefill_gemm_workspace_bytes(kPrefillChunk, static_cast<int>(maxk));
    std::unique_ptr<DeviceArena> ar(new DeviceArena(device_));
    const size_t sizes[] = {C * 4, C * H * 4, C * H * 4, C * qkv * 4, C * q_ * 4, C * q_ * 4, C * H * 4,
                            C * 2 * f_ * 4, C * f_ * 4, pf_gemm_ws_bytes_, maxw, 256};
    size_t total = 0;
    for (size_t z : sizes) total += pad256(z) + 256;
    FB_RC(ar->reserve(total));
    pf_tok_ = static_cast<int32_t*>(ar->alloc(C * 4));
    pf_x_ = static_cast<float*>(ar->alloc(C * H * 4));
    pf_xn_ = static_cast<float*>(ar->alloc(C * H * 4));
    pf_qkv_ = static_cast<float*>(ar->alloc(C * qkv * 4));
    pf_q_ = static_cast<float*>(ar->alloc(C * q_ * 4));
    pf_att_ = static_cast<float*>(ar->alloc(C * q_ * 4));
    pf_o_ = static_cast<float*>(ar->alloc(C * H * 4));
    pf_gu_ = static_cast<float*>(ar->alloc(C * 2 * f_ * 4));
    pf_act_ = static_cast<float*>(ar->alloc(C * f_ * 4));
    pf_gemm_ws_ = ar->alloc(pf_gemm_ws_bytes_);
    pf_w_ = ar->alloc(maxw);
    pf_err_ = static_cast<int*>(ar->alloc(256));
    if (!pf_tok_ || !pf_x_ || !pf_xn_ || !pf_qkv_ || !pf_q_ || !pf_att_ || !pf_o_ || !pf_gu_ || !pf_act_ ||
        !pf_gemm_ws_ || !pf_w_ || !pf_err_)
        return FIRE_B200_ERR_NOMEM;
    FB_CK(cudaMemset(pf_err_, 0, 256));
    prefill_arena_ = std::move(ar);
    return 0;
}

// y[mp, n] = x[mp, k] . W^T for a layer-stack item matrix W, dequantised into FP16 scratch
// first (two-pass, the default) or, with FIRE_B200_PREFILL_FUSED=1, into shared memory
// inside the GEMM
int Qwen3Engine::prefill_linear(const float* x, const uint8_t* items, int n, int k, float* y, int mp,
                                cudaStream_t s) {
    if (prefill_one_pass()) {
        FB_CK(prefill_w4_fused_launch(x, items, nullptr, nullptr, true, y, mp, n, k, pf_gemm_ws_, pf_gemm_ws_bytes_,
                                      pf_err_, s));
        return 0;
    }
    FB_CK(prefill_dequant_items_launch(items, n, k, pf_w_, pf_err_, s));
    FB_CK(prefill_gemm_launch(x, pf_w_, y, mp, n, k, pf_gemm_ws_, pf_gemm_ws_bytes_, pf_err_, s));
    return 0;
}

int Qwen3Engine::prefill_chunk(int m, int mp, int pos0, cudaStream_t s) {
    const int H = d_.hidden;
    FB_CK(embedding_launch(pf_tok_, m, nullptr, embedding_, emb_bf16_, d_.vocab, H, pf_x_, s, false));
    if (mp > m) {
        FB_CK(cudaMemsetAsync(pf_x_ + size_t(m) * H, 0, size_t(mp - m) * H * 4, s));
        FB_CK(cudaMemsetAsync(pf_att_ + size_t(m) * q_, 0, size_t(mp - m) * q_ * 4, s));
    }
    for (int l = 0; l < d_.layers; ++l) {
        const Layer& L = layers_[l];
        // q/k/v = W_qkv . rmsnorm(x) for every row (qwen.cpp:196-217)
        FB_CK(rmsnorm_rows_launch(pf_x_, L.attn_norm, pf_xn_, mp, H, d_.eps, s));
        FB_RC(prefill_linear(pf_xn_, L.qkv_items, q_ + 2 * kv_, H, pf_qkv_, mp, s));
        // q/k norm + RoPE, KV write (qwen.cpp:222-240), causal attention (qwen.cpp:242-247)
        PrefillRowsArgs pa{};
        pa.n = m;
        pa.pos0 = pos0;
        pa.q_heads = hq_;
        pa.kv_heads = hkv_;
        pa.eps = d_.eps;
        pa.scale = 1.0f / sqrtf(128.0f);
        pa.qkv = pf_qkv_;
        pa.q_norm = L.q_norm;
        pa.k_norm = L.k_norm;
        pa.rope_sin = rope_sin_;
        pa.rope_cos = rope_cos_;
        pa.q_out = pf_q_;
        pa.kcache = kcache_ + size_t(l) * capacity_ * kv_;
        pa.vcache = vcache_ + size_t(l) * capacity_ * kv_;
        pa.attn_out = pf_att_;
        FB_CK(qk_rope_kv_rows_launch(pa, s));
        FB_CK(causal_attention_launch(pa, s));
        // o projection + residual (qwen.cpp:249-262); under tensor parallelism each rank holds
        // a K slice of o (its heads), so the rows are partial sums: all-reduced first
        FB_RC(prefill_linear(pf_att_, L.o_items, H, q_, pf_o_, mp, s));
        if (tp_ > 1 && nccl().AllReduce(pf_o_, pf_o_, size_t(mp) * H, kNcclFloat32, 0, comm_, s) != 0)
            return FIRE_B200_ERR_STATE;
        FB_CK(add_launch(pf_x_, pf_o_, pf_x_, mp * H, sms_, s));
        // SwiGLU FFN + residual (qwen.cpp:264-291)
        FB_CK(rmsnorm_rows_launch(pf_x_, L.ffn_norm, pf_xn_, mp, H, d_.eps, s));
        FB_RC(prefill_linear(pf_xn_, L.gu_items, 2 * f_, H, pf_gu_, mp, s));
        FB_CK(swiglu_packed_rows_launch(pf_gu_, pf_act_, mp, f_, sms_, s));
        FB_RC(prefill_linear(pf_act_, L.down_items, H, f_, pf_o_, mp, s));
        if (tp_ > 1 && nccl().AllReduce(pf_o_, pf_o_, size_t(mp) * H, kNcclFloat32, 0, comm_, s) != 0)
            return FIRE_B200_ERR_STATE;
        FB_CK(add_launch(pf_x_, pf_o_, pf_x_, mp * H, sms_, s));
    }
    return 0;
}

int Qwen3Engine::prefill(const int32_t* tokens, int n, float* logits_out, cudaStream_t s) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    FB_RC(refuse());
    if (tokens == nullptr || n <= 0 || length_ + n > capacity_) return FIRE_B200_ERR_INVALID;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d_.vocab) return FIRE_B200_ERR_INVALID;
    if (!stack_ || n < kPrefillMinRows) {
        for (int i = 0; i < n; ++i) FB_RC(forward(tokens[i], length_, i == n - 1 ? logits_out : nullptr, s));
        return 0;
    }
    FB_RC(prefill_buffers());
    int done = 0, last_m = 0;
    while (done < n) {
        const int m = std::min(kPrefillChunk, n - done);
        const int mp = (m + kPrefillBM - 1) / kPrefillBM * kPrefillBM;
        FB_CK(cudaMemcpyAsync(pf_tok_, tokens + done, size_t(m) * 4, cudaMemcpyHostToDevice, s));
        FB_RC(prefill_chunk(m, mp, length_, s));
        // the token buffer is reused by the next chunk; under tensor parallelism the wait
        // has the host deadline (the chunk holds collectives)
        FB_CK(cudaEventRecord(steps_done_, s));
        FB_RC(wait_event(steps_done_));
        length_ += m;
        done += m;
        last_m = m;
    }
    // final norm + LM head on the last row (qwen.cpp:294-301)
    const float* hx = pf_x_ + size_t(last_m - 1) * d_.hidden;
    if (head_kind_ == 2) {
        W4Args h{};
        h.x = hx;
        h.norm_w = final_norm_;
        h.eps = d_.eps;
        h.qw = head_w4_.qw;
        h.scales = head_w4_.s;
        h.zeros = head_w4_.z;
        h.N = head_w4_.n;
        h.K = head_w4_.k;
        h.y = logits_;
        FB_CK(w4g128_gemv_launch(h, kW4Store, sms_, s, false));
    } else {
        DenseArgs h{};
        h.x = hx;
        h.norm_w = final_norm_;
        h.eps = d_.eps;
        h.w = head_dense_;
        h.scale = 1.0f;
        h.y = logits_;
        h.N = v_;
        h.K = d_.hidden;
        FB_CK(dense_gemv_launch(h, head_kind_ == 1, sms_, s, false));
    }
    // vocab-sharded head: every rank gets the full logits
    if (tp_ > 1 && nccl().AllGather(logits_, logits_full_, size_t(v_), kNcclFloat32, comm_, s) != 0)
        return FIRE_B200_ERR_STATE;
    if (logits_out != nullptr && logits_out != logits())
        FB_CK(cudaMemcpyAsync(logits_out, logits(), size_t(d_.vocab) * 4, cudaMemcpyDeviceToDevice, s));
    FB_CK(cudaEventRecord(steps_done_, s));
    FB_RC(wait_event(steps_done_));  // with the host deadline under tensor parallelism
    int err = 0;
    FB_CK(cudaMemcpy(&err, pf_err_, 4, cudaMemcpyDeviceToHost));
    if (err == 4) return FIRE_B200_ERR_UNSUPPORTED;  // weights beyond the FP16 range of the GEMM
    return err == 0 ? 0 : FIRE_B200_ERR_STATE;
}

int Qwen3Engine::generate(int first_token, int steps, int32_t* tokens_out, cudaStream_t s) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    FB_RC(refuse());
    if (first_token < 0 || first_token >= d_.vocab || steps < 1) return FIRE_B200_ERR_INVALID;
    if (length_ + steps > capacity_) return FIRE_B200_ERR_STATE;
    FB_CK(set_state_launch(state_, first_token, length_, 0, s, false));
    for (int i = 0; i < steps; ++i) FB_RC(launch_step(s, true));
    if (tokens_out != nullptr && tokens_out != tokens_buf_)
        FB_CK(cudaMemcpyAsync(tokens_out, tokens_buf_, size_t(steps) * 4, cudaMemcpyDeviceToDevice, s));
    FB_RC(mark_steps(s));
    length_ += steps;
    return 0;
}

int Qwen3Engine::generate_host(const int32_t* prompt, int n_prompt, int steps, int32_t* out_host, cudaStream_t s) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    FB_RC(refuse());
    if (!prompt || n_prompt < 1 || steps < 1 || !out_host) return FIRE_B200_ERR_INVALID;
    if (length_ + n_prompt + steps - 1 > capacity_) return FIRE_B200_ERR_STATE;
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= d_.vocab) return FIRE_B200_ERR_INVALID;
    for (int i = 0; i + 1 < n_prompt; ++i) {
        FB_CK(set_state_launch(state_, prompt[i], length_, 0, s, false));
        FB_RC(launch_step(s, false));
        ++length_;
    }
    int32_t token = prompt[n_prompt - 1];
    for (int i = 0; i < steps; ++i) {
        // H2D of this step's input from pinned memory, one step, D2H of the sample.
        *host_state_ = DecodeState{token, length_, 0, 0};
        FB_CK(cudaMemcpyAsync(state_, host_state_, sizeof(DecodeState), cudaMemcpyHostToDevice, s));
        FB_RC(launch_step(s, true));
        // D2H of the state (sampled id and error word), then wait (with the host deadline
        // under tensor parallelism)
        FB_RC(mark_steps(s));
        FB_RC(wait_event(steps_done_));
        if (host_seen_->error != 0) return FIRE_B200_ERR_DEVICE;
        token = host_seen_->token;
        out_host[i] = token;
        ++length_;  // the step consumed its input (n_prompt + steps - 1 tokens in all)
    }
    return 0;
}

int Qwen3Engine::truncate(int length) {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    if (length < 0 || length > length_) return FIRE_B200_ERR_INVALID;
    length_ = length;
    return 0;
}

int Qwen3Engine::reset() {
    if (capacity_ == 0) return FIRE_B200_ERR_STATE;
    if (aborted_) return FIRE_B200_ERR_TIMEOUT;
    // a failed step leaves its error word in the state until here
    FB_RC(wait_event(steps_done_));
    FB_CK(cudaMemset(state_, 0, sizeof(DecodeState)));
    if (stall_) FB_CK(cudaMemset(stall_, 0, sizeof(int)));  // an injected failure lasts until here
    FB_CK(cudaDeviceSynchronize());
    *host_seen_ = DecodeState{0, 0, 0, 0};
    length_ = 0;  // KVCache::reset (src/model/kv_cache.cpp:85)
    return 0;
}

}  // namespace fb
