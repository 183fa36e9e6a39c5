// extern "C" engine entry points (include/fire_b200_qwen3.h).
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "engine/fire_file.h"
#include "engine/nccl_shim.h"
#include "engine/qwen3.h"
#include "fire_b200_qwen3.h"

struct fire_b200_qwen3 {
    std::unique_ptr<fb::Qwen3Engine> e;
};

namespace {
thread_local std::string g_last_error;

fb::Qwen3Dims dims(const fire_b200_qwen3_profile* p) {
    fb::Qwen3Dims d;
    d.vocab = p->vocab_size;
    d.max_seq = p->max_seq_len;
    d.hidden = p->hidden_size;
    d.inter = p->intermediate_size;
    d.layers = p->num_layers;
    d.q_heads = p->num_attention_heads;
    d.kv_heads = p->num_kv_heads;
    d.head_dim = p->head_dim;
    d.eps = p->rms_norm_eps;
    d.theta = p->rope_theta;
    return d;
}

fb::EngineOptions options(const fire_b200_qwen3_options* o) {
    fb::EngineOptions eo;
    if (o != nullptr) {
        eo.tp_rank = o->tp_rank;
        eo.tp_size = o->tp_size;
        eo.nccl_id = o->nccl_id;
        eo.use_graph = o->use_graph != 0;
        eo.pdl = o->pdl != 0;
        eo.deadline_ms = o->deadline_ms;
    }
    return eo;
}

int make(const fire_b200_qwen3_profile* p, const std::vector<fb::TensorSrc>& src, const fire_b200_qwen3_options* o,
         fire_b200_qwen3** out) {
    std::unique_ptr<fb::Qwen3Engine> e;
    std::string err;
    const int rc = fb::Qwen3Engine::create(dims(p), src, options(o), &e, &err);
    if (rc != 0) {
        g_last_error = err.empty() ? "engine creation failed" : err;
        return rc;
    }
    *out = new fire_b200_qwen3{std::move(e)};
    return FIRE_B200_OK;
}
}  // namespace

extern "C" {

int fire_b200_nccl_unique_id(void* id128) {
    if (id128 == nullptr) return FIRE_B200_ERR_INVALID;
    if (!fb::nccl().ok) return FIRE_B200_ERR_UNSUPPORTED;
    return fb::nccl().GetUniqueId(id128) == 0 ? FIRE_B200_OK : FIRE_B200_ERR_STATE;
}

int fire_b200_qwen3_create(const fire_b200_qwen3_profile* profile, const fire_b200_tensor* tensors, int count,
                           const fire_b200_qwen3_options* opts, fire_b200_qwen3** out) {
    g_last_error.clear();
    if (!profile || !tensors || count < 1 || !out) return FIRE_B200_ERR_INVALID;
    *out = nullptr;
    std::vector<fb::TensorSrc> src(static_cast<size_t>(count));
    for (int i = 0; i < count; ++i) {
        const fire_b200_tensor& t = tensors[i];
        if (!t.name || t.ndim < 1 || t.ndim > 2 || t.dtype < FIRE_B200_F32 || t.dtype > FIRE_B200_U8) {
            g_last_error = "malformed tensor descriptor";
            return FIRE_B200_ERR_INVALID;
        }
        src[i].name = t.name;
        src[i].dtype = t.dtype;
        src[i].shape.assign(t.shape, t.shape + t.ndim);
        src[i].data = t.data;
        src[i].on_device = t.on_device != 0;
    }
    return make(profile, src, opts, out);
}

int fire_b200_qwen3_open(const char* fire_path, const fire_b200_qwen3_profile* profile,
                         const fire_b200_qwen3_options* opts, fire_b200_qwen3** out) {
    g_last_error.clear();
    if (!fire_path || !profile || !out) return FIRE_B200_ERR_INVALID;
    *out = nullptr;
    fb::FireFile f;
    std::string err;
    if (!f.open(fire_path, &err)) {
        g_last_error = err;
        return FIRE_B200_ERR_IO;
    }
    std::vector<fb::TensorSrc> src;
    src.reserve(f.count());
    for (const auto& t : f.tensors()) {
        fb::TensorSrc s;
        s.name = t.name;
        s.dtype = t.dtype == fb::kWireF32 ? fb::kSrcF32 : (t.dtype == fb::kWireBF16 ? fb::kSrcBF16 : fb::kSrcU8);
        s.shape = t.shape;
        s.data = t.data;
        s.on_device = false;
        src.push_back(std::move(s));
    }
    return make(profile, src, opts, out);  // weights are copied before `f` unmaps
}

const char* fire_b200_qwen3_last_error(void) { return g_last_error.c_str(); }

int fire_b200_qwen3_prepare(fire_b200_qwen3* m, int capacity) {
    return m ? m->e->prepare(capacity) : FIRE_B200_ERR_INVALID;
}

int fire_b200_qwen3_forward(fire_b200_qwen3* m, int token_id, int pos, float* logits, void* stream) {
    return m ? m->e->forward(token_id, pos, logits, static_cast<cudaStream_t>(stream)) : FIRE_B200_ERR_INVALID;
}

int fire_b200_qwen3_generate(fire_b200_qwen3* m, int first_token, int steps, int32_t* tokens_out, void* stream) {
    return m ? m->e->generate(first_token, steps, tokens_out, static_cast<cudaStream_t>(stream))
             : FIRE_B200_ERR_INVALID;
}

int fire_b200_qwen3_generate_host(fire_b200_qwen3* m, const int32_t* prompt, int n_prompt, int steps, int32_t* out,
                                  void* stream) {
    return m ? m->e->generate_host(prompt, n_prompt, steps, out, static_cast<cudaStream_t>(stream))
             : FIRE_B200_ERR_INVALID;
}

int fire_b200_qwen3_reset(fire_b200_qwen3* m) { return m ? m->e->reset() : FIRE_B200_ERR_INVALID; }
int fire_b200_qwen3_status(fire_b200_qwen3* m, int* device_error) {
    return m ? m->e->status(device_error) : FIRE_B200_ERR_INVALID;
}
int fire_b200_qwen3_abort(fire_b200_qwen3* m) { return m ? m->e->abort() : FIRE_B200_ERR_INVALID; }
int fire_b200_qwen3_kv_export(const fire_b200_qwen3* m, int length, float* key, float* value, void* stream) {
    return m ? m->e->kv_export(length, key, value, static_cast<cudaStream_t>(stream)) : FIRE_B200_ERR_INVALID;
}
int fire_b200_qwen3_kv_import(fire_b200_qwen3* m, int length, const float* key, const float* value, void* stream) {
    return m ? m->e->kv_import(length, key, value, static_cast<cudaStream_t>(stream)) : FIRE_B200_ERR_INVALID;
}
int fire_b200_qwen3_truncate(fire_b200_qwen3* m, int length) {
    return m ? m->e->truncate(length) : FIRE_B200_ERR_INVALID;
}
int fire_b200_qwen3_length(const fire_b200_qwen3* m) { return m ? m->e->length() : -1; }
const float* fire_b200_qwen3_logits(const fire_b200_qwen3* m) { return m ? m->e->logits() : nullptr; }
int fire_b200_qwen3_kernels_per_step(const fire_b200_qwen3* m) { return m ? m->e->kernels_per_step() : 0; }
int fire_b200_qwen3_prefill(fire_b200_qwen3* m, const int32_t* tokens, int n, float* logits_out, void* stream) {
    if (m == nullptr) return FIRE_B200_ERR_INVALID;
    return m->e->prefill(tokens, n, logits_out, static_cast<cudaStream_t>(stream));
}
int fire_b200_qwen3_time_layer_stack(fire_b200_qwen3* m, int reps, float* ms_out, void* stream) {
    if (m == nullptr) return FIRE_B200_ERR_INVALID;
    return m->e->time_layer_stack(reps, ms_out, static_cast<cudaStream_t>(stream));
}
int64_t fire_b200_qwen3_stack_trace(const fire_b200_qwen3* m, uint64_t* out, int64_t capacity_words) {
    return m ? m->e->stack_trace(out, capacity_words) : 0;
}
uint64_t fire_b200_qwen3_step_weight_bytes(const fire_b200_qwen3* m) {
    return m ? static_cast<uint64_t>(m->e->step_weight_bytes()) : 0;
}
void fire_b200_qwen3_destroy(fire_b200_qwen3* m) { delete m; }

}  // extern "C"
