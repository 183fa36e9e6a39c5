// TEST INFRASTRUCTURE ONLY. extern "C" wrappers that call the REFERENCE's own
// kernels (compiled from its sources by oracle/Makefile) on caller pointers, so
// the parity tests can compare fire_b200 against Fire's own CPU and CUDA code.
// Nothing here is part of the fire_b200 product.
#include "Fire/base/alloc.h"
#include "Fire/tensor/tensor.h"
#include "cpu/mha_kernel.h"
#include "cpu/rmsnorm_kernel.h"
#include "cpu/rope_kernel.h"
#include "cpu/softmax_kernel.h"
#include "cuda/add_kernel.cuh"
#include "cuda/argmax_kernel.cuh"
#include "cuda/emb_kernel.cuh"
#include "cuda/matmul_kernel.cuh"
#include "cuda/mha_kernel.cuh"
#include "cuda/rmsnorm_kernel.cuh"
#include "cuda/rope_kernel.cuh"
#include "cuda/swiglu_kernel.cuh"

#include <cstdint>
#include <vector>

using base::DataType;
using base::DeviceType;
using tensor::Tensor;

namespace {
Tensor gpu(const void* p, DataType t, std::vector<int32_t> d) {
    return Tensor::from_blob(const_cast<void*>(p), t, std::move(d), DeviceType::GPU);
}
Tensor cpu(const void* p, DataType t, std::vector<int32_t> d) {
    return Tensor::from_blob(const_cast<void*>(p), t, std::move(d), DeviceType::CPU);
}
std::vector<int32_t> vec_or_mat(int rows, int cols) {
    return rows == 1 ? std::vector<int32_t>{cols} : std::vector<int32_t>{rows, cols};
}
}  // namespace

extern "C" {

// src/op/kernels/cuda/matmul_kernel.cu:280-314 (INT4 group-wise, any group).
void ref_matmul_quant_cu(const float* x, const uint8_t* qw, const float* s, const uint8_t* z,
                         float* y, int rows, int n, int k, int group, void* stream) {
    Tensor in = gpu(x, DataType::Fp32, vec_or_mat(rows, k));
    Tensor w = gpu(qw, DataType::UInt8, {n, k / 2});
    Tensor out = gpu(y, DataType::Fp32, vec_or_mat(rows, n));
    Tensor sc = gpu(s, DataType::Fp32, {n, k / group});
    Tensor zp = gpu(z, DataType::UInt8, {n, k / group});
    kernel::matmul_quant_kernel_cu(in, w, out, group, sc, zp, stream);
}

// src/op/kernels/cuda/matmul_kernel.cu:146-199 (FP32 or BF16 weights).
void ref_matmul_cu(const float* x, const void* w, int bf16, float scale, float* y, int rows,
                   int n, int k, void* stream) {
    Tensor in = gpu(x, DataType::Fp32, vec_or_mat(rows, k));
    Tensor wt = gpu(w, bf16 ? DataType::Bf16 : DataType::Fp32, {n, k});
    Tensor out = gpu(y, DataType::Fp32, vec_or_mat(rows, n));
    kernel::matmul_kernel_cu(in, wt, scale, out, stream);
}

// src/op/kernels/cuda/rmsnorm_kernel.cu:152-201.
void ref_rmsnorm_cu(const float* x, const float* w, float* y, int rows, int width, int per_row,
                    float eps, void* stream) {
    Tensor in = gpu(x, DataType::Fp32, vec_or_mat(rows, width));
    Tensor wt = gpu(w, DataType::Fp32, {per_row ? width : rows * width});
    Tensor out = gpu(y, DataType::Fp32, vec_or_mat(rows, width));
    if (per_row) kernel::rmsnorm_kernel_cu_dim(in, wt, out, eps, stream);
    else kernel::rmsnorm_kernel_cu(in, wt, out, eps, stream);
}

// src/op/kernels/cuda/rope_kernel.cu:11-105.
void ref_rope_cache_cu(int head, int max_seq, float theta, float* sin_c, float* cos_c,
                       void* stream) {
    Tensor s = gpu(sin_c, DataType::Fp32, {max_seq, head / 2});
    Tensor c = gpu(cos_c, DataType::Fp32, {max_seq, head / 2});
    kernel::sin_cos_cache_kernel_cu(head, max_seq, theta, s, c, stream);
}
void ref_rope_cu(float* q, float* k, const float* cos_c, const float* sin_c, int q_heads,
                 int k_heads, int head, int max_seq, int pos, void* stream) {
    Tensor tq = gpu(q, DataType::Fp32, {q_heads, head});
    Tensor tk = gpu(k, DataType::Fp32, {k_heads, head});
    Tensor c = gpu(cos_c, DataType::Fp32, {max_seq, head / 2});
    Tensor s = gpu(sin_c, DataType::Fp32, {max_seq, head / 2});
    kernel::rope_kernel_cu(tq, tk, c, s, pos, stream);
}

// src/op/kernels/cuda/mha_kernel.cu:104-144.
void ref_mha_cu(const float* q, const float* kc, const float* vc, float* score, float* out,
                int layers, int capacity, int q_heads, int kv_heads, int head, int layer, int pos,
                void* stream) {
    Tensor tq = gpu(q, DataType::Fp32, {q_heads, head});
    Tensor k = gpu(kc, DataType::Fp32, {layers, capacity, kv_heads, head});
    Tensor v = gpu(vc, DataType::Fp32, {layers, capacity, kv_heads, head});
    Tensor sc = gpu(score, DataType::Fp32, {q_heads, capacity});
    Tensor o = gpu(out, DataType::Fp32, {q_heads, head});
    kernel::mha_kernel_cu(tq, k, v, sc, o, layer, pos, stream);
}

// src/op/kernels/cuda/emb_kernel.cu:64-86.
void ref_embedding_cu(const int32_t* tokens, int count, const void* table, int bf16, int vocab,
                      int dim, float* out, void* stream) {
    Tensor t = gpu(tokens, DataType::Int32, {count});
    Tensor w = gpu(table, bf16 ? DataType::Bf16 : DataType::Fp32, {vocab, dim});
    Tensor o = gpu(out, DataType::Fp32, vec_or_mat(count, dim));
    kernel::emb_kernel_cu(t, w, o, stream);
}

// src/op/kernels/cuda/swiglu_kernel.cu:15-28 and add_kernel.cu:12-31.
void ref_swiglu_cu(const float* g, const float* u, float* o, int n, void* stream) {
    Tensor a = gpu(g, DataType::Fp32, {n}), b = gpu(u, DataType::Fp32, {n});
    Tensor c = gpu(o, DataType::Fp32, {n});
    kernel::swiglu_kernel_cu(a, b, c, stream);
}
void ref_add_cu(const float* x, const float* y, float* o, int n, void* stream) {
    Tensor a = gpu(x, DataType::Fp32, {n}), b = gpu(y, DataType::Fp32, {n});
    Tensor c = gpu(o, DataType::Fp32, {n});
    kernel::add_kernel_cu(a, b, c, stream);
}

// src/op/kernels/cuda/argmax_kernel.cu:39-61 (allocates, synchronises).
int64_t ref_argmax_cu(const float* x, int64_t n, void* stream) {
    return static_cast<int64_t>(kernel::argmax_kernel_cu(x, static_cast<size_t>(n), stream));
}

// CPU kernels: src/op/kernels/cpu/{rmsnorm,rope,mha,softmax}_kernel.cpp.
void ref_rmsnorm_cpu(const float* x, const float* w, float* y, int rows, int width, int per_row,
                     float eps) {
    Tensor in = cpu(x, DataType::Fp32, vec_or_mat(rows, width));
    Tensor wt = cpu(w, DataType::Fp32, {per_row ? width : rows * width});
    Tensor out = cpu(y, DataType::Fp32, vec_or_mat(rows, width));
    if (per_row) kernel::rmsnorm_kernel_cpu_dim(in, wt, out, eps, nullptr);
    else kernel::rmsnorm_kernel_cpu(in, wt, out, eps, nullptr);
}
void ref_rope_cache_cpu(int head, int max_seq, float theta, float* sin_c, float* cos_c) {
    Tensor s = cpu(sin_c, DataType::Fp32, {max_seq, head / 2});
    Tensor c = cpu(cos_c, DataType::Fp32, {max_seq, head / 2});
    kernel::sin_cos_cache_kernel_cpu(head, max_seq, theta, s, c, nullptr);
}
void ref_rope_cpu(float* q, float* k, const float* cos_c, const float* sin_c, int q_heads,
                  int k_heads, int head, int max_seq, int pos) {
    Tensor tq = cpu(q, DataType::Fp32, {q_heads, head});
    Tensor tk = cpu(k, DataType::Fp32, {k_heads, head});
    Tensor c = cpu(cos_c, DataType::Fp32, {max_seq, head / 2});
    Tensor s = cpu(sin_c, DataType::Fp32, {max_seq, head / 2});
    kernel::rope_kernel_cpu(tq, tk, c, s, pos, nullptr);
}
void ref_mha_cpu(const float* q, const float* kc, const float* vc, float* score, float* out,
                 int layers, int capacity, int q_heads, int kv_heads, int head, int layer,
                 int pos) {
    Tensor tq = cpu(q, DataType::Fp32, {q_heads, head});
    Tensor k = cpu(kc, DataType::Fp32, {layers, capacity, kv_heads, head});
    Tensor v = cpu(vc, DataType::Fp32, {layers, capacity, kv_heads, head});
    Tensor sc = cpu(score, DataType::Fp32, {q_heads, capacity});
    Tensor o = cpu(out, DataType::Fp32, {q_heads, head});
    kernel::mha_kernel_cpu(tq, k, v, sc, o, layer, pos, nullptr);
}
void ref_softmax_cpu(float* x, int n) {
    Tensor t = cpu(x, DataType::Fp32, {n});
    kernel::softmax_kernel_cpu(t, t, nullptr);
}

}  // extern "C"
