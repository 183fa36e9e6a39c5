// TEST INFRASTRUCTURE ONLY: the reference's own LinearOp::forward (src/op/linear.cpp:11-36),
// compiled from its sources by oracle/Makefile `boundary`, with its CUDA kernel dispatch
// (src/op/kernels/kernels_interface.cpp) bound to fire_b200 through the shims a Fire
// maintainer would add. It proves the drop-in boundary end to
// end: Fire's operator validation and Tensor/Parameter types on one side, the fire_b200
// C ABI (libfire_b200.so, linked) on the other. Nothing here is part of the product.
#include "Fire/base/base.h"
#include "Fire/op/linear.h"
#include "Fire/op/operator.h"
#include "Fire/tensor/tensor.h"
#include "fire_b200.h"
#include "kernels_interface.h"

#include <cstdint>
#include <vector>

namespace {

// the last fire_b200 status a shim saw (Fire's kernel signatures return void);
// kNotCalled until a shim runs
constexpr int kNotCalled = -1000;
thread_local int g_last_rc = kNotCalled;

// src/op/kernels/cuda/matmul_kernel.cu:280-314, replaced
void matmul_quant_kernel_cu(const tensor::Tensor& in, const tensor::Tensor& qw, tensor::Tensor& out,
                            int32_t group_size, const tensor::Tensor& scales, const tensor::Tensor& zero_points,
                            void* stream) {
    const int rows = in.dims_size() == 1 ? 1 : in.get_dim(0);
    const int k = in.get_dim(in.dims_size() - 1);
    g_last_rc = fire_b200_linear_w4(in.ptr<float>(), qw.ptr<uint8_t>(), scales.ptr<float>(),
                                    zero_points.ptr<uint8_t>(), out.ptr<float>(), rows, qw.get_dim(0), k, group_size,
                                    stream);
    CHECK(g_last_rc == FIRE_B200_OK) << fire_b200_status_string(g_last_rc);
}

// src/op/kernels/cuda/matmul_kernel.cu:146-199, replaced (FP32 or BF16 weights)
void matmul_kernel_cu(const tensor::Tensor& in, const tensor::Tensor& w, float scale, tensor::Tensor& out,
                      void* stream) {
    const int rows = in.dims_size() == 1 ? 1 : in.get_dim(0);
    const int dt = w.data_type() == base::DataType::Bf16 ? FIRE_B200_BF16 : FIRE_B200_F32;
    g_last_rc = fire_b200_linear_dense(in.ptr<float>(), w.ptr<void>(), dt, scale, out.ptr<float>(), rows,
                                       w.get_dim(0), w.get_dim(1), stream);
    CHECK(g_last_rc == FIRE_B200_OK) << fire_b200_status_string(g_last_rc);
}

// src/op/kernels/cuda/add_kernel.cu:12-31, replaced
void add_kernel_cu(const tensor::Tensor& a, const tensor::Tensor& b, tensor::Tensor& out, void* stream) {
    g_last_rc = fire_b200_add(a.ptr<float>(), b.ptr<float>(), out.ptr<float>(), static_cast<int>(a.size()), stream);
    CHECK(g_last_rc == FIRE_B200_OK) << fire_b200_status_string(g_last_rc);
}

tensor::Tensor gpu(const void* p, base::DataType t, std::vector<int32_t> d) {
    return tensor::Tensor::from_blob(const_cast<void*>(p), t, std::move(d), base::DeviceType::GPU);
}
std::vector<int32_t> vec_or_mat(int rows, int cols) {
    return rows == 1 ? std::vector<int32_t>{cols} : std::vector<int32_t>{rows, cols};
}

}  // namespace

// The three getters LinearOp::forward reaches (kernels_interface.h:46-66), GPU only here.
namespace kernel {
MatmulKernelQuant get_matmul_quant_kernel(base::DeviceType) { return matmul_quant_kernel_cu; }
MatmulKernel get_matmul_kernel(base::DeviceType) { return matmul_kernel_cu; }
AddKernel get_add_kernel(base::DeviceType) { return add_kernel_cu; }
}  // namespace kernel

extern "C" {

// Fire's LinearOp with an Int4GroupWise Parameter on GPU tensors viewing the caller's device
// pointers: returns LinearOp::forward's StatusCode (0 = Success); *kernel_rc receives the
// fire_b200 status the shim saw, or -1000 when no kernel was called.
int boundary_linear_w4(const float* x, const uint8_t* qw, const float* s, const uint8_t* z, float* y, int rows,
                       int n, int k, int group, void* stream, int* kernel_rc) {
    op::LinearOp linear;
    linear.reset_param_size(1);
    op::Parameter& p = linear.get_param(0);
    p._data = gpu(qw, base::DataType::UInt8, {n, k / 2});
    p._scales = gpu(s, base::DataType::Fp32, {n, k / group});
    p._zero_points = gpu(z, base::DataType::UInt8, {n, k / group});
    p._quant_config._quant_type = op::QuantType::Int4GroupWise;
    p._quant_config._group_size = group;
    p._quant_config._symmetric = false;
    tensor::Tensor in = gpu(x, base::DataType::Fp32, vec_or_mat(rows, k));
    tensor::Tensor out = gpu(y, base::DataType::Fp32, vec_or_mat(rows, n));
    op::OpContext ctx;
    ctx._device_type = base::DeviceType::GPU;
    ctx._stream = static_cast<cudaStream_t>(stream);
    g_last_rc = kNotCalled;
    const base::Status st = linear.forward(in, out, ctx);
    if (kernel_rc) *kernel_rc = g_last_rc;
    return static_cast<int>(st.code());
}

// The same with a BF16 (bf16 != 0) or FP32 weight [n, k] and scale (the LM head at M = 1).
int boundary_linear_dense(const float* x, const void* w, int bf16, float scale, float* y, int rows, int n, int k,
                          void* stream, int* kernel_rc) {
    op::LinearOp linear(scale);
    linear.reset_param_size(1);
    linear.get_param(0)._data = gpu(w, bf16 ? base::DataType::Bf16 : base::DataType::Fp32, {n, k});
    tensor::Tensor in = gpu(x, base::DataType::Fp32, vec_or_mat(rows, k));
    tensor::Tensor out = gpu(y, base::DataType::Fp32, vec_or_mat(rows, n));
    op::OpContext ctx;
    ctx._device_type = base::DeviceType::GPU;
    ctx._stream = static_cast<cudaStream_t>(stream);
    g_last_rc = kNotCalled;
    const base::Status st = linear.forward(in, out, ctx);
    if (kernel_rc) *kernel_rc = g_last_rc;
    return static_cast<int>(st.code());
}

}  // extern "C"
