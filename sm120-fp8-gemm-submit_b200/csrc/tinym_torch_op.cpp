// tinym_torch_op.cpp -- torch custom-op shim over the C ABI.
//
// Registers the reference's op namespace and schema
// (src/torch_candidate_extension.cu:85-91):
//     sm120_fp8_gemm::run(Tensor a, Tensor b, float alpha) -> Tensor
// plus a device-alpha form used by candidate_kernel.fp8_gemm:
//     sm120_fp8_gemm::run_alpha_tensor(Tensor a, Tensor b, Tensor alpha) -> Tensor
// Input checks mirror check_inputs (src/torch_candidate_extension.cu:17-31)
// and raise the same RuntimeError (TORCH_CHECK) messages; shape support is
// decided by the C ABI (1 <= M <= 16, K % 16 == 0) instead of the six-point
// gate of :40-46.  Y is allocated by the op (as in :49-50) and the kernel is
// launched on the current stream of A's device (:48,:57).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/util/Exception.h>
#include <torch/library.h>

#include <cmath>

#include "../../include/tinym_b200.h"

namespace {

void check_inputs(const at::Tensor& a, const at::Tensor& b) {
    TORCH_CHECK(a.is_cuda() && b.is_cuda(), "A and B must be CUDA tensors");
    TORCH_CHECK(a.get_device() == b.get_device(), "A and B must be on the same CUDA device");
    TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "A and B must both be rank-2 tensors");
    TORCH_CHECK(a.is_contiguous() && b.is_contiguous(), "A and B must be contiguous row-major tensors");
    TORCH_CHECK(a.scalar_type() == at::ScalarType::Float8_e4m3fn &&
                    b.scalar_type() == at::ScalarType::Float8_e4m3fn,
                "A and B must have dtype torch.float8_e4m3fn");
    TORCH_CHECK(a.size(1) == b.size(1), "A and B must have the same K dimension");
}

void raise_status(int st) {
    TORCH_CHECK(st == TINYM_OK, tinym_status_string(st), ": ", tinym_last_error());
}

at::Tensor launch(const at::Tensor& a, const at::Tensor& b, const float* alpha_dev, float alpha) {
    const int64_t m = a.size(0), k = a.size(1), n = b.size(0);
    const c10::cuda::CUDAGuard guard(a.device());
    at::Tensor y = at::empty({m, n}, a.options().dtype(at::ScalarType::BFloat16));
    if (m == 0 || n == 0) return y;
    cudaStream_t stream = at::cuda::getCurrentCUDAStream(a.get_device());
    const int st = tinym_fp8_gemm_ex(a.data_ptr(), b.data_ptr(), y.data_ptr(), n, m, n, k,
                                     alpha_dev, alpha, nullptr, stream);
    raise_status(st);
    return y;
}

at::Tensor run_host_alpha(const at::Tensor& a, const at::Tensor& b, double alpha) {
    check_inputs(a, b);
    TORCH_CHECK(std::isfinite(alpha), "alpha must be finite");
    return launch(a, b, nullptr, static_cast<float>(alpha));
}

at::Tensor run_alpha_tensor(const at::Tensor& a, const at::Tensor& b, const at::Tensor& alpha) {
    check_inputs(a, b);
    TORCH_CHECK(alpha.is_cuda() && alpha.scalar_type() == at::ScalarType::Float &&
                    alpha.numel() == 1,
                "alpha must be a one-element CUDA float32 tensor");
    TORCH_CHECK(alpha.get_device() == a.get_device(), "alpha must be on A's device");
    return launch(a, b, alpha.data_ptr<float>(), 0.0f);
}

}  // namespace

TORCH_LIBRARY(sm120_fp8_gemm, module) {
    module.def("run(Tensor a, Tensor b, float alpha) -> Tensor");
    module.def("run_alpha_tensor(Tensor a, Tensor b, Tensor alpha) -> Tensor");
}

TORCH_LIBRARY_IMPL(sm120_fp8_gemm, CUDA, module) {
    module.impl("run", &run_host_alpha);
    module.impl("run_alpha_tensor", &run_alpha_tensor);
}
