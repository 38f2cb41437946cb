// tinym_torch_op.cpp -- torch custom-op shim over the C ABI.
//
// Registers the reference's op namespace and schema
// (src/torch_candidate_extension.cu:85-91):
//     sm120_fp8_gemm::run(Tensor a, Tensor b, float alpha) -> Tensor
// plus a device-alpha form used by candidate_kernel.fp8_gemm:
//     sm120_fp8_gemm::run_alpha_tensor(Tensor a, Tensor b, Tensor alpha) -> Tensor
// and the packed-weight pair behind candidate_kernel.prepare_weights'
// optional repack (tinym_pack_weights / tinym_fp8_gemm_packed):
//     sm120_fp8_gemm::pack_weights(Tensor b) -> Tensor            (uint8, packed layout)
//     sm120_fp8_gemm::run_packed(Tensor a, Tensor b_packed, int n, int k, Tensor alpha) -> Tensor
// and the fused activation path (tinym_fp8_gemm_quant_act): a BF16 / FP32
// activation quantised per tensor on the device, then the GEMM:
//     sm120_fp8_gemm::run_quant_act(Tensor x, Tensor b, Tensor w_scale) -> (Tensor y, Tensor x_scale)
// Input checks mirror check_inputs (src/torch_candidate_extension.cu:17-31)
// and raise the same RuntimeError (TORCH_CHECK) messages; every op also
// raises before launching if an earlier GEMM on the device ran out of a
// bounded wait (tinym_pending_errors).  Shape support is
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

// A GEMM whose bounded device wait ran out left its output unspecified; the
// kernel posted that to the device's pending-error word, which is checked
// (without synchronising) before every launch, so the caller gets a
// RuntimeError here instead of using that output silently.  The word is
// cleared, so the call after this one runs normally.  Needs the operands'
// device current.
void check_pending() {
    uint32_t flags = 0;
    const int st = tinym_pending_errors(&flags, 1);
    TORCH_CHECK(st == TINYM_OK || st == TINYM_ERR_DEVICE_TIMEOUT, tinym_status_string(st), ": ",
                tinym_last_error());
    TORCH_CHECK(flags == 0u, "TINYM_ERR_DEVICE_TIMEOUT: ", tinym_last_error());
}

at::Tensor launch(const at::Tensor& a, const at::Tensor& b, const float* alpha_dev, float alpha) {
    const int64_t m = a.size(0), k = a.size(1), n = b.size(0);
    const c10::cuda::CUDAGuard guard(a.device());
    check_pending();
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

at::Tensor pack_weights(const at::Tensor& b) {
    TORCH_CHECK(b.is_cuda(), "B must be a CUDA tensor");
    TORCH_CHECK(b.dim() == 2 && b.is_contiguous(), "B must be a contiguous rank-2 tensor");
    TORCH_CHECK(b.scalar_type() == at::ScalarType::Float8_e4m3fn,
                "B must have dtype torch.float8_e4m3fn");
    const int64_t n = b.size(0), k = b.size(1);
    int64_t bytes = 0;
    raise_status(tinym_packed_weight_bytes(n, k, &bytes));
    const c10::cuda::CUDAGuard guard(b.device());
    at::Tensor out = at::empty({bytes}, b.options().dtype(at::ScalarType::Byte));
    raise_status(tinym_pack_weights(b.data_ptr(), out.data_ptr(), n, k,
                                    at::cuda::getCurrentCUDAStream(b.get_device())));
    return out;
}

at::Tensor run_packed(const at::Tensor& a, const at::Tensor& bp, int64_t n, int64_t k,
                      const at::Tensor& alpha) {
    TORCH_CHECK(a.is_cuda() && bp.is_cuda(), "A and B must be CUDA tensors");
    TORCH_CHECK(a.get_device() == bp.get_device(), "A and B must be on the same CUDA device");
    TORCH_CHECK(a.dim() == 2 && a.is_contiguous(), "A must be a contiguous rank-2 tensor");
    TORCH_CHECK(a.scalar_type() == at::ScalarType::Float8_e4m3fn,
                "A must have dtype torch.float8_e4m3fn");
    TORCH_CHECK(a.size(1) == k, "A and B must have the same K dimension");
    TORCH_CHECK(bp.scalar_type() == at::ScalarType::Byte && bp.dim() == 1 && bp.is_contiguous(),
                "B_packed must be the uint8 tensor returned by pack_weights");
    int64_t bytes = 0;
    raise_status(tinym_packed_weight_bytes(n, k, &bytes));
    TORCH_CHECK(bp.numel() == bytes, "B_packed has ", bp.numel(), " bytes, packed [", n, ", ",
                k, "] needs ", bytes);
    TORCH_CHECK(alpha.is_cuda() && alpha.scalar_type() == at::ScalarType::Float &&
                    alpha.numel() == 1,
                "alpha must be a one-element CUDA float32 tensor");
    TORCH_CHECK(alpha.get_device() == a.get_device(), "alpha must be on A's device");
    const int64_t m = a.size(0);
    const c10::cuda::CUDAGuard guard(a.device());
    check_pending();
    at::Tensor y = at::empty({m, n}, a.options().dtype(at::ScalarType::BFloat16));
    if (m == 0 || n == 0) return y;
    raise_status(tinym_fp8_gemm_packed(a.data_ptr(), bp.data_ptr(), y.data_ptr(), n, m, n, k,
                                       alpha.data_ptr<float>(), 0.0f, nullptr,
                                       at::cuda::getCurrentCUDAStream(a.get_device())));
    return y;
}

std::tuple<at::Tensor, at::Tensor> run_quant_act(const at::Tensor& x, const at::Tensor& b,
                                                 const at::Tensor& w_scale) {
    TORCH_CHECK(x.is_cuda() && b.is_cuda() && w_scale.is_cuda(), "X, B and w_scale must be CUDA tensors");
    TORCH_CHECK(x.get_device() == b.get_device() && w_scale.get_device() == b.get_device(),
                "X, B and w_scale must be on the same CUDA device");
    TORCH_CHECK(x.dim() == 2 && b.dim() == 2, "X and B must both be rank-2 tensors");
    TORCH_CHECK(x.is_contiguous() && b.is_contiguous(), "X and B must be contiguous row-major tensors");
    TORCH_CHECK(x.scalar_type() == at::ScalarType::BFloat16 || x.scalar_type() == at::ScalarType::Float,
                "X must have dtype torch.bfloat16 or torch.float32");
    TORCH_CHECK(b.scalar_type() == at::ScalarType::Float8_e4m3fn, "B must have dtype torch.float8_e4m3fn");
    TORCH_CHECK(x.size(1) == b.size(1), "X and B must have the same K dimension");
    TORCH_CHECK(w_scale.scalar_type() == at::ScalarType::Float && w_scale.numel() == 1,
                "w_scale must be a one-element float32 tensor");
    const int64_t m = x.size(0), k = x.size(1), n = b.size(0);
    const c10::cuda::CUDAGuard guard(x.device());
    check_pending();
    at::Tensor y = at::empty({m, n}, b.options().dtype(at::ScalarType::BFloat16));
    int64_t ws_bytes = 0;
    raise_status(tinym_quant_workspace_bytes(m, k, &ws_bytes));
    at::Tensor ws = at::empty({ws_bytes}, b.options().dtype(at::ScalarType::Byte));
    const int dt = x.scalar_type() == at::ScalarType::BFloat16 ? TINYM_ACT_BF16 : TINYM_ACT_F32;
    raise_status(tinym_fp8_gemm_quant_act(x.data_ptr(), dt, b.data_ptr(), w_scale.data_ptr<float>(),
                                          y.data_ptr(), n, m, n, k, ws.data_ptr(), nullptr,
                                          at::cuda::getCurrentCUDAStream(x.get_device())));
    // x_scale is the workspace's first float (a view keeps the workspace alive).
    return {y, ws.narrow(0, 0, 4).view(at::ScalarType::Float)};
}

}  // namespace

TORCH_LIBRARY(sm120_fp8_gemm, module) {
    module.def("run(Tensor a, Tensor b, float alpha) -> Tensor");
    module.def("run_alpha_tensor(Tensor a, Tensor b, Tensor alpha) -> Tensor");
    module.def("pack_weights(Tensor b) -> Tensor");
    module.def("run_packed(Tensor a, Tensor b_packed, int n, int k, Tensor alpha) -> Tensor");
    module.def("run_quant_act(Tensor x, Tensor b, Tensor w_scale) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(sm120_fp8_gemm, CUDA, module) {
    module.impl("run", &run_host_alpha);
    module.impl("run_alpha_tensor", &run_alpha_tensor);
    module.impl("pack_weights", &pack_weights);
    module.impl("run_packed", &run_packed);
    module.impl("run_quant_act", &run_quant_act);
}
