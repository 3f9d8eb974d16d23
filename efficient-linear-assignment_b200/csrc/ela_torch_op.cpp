// ela_torch_op.cpp -- the solve as a C++ torch operator over the C ABI.
//
// torch.ops.ela_native.auction_solve(cost, eps, max_iter, path, tie_rule)
//   -> (assignment int64 (B,N), prices (B,M), stats int64 (B,4), status int32 (1,), rc)
// rc is the library's return code (ELA_OK once the work is enqueued): a status
// is returned, not thrown, and the Python wrapper raises AuctionError with it;
// only malformed calls (not CUDA, not (B,N,M), unknown dtype) raise here.
// The reference binds its CUDA solver through a pybind11 function
// (src/csrc/interface.cpp:4,64); this is the same boundary as a registered
// operator: device guard on the cost's device, argument checks that raise,
// outputs and workspace from the caching allocator, one ela_auction_solve call
// on the current stream, no synchronisation (the device status word is read
// by the caller).
#include <torch/library.h>
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <tuple>
#include <vector>

#include "ela_auction.h"

namespace {

int dtype_code(at::ScalarType t) {
    switch (t) {
    case at::kFloat: return ELA_DTYPE_F32;
    case at::kHalf: return ELA_DTYPE_F16;
    case at::kBFloat16: return ELA_DTYPE_BF16;
    case at::kDouble: return ELA_DTYPE_F64;
    default: return -1;
    }
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t> auction_solve_cuda(const at::Tensor& cost_in,
                                                                             std::vector<double> eps,
                                                                             int64_t max_iter, int64_t path,
                                                                             int64_t tie_rule) {
    TORCH_CHECK(cost_in.is_cuda(), "ela_native::auction_solve needs a CUDA tensor (there is no CPU path)");
    TORCH_CHECK(cost_in.dim() == 3, "cost must be (B, N, M)");
    const int code = dtype_code(cost_in.scalar_type());
    TORCH_CHECK(code >= 0, "unsupported cost dtype ", cost_in.scalar_type());
    TORCH_CHECK(!eps.empty(), "epsilon schedule is empty");
    c10::cuda::CUDAGuard guard(cost_in.device());
    const at::Tensor cost = cost_in.stride(2) == 1 ? cost_in : cost_in.contiguous();
    const int64_t B = cost.size(0), N = cost.size(1), M = cost.size(2);
    const auto dev = cost.device();
    const auto pdt = code == ELA_DTYPE_F64 ? at::kDouble : at::kFloat;
    at::Tensor assign = at::empty({B, N}, at::TensorOptions().dtype(at::kLong).device(dev));
    at::Tensor prices = at::empty({B, M}, at::TensorOptions().dtype(pdt).device(dev));
    at::Tensor stats = at::empty({B, 4}, at::TensorOptions().dtype(at::kLong).device(dev));
    at::Tensor status = at::empty({1}, at::TensorOptions().dtype(at::kInt).device(dev));
    if (B == 0 || N == 0) {
        prices.zero_();
        stats.zero_();
        status.zero_();
        return {assign, prices, stats, status, (int64_t)ELA_OK};
    }
    const size_t ws_bytes = ela_auction_workspace_bytes(code, B, N, M, (int)path);
    if (ws_bytes == 0) return {assign, prices, stats, status, (int64_t)(M >= 2 ? ELA_ERR_UNSUPPORTED : ELA_ERR_ARGUMENT)};
    at::Tensor ws = at::empty({(int64_t)ws_bytes}, at::TensorOptions().dtype(at::kByte).device(dev));
    const int rc = ela_auction_solve(cost.data_ptr(), code, B, N, M, cost.stride(0), cost.stride(1), eps.data(),
                                     (int)eps.size(), (int)max_iter, (int)path, (int)tie_rule,
                                     assign.data_ptr<int64_t>(), prices.data_ptr(), stats.data_ptr<int64_t>(),
                                     status.data_ptr<int32_t>(), ws.data_ptr(), ws_bytes,
                                     c10::cuda::getCurrentCUDAStream(dev.index()).stream());
    return {assign, prices, stats, status, (int64_t)rc};
}

}  // namespace

TORCH_LIBRARY(ela_native, m) {
    m.def("auction_solve(Tensor cost, float[] eps, int max_iter, int path, int tie_rule) -> "
          "(Tensor, Tensor, Tensor, Tensor, int)");
}

TORCH_LIBRARY_IMPL(ela_native, CUDA, m) { m.impl("auction_solve", &auction_solve_cuda); }
