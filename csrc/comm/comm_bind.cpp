// Python bindings of the fused communication kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "comm.h"

namespace {

ArPeers make_peers(const std::vector<int64_t>& bases, int64_t rank, int64_t max_t) {
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kArMaxRanks, "1..8 ranks");
  ArPeers p{};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  p.rank = rank;
  p.world = bases.size();
  p.max_t = max_t;
  return p;
}

template <typename T>
T* optr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void ar_push(const at::Tensor& x, std::vector<int64_t> bases, int64_t rank, int64_t max_t, const at::Tensor& epoch,
             at::Tensor ticket, int64_t nctas) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x bf16 [T,H]");
  const c10::cuda::CUDAGuard g(x.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_ar_push(x.data_ptr(), x.size(0), x.size(1), &p, reinterpret_cast<const uint32_t*>(epoch.data_ptr()),
                              reinterpret_cast<uint32_t*>(ticket.data_ptr()), nctas,
                              at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "ar_push failed ", rc);
}

void ar_reduce_norm(int64_t T, int64_t hidden, std::vector<int64_t> bases, int64_t rank, int64_t max_t,
                    at::Tensor epoch, at::Tensor ticket, int64_t push_ctas, at::Tensor residual, const at::Tensor& w,
                    double eps, c10::optional<at::Tensor> y, c10::optional<at::Tensor> q,
                    c10::optional<at::Tensor> sf, at::Tensor err) {
  TORCH_CHECK(residual.is_cuda() && residual.scalar_type() == at::kFloat && residual.is_contiguous(), "residual fp32");
  const c10::cuda::CUDAGuard g(residual.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_ar_reduce_norm(T, hidden, &p, reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                     reinterpret_cast<uint32_t*>(ticket.data_ptr()), push_ctas,
                                     reinterpret_cast<float*>(residual.data_ptr()),
                                     reinterpret_cast<const float*>(w.data_ptr()), eps, optr<void>(y), optr<uint8_t>(q),
                                     optr<uint8_t>(sf), reinterpret_cast<uint32_t*>(err.data_ptr()),
                                     at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "ar_reduce_norm failed ", rc);
}

void moe_combine_push(const at::Tensor& y, const at::Tensor& pair_row, c10::optional<at::Tensor> add,
                      std::vector<int64_t> bases, int64_t rank, int64_t max_t, const at::Tensor& epoch,
                      at::Tensor ticket, int64_t nctas) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous(), "y bf16");
  TORCH_CHECK(pair_row.scalar_type() == at::kInt && pair_row.is_contiguous(), "pair_row int32 [T,K]");
  if (add.has_value()) TORCH_CHECK(add->scalar_type() == at::kBFloat16 && add->is_contiguous(), "add bf16 [T,H]");
  const c10::cuda::CUDAGuard g(y.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_moe_combine_push(y.data_ptr(), reinterpret_cast<const int*>(pair_row.data_ptr()), pair_row.size(0),
                                       pair_row.size(1), y.size(1), optr<void>(add), &p,
                                       reinterpret_cast<const uint32_t*>(epoch.data_ptr()),
                                       reinterpret_cast<uint32_t*>(ticket.data_ptr()), nctas,
                                       at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "moe_combine_push failed ", rc);
}

int64_t ar_buffer_size(int64_t world, int64_t max_t, int64_t hidden) { return ar_buffer_bytes(world, max_t, hidden); }

}  // namespace

void register_comm(pybind11::module& m) {
  m.def("ar_push", &ar_push);
  m.def("ar_reduce_norm", &ar_reduce_norm);
  m.def("ar_buffer_size", &ar_buffer_size);
  m.def("moe_combine_push", &moe_combine_push);
}
