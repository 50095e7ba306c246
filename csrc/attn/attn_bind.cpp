// Python bindings of the attention kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attn.h"

namespace {

void mla_simt(const at::Tensor& q_abs, const at::Tensor& q_pe, const at::Tensor& cache, double kv_scale,
              const at::Tensor& block_table, const at::Tensor& q_seq, const at::Tensor& q_pos,
              c10::optional<at::Tensor> topk, int64_t page_size, double sm_scale, at::Tensor out) {
  TORCH_CHECK(q_abs.is_cuda() && q_abs.scalar_type() == at::kBFloat16 && q_abs.is_contiguous(), "q_abs bf16 [T,H,L]");
  TORCH_CHECK(q_pe.scalar_type() == at::kBFloat16 && q_pe.is_contiguous(), "q_pe bf16 [T,H,R]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && q_seq.scalar_type() == at::kInt && q_pos.scalar_type() == at::kInt,
              "int32 metadata");
  const c10::cuda::CUDAGuard g(q_abs.device());
  const int T = q_abs.size(0), H = q_abs.size(1), L = q_abs.size(2), R = q_pe.size(2);
  const int* tk = nullptr;
  int tn = 0;
  if (topk.has_value() && topk->defined()) {
    TORCH_CHECK(topk->scalar_type() == at::kInt && topk->is_contiguous(), "topk int32");
    tk = reinterpret_cast<const int*>(topk->data_ptr());
    tn = topk->size(1);
  }
  const int rc = b200_mla_simt(q_abs.data_ptr(), q_pe.data_ptr(), T, H, L, R,
                               reinterpret_cast<const uint8_t*>(cache.data_ptr()), float(kv_scale),
                               reinterpret_cast<const int*>(block_table.data_ptr()), block_table.stride(0),
                               reinterpret_cast<const int*>(q_seq.data_ptr()), reinterpret_cast<const int*>(q_pos.data_ptr()),
                               tk, tn, page_size, float(sm_scale), out.data_ptr(), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "mla_simt failed ", rc);
}

}  // namespace

void register_attn(pybind11::module& m) { m.def("mla_simt", &mla_simt); }
