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

void mla_q_quant(const at::Tensor& q_abs, const at::Tensor& q_pe, at::Tensor q8, at::Tensor qs) {
  TORCH_CHECK(q_abs.is_contiguous() && q_pe.is_contiguous() && q_abs.scalar_type() == at::kBFloat16, "bf16 q");
  TORCH_CHECK(q_abs.size(-1) == 512 && q_pe.size(-1) == 64, "latent 512 + rope 64");
  const c10::cuda::CUDAGuard g(q_abs.device());
  const int TH = q_abs.numel() / 512;
  TORCH_CHECK(b200_mla_q_quant(q_abs.data_ptr(), q_pe.data_ptr(), TH, reinterpret_cast<uint8_t*>(q8.data_ptr()),
                               reinterpret_cast<float*>(qs.data_ptr()), at::cuda::getCurrentCUDAStream().stream()) == 0,
              "mla_q_quant failed");
}

void mla_tc(const at::Tensor& q8, const at::Tensor& qs, const at::Tensor& cache, double kv_scale,
            const at::Tensor& block_table, const at::Tensor& q_seq, const at::Tensor& q_pos, int64_t page_size,
            double sm_scale, int64_t nsplit, at::Tensor out, c10::optional<at::Tensor> part_o,
            c10::optional<at::Tensor> part_lse) {
  TORCH_CHECK(q8.is_cuda() && q8.dim() == 3 && q8.size(2) == 576 && q8.is_contiguous(), "q8 e4m3 [T,H,576]");
  TORCH_CHECK(cache.dim() == 2 && cache.size(1) == 576 && cache.is_contiguous(), "cache [slots, 576]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && q_seq.scalar_type() == at::kInt && q_pos.scalar_type() == at::kInt,
              "int32 metadata");
  const c10::cuda::CUDAGuard g(q8.device());
  MlaTcArgs a{};
  a.q8 = reinterpret_cast<const uint8_t*>(q8.data_ptr());
  a.q_scale = reinterpret_cast<const float*>(qs.data_ptr());
  a.cache = reinterpret_cast<const uint8_t*>(cache.data_ptr());
  a.cache_rows = cache.size(0);
  a.block_table = reinterpret_cast<const int*>(block_table.data_ptr());
  a.bt_stride = block_table.stride(0);
  a.q_seq = reinterpret_cast<const int*>(q_seq.data_ptr());
  a.q_pos = reinterpret_cast<const int*>(q_pos.data_ptr());
  a.T = q8.size(0);
  a.H = q8.size(1);
  a.page_size = page_size;
  a.nsplit = nsplit;
  a.sm_scale = sm_scale;
  a.kv_scale = kv_scale;
  a.out = out.data_ptr();
  if (nsplit > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split partial buffers");
    a.part_o = reinterpret_cast<float*>(part_o->data_ptr());
    a.part_lse = reinterpret_cast<float*>(part_lse->data_ptr());
  }
  const int rc = b200_mla_tc(&a, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "mla_tc failed ", rc);
}

}  // namespace

void register_attn(pybind11::module& m) {
  m.def("mla_simt", &mla_simt);
  m.def("mla_q_quant", &mla_q_quant);
  m.def("mla_tc", &mla_tc);
}
