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

void mla_q_prep(const at::Tensor& q_abs, const at::Tensor& q_pe, const at::Tensor& pos, const at::Tensor& table,
                at::Tensor q8, at::Tensor qs) {
  TORCH_CHECK(q_abs.is_cuda() && q_abs.dim() == 3 && q_abs.size(2) == 512 && q_abs.stride(2) == 1, "q_abs [T,H,512]");
  TORCH_CHECK(q_pe.dim() == 3 && q_pe.size(2) == 64 && q_pe.stride(2) == 1, "q_pe [T,H,64]");
  TORCH_CHECK(q_abs.scalar_type() == at::kBFloat16 && q_pe.scalar_type() == at::kBFloat16, "bf16");
  TORCH_CHECK(table.size(1) == 64 && pos.scalar_type() == at::kInt, "rope table [P, 64], pos int32");
  const c10::cuda::CUDAGuard g(q_abs.device());
  const int rc = b200_mla_q_prep(q_abs.data_ptr(), q_abs.stride(0), q_abs.stride(1), q_pe.data_ptr(), q_pe.stride(0),
                                 q_pe.stride(1), q_abs.size(0), q_abs.size(1), pos.data_ptr<int>(), table.data_ptr<float>(),
                                 reinterpret_cast<uint8_t*>(q8.data_ptr()), qs.data_ptr<float>(),
                                 at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "mla_q_prep failed ", rc);
}

void mla_tc(const at::Tensor& q8, const at::Tensor& qs, const at::Tensor& cache, double kv_scale,
            const at::Tensor& block_table, const at::Tensor& q_seq, const at::Tensor& q_pos, int64_t page_size,
            double sm_scale, int64_t nsplit, at::Tensor out, c10::optional<at::Tensor> part_o,
            c10::optional<at::Tensor> part_lse, c10::optional<at::Tensor> topk, int64_t hb,
            c10::optional<at::Tensor> lse_out, c10::optional<at::Tensor> cache2, int64_t ratio2) {
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
  a.hb = hb;
  if (lse_out.has_value() && lse_out->defined()) {
    TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->numel() >= (int64_t)a.T * a.H, "lse_out fp32 [T, H]");
    a.lse_out = reinterpret_cast<float*>(lse_out->data_ptr());
  }
  a.sm_scale = sm_scale;
  a.kv_scale = kv_scale;
  a.out = out.data_ptr();
  if (cache2.has_value() && cache2->defined()) {
    TORCH_CHECK(cache2->dim() == 2 && cache2->size(1) == 576 && cache2->is_contiguous() && ratio2 >= 2 &&
                    64 % ratio2 == 0, "cache2 [rows, 576] with ratio2 in 2..64 dividing 64");
    a.cache2 = reinterpret_cast<const uint8_t*>(cache2->data_ptr());
    a.cache2_rows = cache2->size(0);
    a.ratio2 = int(ratio2);
  }
  if (nsplit > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "split partial buffers");
    a.part_o = reinterpret_cast<float*>(part_o->data_ptr());
    a.part_lse = reinterpret_cast<float*>(part_lse->data_ptr());
  }
  if (topk.has_value() && topk->defined()) {
    TORCH_CHECK(topk->scalar_type() == at::kInt && topk->is_contiguous() && topk->dim() == 2 && topk->size(0) == a.T,
                "topk int32 [T, k]");
    a.topk = reinterpret_cast<const int*>(topk->data_ptr());
    a.topk_n = topk->size(1);
  }
  const int rc = b200_mla_tc(&a, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "mla_tc failed ", rc);
}

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }

void ix_k_store(const at::Tensor& k, const at::Tensor& ln_w, const at::Tensor& ln_b, double eps, const at::Tensor& pos,
                const at::Tensor& table, const at::Tensor& slots, at::Tensor cache, at::Tensor scale) {
  TORCH_CHECK(k.is_cuda() && k.dim() == 2 && k.stride(1) == 1 && k.size(1) == 128, "k [T, 128] unit inner stride");
  TORCH_CHECK(k.scalar_type() == at::kBFloat16 || k.scalar_type() == at::kFloat, "k bf16/fp32");
  TORCH_CHECK(slots.scalar_type() == at::kLong && pos.scalar_type() == at::kInt, "slots int64, pos int32");
  TORCH_CHECK(cache.dim() == 2 && cache.size(1) == 128 && cache.is_contiguous(), "cache [slots, 128]");
  const c10::cuda::CUDAGuard g(k.device());
  const int rc = b200_ix_k_store(k.data_ptr(), k.scalar_type() == at::kFloat, k.stride(0), k.size(0),
                                 ln_w.data_ptr<float>(), ln_b.data_ptr<float>(), float(eps), pos.data_ptr<int>(),
                                 table.data_ptr<float>(), table.size(1), slots.data_ptr<int64_t>(),
                                 reinterpret_cast<uint8_t*>(cache.data_ptr()), scale.data_ptr<float>(), cur());
  TORCH_CHECK(rc == 0, "ix_k_store failed ", rc);
}

void ix_q_quant(const at::Tensor& q, const at::Tensor& wraw, int64_t NH, double w_factor, const at::Tensor& pos,
                const at::Tensor& table, at::Tensor q8, at::Tensor wq) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 2 && q.stride(1) == 1 && q.size(1) == NH * 128, "q [T, NH*128]");
  TORCH_CHECK(wraw.dim() == 2 && wraw.stride(1) == 1 && wraw.size(1) == NH, "w [T, NH]");
  TORCH_CHECK(q8.is_contiguous() && q8.numel() == q.size(0) * NH * 128, "q8 [T*NH, 128]");
  const c10::cuda::CUDAGuard g(q.device());
  const int rc = b200_ix_q_quant(q.data_ptr(), q.scalar_type() == at::kFloat, q.stride(0), wraw.data_ptr(),
                                 wraw.scalar_type() == at::kFloat, wraw.stride(0), q.size(0), NH, float(w_factor),
                                 pos.data_ptr<int>(), table.data_ptr<float>(), table.size(1),
                                 reinterpret_cast<uint8_t*>(q8.data_ptr()), wq.data_ptr<float>(), cur());
  TORCH_CHECK(rc == 0, "ix_q_quant failed ", rc);
}

void ix_score(const at::Tensor& q8, const at::Tensor& wq, const at::Tensor& k_cache, const at::Tensor& k_scale,
              const at::Tensor& block_table, const at::Tensor& q_seq, const at::Tensor& q_pos, int64_t page_size,
              int64_t nsplit, at::Tensor scores) {
  TORCH_CHECK(q8.is_cuda() && q8.is_contiguous() && wq.is_contiguous() && wq.dim() == 2, "q8 / wq");
  TORCH_CHECK(k_cache.is_contiguous() && k_cache.dim() == 2 && k_cache.size(1) == 128, "k_cache [slots, 128]");
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "scores fp32 [T, ld]");
  const c10::cuda::CUDAGuard g(q8.device());
  const int T = wq.size(0), NH = wq.size(1);
  const int rc = b200_ix_score(reinterpret_cast<const uint8_t*>(q8.data_ptr()), wq.data_ptr<float>(), T, NH,
                               reinterpret_cast<const uint8_t*>(k_cache.data_ptr()), k_cache.size(0),
                               k_scale.data_ptr<float>(), block_table.data_ptr<int>(), block_table.stride(0),
                               q_seq.data_ptr<int>(), q_pos.data_ptr<int>(), page_size, nsplit,
                               scores.data_ptr<float>(), scores.stride(0), nullptr, cur());
  TORCH_CHECK(rc == 0, "ix_score failed ", rc);
}

void topk_select(const at::Tensor& scores, const at::Tensor& q_pos, at::Tensor out, int64_t max_n) {
  TORCH_CHECK(scores.is_cuda() && scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "scores fp32");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.is_contiguous() && out.dim() == 2, "out int32 [T, K]");
  const c10::cuda::CUDAGuard g(scores.device());
  const int rc = b200_topk_select(scores.data_ptr<float>(), scores.stride(0), q_pos.data_ptr<int>(), out.size(0),
                                  out.size(1), out.data_ptr<int>(), cur(), int(max_n));
  TORCH_CHECK(rc == 0, "topk_select failed ", rc);
}

}  // namespace

void register_attn(pybind11::module& m) {
  m.def("mla_simt", &mla_simt);
  m.def("mla_q_quant", &mla_q_quant);
  m.def("mla_q_prep", &mla_q_prep);
  m.def("mla_tc", &mla_tc, pybind11::arg("q8"), pybind11::arg("qs"), pybind11::arg("cache"), pybind11::arg("kv_scale"),
        pybind11::arg("block_table"), pybind11::arg("q_seq"), pybind11::arg("q_pos"), pybind11::arg("page_size"),
        pybind11::arg("sm_scale"), pybind11::arg("nsplit"), pybind11::arg("out"), pybind11::arg("part_o"),
        pybind11::arg("part_lse"), pybind11::arg("topk") = pybind11::none(), pybind11::arg("hb") = 0,
        pybind11::arg("lse_out") = pybind11::none(), pybind11::arg("cache2") = pybind11::none(), pybind11::arg("ratio2") = 0);
  m.def("ix_k_store", &ix_k_store);
  m.def("ix_q_quant", &ix_q_quant);
  m.def("ix_score", &ix_score);
  m.def("topk_select", &topk_select, pybind11::arg("scores"), pybind11::arg("q_pos"), pybind11::arg("out"),
        pybind11::arg("max_n") = 0);
}
