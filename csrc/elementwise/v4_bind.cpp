// Python bindings of the DeepSeek-V4-family kernels (v4.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include "elementwise.h"

namespace {

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
T* optr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void chk(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed (", rc, ")"); }

// L2 prefetch of the given tensors' bytes (each at most the first `limit`
// bytes; 16-byte aligned starts) on the current stream.
void l2_prefetch(std::vector<at::Tensor> ts, int64_t limit, int64_t nctas) {
  TORCH_CHECK(ts.size() <= 4, "at most 4 regions");
  L2Regions r{};
  for (auto& t : ts) {
    TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "contiguous CUDA tensors");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, "regions must start on 16 bytes");
    r.ptr[r.n] = t.data_ptr();
    r.bytes[r.n] = std::min<int64_t>(t.numel() * t.element_size(), limit);
    ++r.n;
  }
  if (r.n == 0) return;
  const c10::cuda::CUDAGuard g(ts[0].device());
  chk(b200_l2_prefetch(&r, nctas, at::cuda::getCurrentCUDAStream().stream()), "l2_prefetch");
}

void hc_post(at::Tensor X, const at::Tensor& y, const at::Tensor& post, const at::Tensor& comb, at::Tensor sumsq) {
  TORCH_CHECK(X.is_cuda() && X.dim() == 3 && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "X bf16 [T,hc,D]");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.stride(1) == 1, "y bf16 [T, D]");
  TORCH_CHECK(post.is_contiguous() && comb.is_contiguous() && post.scalar_type() == at::kFloat, "post/comb fp32");
  const c10::cuda::CUDAGuard g(X.device());
  chk(b200_hc_post(X.data_ptr(), y.data_ptr(), y.stride(0), post.data_ptr<float>(), comb.data_ptr<float>(), X.size(0),
                   X.size(1), X.size(2), sumsq.data_ptr<float>(), cur()),
      "hc_post");
}

void hc_pre(const at::Tensor& raw, int64_t parts, int64_t pstride, const at::Tensor& sumsq, const at::Tensor& scale,
            const at::Tensor& base, int64_t mode, int64_t iters, double eps, const at::Tensor& X,
            const at::Tensor& norm_w, double norm_eps, c10::optional<at::Tensor> post, c10::optional<at::Tensor> comb,
            c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf, c10::optional<at::Tensor> hb,
            c10::optional<at::Tensor> hf) {
  TORCH_CHECK(X.is_cuda() && X.dim() == 3 && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "X bf16 [T,hc,D]");
  TORCH_CHECK(raw.scalar_type() == at::kFloat && raw.stride(1) == 1, "raw fp32 rows");
  const c10::cuda::CUDAGuard g(X.device());
  const int T = X.size(0), hc = X.size(1), D = X.size(2);
  chk(b200_hc_pre(raw.data_ptr<float>(), raw.stride(0), parts, pstride, sumsq.data_ptr<float>(), scale.data_ptr<float>(),
                  base.data_ptr<float>(), mode, iters, float(eps), 1.f / float(hc * D), X.data_ptr(), T, hc, D,
                  norm_w.data_ptr<float>(), float(norm_eps), optr<float>(post), optr<float>(comb), optr<uint8_t>(q),
                  optr<uint8_t>(sf), optr<void>(hb), optr<float>(hf), cur()),
      "hc_pre");
}

void hc_mean(const at::Tensor& X, at::Tensor out) {
  TORCH_CHECK(X.is_cuda() && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "X bf16");
  const c10::cuda::CUDAGuard g(X.device());
  chk(b200_hc_mean(X.data_ptr(), X.size(0), X.size(1), X.size(2), out.data_ptr(), cur()), "hc_mean");
}

void engram_hash(const at::Tensor& ids, const at::Tensor& pos, const at::Tensor& q_seq, const at::Tensor& block_table,
                 const at::Tensor& out_slots, int64_t page_size, at::Tensor tok_cache, int64_t heads, int64_t rows,
                 int64_t max_n, const at::Tensor& mults, at::Tensor out) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kInt && out_slots.scalar_type() == at::kLong, "metadata");
  TORCH_CHECK(mults.scalar_type() == at::kLong && mults.numel() >= heads, "multipliers int64 [heads]");
  const c10::cuda::CUDAGuard g(ids.device());
  chk(b200_engram_hash(ids.data_ptr<int>(), pos.data_ptr<int>(), q_seq.data_ptr<int>(), block_table.data_ptr<int>(),
                       block_table.stride(0), out_slots.data_ptr<int64_t>(), page_size, tok_cache.data_ptr<int>(),
                       ids.size(0), heads, rows / heads, max_n,
                       reinterpret_cast<const unsigned long long*>(mults.data_ptr<int64_t>()), out.data_ptr<int>(),
                       cur()),
      "engram_hash");
}

// Host memory mapped into the device address space (cudaHostAllocMapped):
// the Engram tables live here and the gather kernel reads them directly.
at::Tensor host_mapped(int64_t nbytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaHostAlloc(&p, nbytes > 0 ? nbytes : 1, cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess,
              "cudaHostAlloc failed");
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFreeHost(q); },
                          at::TensorOptions().dtype(at::kByte).device(at::kCPU));
}

// table / scale: device tensors or host_mapped tensors (read through their
// device mapping)
const uint8_t* device_view(const at::Tensor& t) {
  if (t.is_cuda()) return reinterpret_cast<const uint8_t*>(t.data_ptr());
  void* d = nullptr;
  TORCH_CHECK(cudaHostGetDevicePointer(&d, t.data_ptr(), 0) == cudaSuccess,
              "host Engram tables must come from host_mapped()");
  return reinterpret_cast<const uint8_t*>(d);
}

void engram_gather(const at::Tensor& table, const at::Tensor& scale, const at::Tensor& ids, int64_t row_lo,
                   at::Tensor out) {
  TORCH_CHECK(table.dim() == 2 && table.size(1) == 256 && table.is_contiguous(), "table [rows, 256] bytes");
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.scalar_type() == at::kInt, "ids int32");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "out bf16");
  const c10::cuda::CUDAGuard g(ids.device());
  chk(b200_engram_gather(device_view(table), device_view(scale), ids.data_ptr<int>(), ids.numel(), row_lo,
                         row_lo + table.size(0), out.data_ptr(), cur()),
      "engram_gather");
}

void engram_gate(at::Tensor X, const at::Tensor& kv, const at::Tensor& q_w, const at::Tensor& k_w, double eps,
                 double clampv, at::Tensor sumsq) {
  TORCH_CHECK(X.is_cuda() && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "X bf16 [T,hc,D]");
  TORCH_CHECK(kv.stride(1) == 1 && (kv.scalar_type() == at::kBFloat16 || kv.scalar_type() == at::kFloat), "kv");
  const c10::cuda::CUDAGuard g(X.device());
  chk(b200_engram_gate(X.data_ptr(), X.size(0), X.size(1), X.size(2), kv.data_ptr(), kv.scalar_type() == at::kFloat,
                       kv.stride(0), q_w.data_ptr<float>(), k_w.data_ptr<float>(), float(eps), float(clampv),
                       sumsq.data_ptr<float>(), cur()),
      "engram_gate");
}

void hc_embed(const at::Tensor& embed, const at::Tensor& ids, at::Tensor X, at::Tensor sumsq) {
  TORCH_CHECK(embed.is_cuda() && embed.scalar_type() == at::kBFloat16 && embed.is_contiguous(), "embed bf16 [V, D]");
  TORCH_CHECK(ids.scalar_type() == at::kInt && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "ids / X");
  const c10::cuda::CUDAGuard g(X.device());
  chk(b200_hc_embed(embed.data_ptr(), ids.data_ptr<int>(), X.size(0), X.size(1), X.size(2), X.data_ptr(),
                    sumsq.data_ptr<float>(), cur()),
      "hc_embed");
}

void kv_store_v4(const at::Tensor& kv, const at::Tensor& w, double eps, const at::Tensor& pos,
                 const at::Tensor& table, at::Tensor cache, const at::Tensor& slots, double kv_scale, int64_t rd) {
  TORCH_CHECK(kv.is_cuda() && kv.stride(1) == 1, "kv rows");
  TORCH_CHECK(cache.size(1) == 576 && cache.element_size() == 1, "cache rows of 576 e4m3");
  const c10::cuda::CUDAGuard g(kv.device());
  chk(b200_kv_store_v4(kv.data_ptr(), kv.scalar_type() == at::kFloat, kv.stride(0), kv.size(0), kv.size(1), rd,
                       w.data_ptr<float>(), float(eps), pos.data_ptr<int>(), table.data_ptr<float>(),
                       slots.data_ptr<int64_t>(), reinterpret_cast<uint8_t*>(cache.data_ptr()), float(kv_scale), cur()),
      "kv_store_v4");
}

// Compressed attention: gate logits of this step's rows to their slots, then
// the compressed latent rows / indexer keys of the blocks the step completes.
void compress_store(const at::Tensor& g, const at::Tensor& bias, const at::Tensor& pos, const at::Tensor& slots,
                    const at::Tensor& q_seq, const at::Tensor& block_table, int64_t page, int64_t r,
                    const at::Tensor& kv, double kv_scale, const at::Tensor& ik, const at::Tensor& iks, at::Tensor gate,
                    at::Tensor ckv, at::Tensor cik, at::Tensor cis) {
  TORCH_CHECK(g.is_cuda() && g.dim() == 1 && (g.scalar_type() == at::kBFloat16 || g.scalar_type() == at::kFloat),
              "g bf16 / fp32 [T]");
  TORCH_CHECK(bias.scalar_type() == at::kFloat && bias.is_contiguous() && bias.numel() == r, "bias fp32 [r]");
  TORCH_CHECK(kv.dim() == 2 && kv.is_contiguous() && kv.element_size() == 1 && ckv.dim() == 2 &&
                  ckv.is_contiguous() && ckv.element_size() == 1 && ckv.size(1) == kv.size(1),
              "kv / ckv e4m3 rows of one width");
  TORCH_CHECK(ik.dim() == 2 && ik.is_contiguous() && ik.element_size() == 1 && cik.dim() == 2 &&
                  cik.is_contiguous() && cik.element_size() == 1 && cik.size(1) == ik.size(1),
              "ik / cik e4m3 rows of one width");
  TORCH_CHECK(iks.scalar_type() == at::kFloat && cis.scalar_type() == at::kFloat && gate.scalar_type() == at::kFloat &&
                  gate.is_contiguous() && cis.is_contiguous(),
              "scales / gate fp32");
  TORCH_CHECK(ckv.size(0) * r >= kv.size(0) && cik.size(0) == ckv.size(0) && cis.numel() == ckv.size(0),
              "compressed tensors hold one row per r slots");
  TORCH_CHECK(pos.scalar_type() == at::kInt && q_seq.scalar_type() == at::kInt && slots.scalar_type() == at::kLong &&
                  block_table.scalar_type() == at::kInt,
              "int32 positions / sequences / block table, int64 slots");
  const c10::cuda::CUDAGuard gd(g.device());
  chk(b200_compress_store(g.data_ptr(), g.stride(0), g.scalar_type() == at::kFloat, slots.data_ptr<int64_t>(),
                          pos.data_ptr<int>(), q_seq.data_ptr<int>(), block_table.data_ptr<int>(),
                          block_table.stride(0), page, r, g.size(0), gate.data_ptr<float>(), bias.data_ptr<float>(),
                          reinterpret_cast<const uint8_t*>(kv.data_ptr()), kv.size(1), float(kv_scale),
                          reinterpret_cast<const uint8_t*>(ik.data_ptr()), iks.data_ptr<float>(), ik.size(1),
                          reinterpret_cast<uint8_t*>(ckv.data_ptr()), reinterpret_cast<uint8_t*>(cik.data_ptr()),
                          cis.data_ptr<float>(), cur()),
      "compress_store");
}

void hc_boundary(const at::Tensor& X, c10::optional<at::Tensor> y, c10::optional<at::Tensor> post_in,
                 c10::optional<at::Tensor> comb_in, const at::Tensor& fn, const at::Tensor& scale,
                 const at::Tensor& base, int64_t mode, int64_t iters, double eps, const at::Tensor& norm_w,
                 double norm_eps, c10::optional<at::Tensor> post, c10::optional<at::Tensor> comb,
                 c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf, c10::optional<at::Tensor> hb,
                 c10::optional<at::Tensor> hf) {
  TORCH_CHECK(X.is_cuda() && X.dim() == 3 && X.is_contiguous() && X.scalar_type() == at::kBFloat16, "X bf16 [T,hc,D]");
  TORCH_CHECK(fn.is_contiguous() && fn.scalar_type() == at::kFloat && fn.size(1) == X.size(1) * X.size(2),
              "fn fp32 [M, hc*D]");
  const bool has_y = y.has_value() && y->defined();
  if (has_y)
    TORCH_CHECK(y->scalar_type() == at::kBFloat16 && y->stride(1) == 1 && y->size(0) == X.size(0), "y bf16 [T, D]");
  const c10::cuda::CUDAGuard g(X.device());
  const int T = X.size(0), hc = X.size(1), D = X.size(2);
  chk(b200_hc_boundary(X.data_ptr(), T, hc, D, has_y ? y->data_ptr() : nullptr, has_y ? y->stride(0) : 0,
                       optr<float>(post_in), optr<float>(comb_in), fn.data_ptr<float>(), fn.size(0),
                       scale.data_ptr<float>(), base.data_ptr<float>(), mode, iters, float(eps), 1.f / float(hc * D),
                       norm_w.data_ptr<float>(), float(norm_eps), optr<float>(post), optr<float>(comb),
                       optr<uint8_t>(q), optr<uint8_t>(sf), optr<void>(hb), optr<float>(hf), cur()),
      "hc_boundary");
}

void mqa_q_prep(const at::Tensor& q, const at::Tensor& pos, const at::Tensor& table, int64_t rd, at::Tensor q8,
                at::Tensor qs) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.size(2) == 512 && q.stride(2) == 1 && q.scalar_type() == at::kBFloat16,
              "q bf16 [T, H, 512]");
  const c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(q8.dim() == 3 && q8.size(0) == q.size(0) && q8.size(1) >= q.size(1) && q8.size(2) == 576 &&
                  qs.numel() >= q8.size(0) * q8.size(1),
              "q8 [T, Hq >= H, 576], qs [T, Hq]");
  chk(b200_mqa_q_prep(q.data_ptr(), q.stride(0), q.stride(1), q.size(0), q.size(1), q8.size(1), rd, pos.data_ptr<int>(),
                      table.data_ptr<float>(), reinterpret_cast<uint8_t*>(q8.data_ptr()), qs.data_ptr<float>(), cur()),
      "mqa_q_prep");
}

void attn_fixup(at::Tensor o, c10::optional<at::Tensor> lse, c10::optional<at::Tensor> sink, int64_t rd,
                const at::Tensor& pos, const at::Tensor& table) {
  TORCH_CHECK(o.is_cuda() && o.is_contiguous() && o.size(2) == 512 && o.scalar_type() == at::kBFloat16, "o");
  const c10::cuda::CUDAGuard g(o.device());
  chk(b200_attn_fixup(o.data_ptr(), o.size(0), o.size(1), optr<float>(lse), optr<float>(sink), rd, pos.data_ptr<int>(),
                      table.data_ptr<float>(), cur()),
      "attn_fixup");
}

void e5_prune(at::Tensor ids, at::Tensor w, int64_t E, double budget, int64_t max_count) {
  TORCH_CHECK(ids.is_cuda() && ids.is_contiguous() && ids.scalar_type() == at::kInt, "ids int32 [T, K]");
  TORCH_CHECK(w.is_contiguous() && w.scalar_type() == at::kFloat, "w fp32 [T, K]");
  const c10::cuda::CUDAGuard g(ids.device());
  chk(b200_e5_prune(ids.data_ptr<int>(), w.data_ptr<float>(), ids.size(0), ids.size(1), E, float(budget), max_count,
                    cur()),
      "e5_prune");
}

void trace_stamp(at::Tensor buf, int64_t idx) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kLong && idx >= 0 && idx < buf.numel(), "buf int64 [n]");
  const c10::cuda::CUDAGuard g(buf.device());
  chk(b200_trace_stamp(buf.data_ptr(), int(idx), cur()), "trace_stamp");
}

}  // namespace

void register_v4(pybind11::module& m) {
  m.def("trace_stamp", &trace_stamp);
  m.def("hc_post", &hc_post);
  m.def("l2_prefetch", &l2_prefetch);
  m.def("hc_pre", &hc_pre);
  m.def("hc_boundary", &hc_boundary);
  m.def("hc_mean", &hc_mean);
  m.def("hc_embed", &hc_embed);
  m.def("engram_hash", &engram_hash);
  m.def("engram_gather", &engram_gather);
  m.def("host_mapped", &host_mapped);
  m.def("engram_gate", &engram_gate);
  m.def("kv_store_v4", &kv_store_v4);
  m.def("mqa_q_prep", &mqa_q_prep);
  m.def("compress_store", &compress_store);
  m.def("attn_fixup", &attn_fixup);
  m.def("e5_prune", &e5_prune);
}
