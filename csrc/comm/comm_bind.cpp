// Python bindings of the fused communication kernels.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "comm.h"
#include "../elementwise/elementwise.h"

namespace {

ArPeers make_peers(const std::vector<int64_t>& bases, int64_t rank, int64_t max_t, int64_t mc = 0) {
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kArMaxRanks, "1..8 ranks");
  ArPeers p{};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  p.rank = rank;
  p.world = bases.size();
  p.max_t = max_t;
  p.mc = reinterpret_cast<uint8_t*>(mc);
  return p;
}

template <typename T>
T* optr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void ar_push(const at::Tensor& x, std::vector<int64_t> bases, int64_t rank, int64_t max_t, const at::Tensor& epoch,
             at::Tensor ticket, int64_t nctas, int64_t mc) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x bf16 [T,H]");
  const c10::cuda::CUDAGuard g(x.device());
  ArPeers p = make_peers(bases, rank, max_t, mc);
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
                      at::Tensor ticket, int64_t nctas, int64_t mc) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous(), "y bf16");
  TORCH_CHECK(pair_row.scalar_type() == at::kInt && pair_row.is_contiguous(), "pair_row int32 [T,K]");
  if (add.has_value()) TORCH_CHECK(add->scalar_type() == at::kBFloat16 && add->is_contiguous(), "add bf16 [T,H]");
  const c10::cuda::CUDAGuard g(y.device());
  ArPeers p = make_peers(bases, rank, max_t, mc);
  const int rc = b200_moe_combine_push(y.data_ptr(), reinterpret_cast<const int*>(pair_row.data_ptr()), pair_row.size(0),
                                       pair_row.size(1), y.size(1), optr<void>(add), &p,
                                       reinterpret_cast<const uint32_t*>(epoch.data_ptr()),
                                       reinterpret_cast<uint32_t*>(ticket.data_ptr()), nctas,
                                       at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "moe_combine_push failed ", rc);
}

void ar_fused_norm(const at::Tensor& x, c10::optional<at::Tensor> pair_row, c10::optional<at::Tensor> add, int64_t T,
                   std::vector<int64_t> bases, int64_t rank, int64_t max_t, at::Tensor epoch, at::Tensor ticket,
                   at::Tensor residual, const at::Tensor& w, double eps, c10::optional<at::Tensor> y,
                   c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf, at::Tensor err, int64_t mc,
                   int64_t chunks) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "x bf16 rows");
  TORCH_CHECK(residual.scalar_type() == at::kFloat && residual.is_contiguous(), "residual fp32");
  const bool comb = pair_row.has_value() && pair_row->defined();
  if (comb) {
    TORCH_CHECK(pair_row->scalar_type() == at::kInt && pair_row->is_contiguous() && pair_row->size(0) == T,
                "pair_row int32 [T, K]");
  } else {
    TORCH_CHECK(x.size(0) >= T, "x holds T rows");
  }
  if (add.has_value() && add->defined()) {
    TORCH_CHECK(add->scalar_type() == at::kBFloat16 && add->is_contiguous(), "add bf16 [T, H]");
  }
  const c10::cuda::CUDAGuard g(x.device());
  ArPeers p = make_peers(bases, rank, max_t, mc);
  const int rc = b200_ar_fused_norm(x.data_ptr(), comb ? reinterpret_cast<const int*>(pair_row->data_ptr()) : nullptr,
                                    comb ? pair_row->size(1) : 0, optr<void>(add), T, x.size(1), &p,
                                    reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                    reinterpret_cast<uint32_t*>(ticket.data_ptr()),
                                    reinterpret_cast<float*>(residual.data_ptr()),
                                    reinterpret_cast<const float*>(w.data_ptr()), eps, optr<void>(y), optr<uint8_t>(q),
                                    optr<uint8_t>(sf), reinterpret_cast<uint32_t*>(err.data_ptr()),
                                    at::cuda::getCurrentCUDAStream().stream(), int(chunks));
  TORCH_CHECK(rc == 0, "ar_fused_norm failed ", rc);
}

int64_t ar_buffer_size(int64_t world, int64_t max_t, int64_t hidden) { return ar_buffer_bytes(world, max_t, hidden); }
int64_t nvls_buffer_size(int64_t max_t, int64_t hidden) { return nvls_buffer_bytes(max_t, hidden); }
int64_t ep_ar_buffer_size(int64_t world, int64_t max_t, int64_t hidden, int64_t K) {
  return ar_buffer_bytes_ep(world, max_t, hidden, K);
}
int64_t ep_combine_offset(int64_t world, int64_t max_t, int64_t hidden) { return ep_combine_off(world, max_t, hidden); }

void ep_comb_reduce_norm(int64_t T_r, int64_t hidden, int64_t K, const at::Tensor& ids, c10::optional<at::Tensor> add,
                         std::vector<int64_t> bases, int64_t rank, int64_t max_t, at::Tensor epoch, at::Tensor ticket,
                         at::Tensor residual, const at::Tensor& w, double eps, c10::optional<at::Tensor> y,
                         c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf, at::Tensor err) {
  TORCH_CHECK(residual.is_cuda() && residual.scalar_type() == at::kFloat && residual.is_contiguous(), "residual fp32");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.size(1) == K, "ids int32 [T, K]");
  if (add.has_value()) TORCH_CHECK(add->scalar_type() == at::kBFloat16 && add->is_contiguous(), "add bf16 [T, H]");
  const c10::cuda::CUDAGuard g(residual.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_ep_comb_reduce_norm(T_r, hidden, K, ids.data_ptr<int>(), optr<void>(add), &p,
                                          reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                          reinterpret_cast<uint32_t*>(ticket.data_ptr()),
                                          reinterpret_cast<float*>(residual.data_ptr()),
                                          reinterpret_cast<const float*>(w.data_ptr()), eps, optr<void>(y),
                                          optr<uint8_t>(q), optr<uint8_t>(sf),
                                          reinterpret_cast<uint32_t*>(err.data_ptr()),
                                          at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "ep_comb_reduce_norm failed ", rc);
}

void ar_hc_post(int64_t T, int64_t D, std::vector<int64_t> bases, int64_t rank, int64_t max_t, at::Tensor epoch,
                at::Tensor ticket, int64_t expected, at::Tensor X, const at::Tensor& post, const at::Tensor& comb,
                at::Tensor sumsq, at::Tensor err) {
  TORCH_CHECK(X.is_cuda() && X.scalar_type() == at::kBFloat16 && X.is_contiguous() && X.dim() == 3 && X.size(1) == 4,
              "X bf16 [T, 4, D]");
  TORCH_CHECK(post.scalar_type() == at::kFloat && comb.scalar_type() == at::kFloat && sumsq.scalar_type() == at::kFloat,
              "post / comb / sumsq fp32");
  const c10::cuda::CUDAGuard g(X.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_ar_hc_post(T, D, &p, reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                 reinterpret_cast<uint32_t*>(ticket.data_ptr()), expected, X.data_ptr(),
                                 post.data_ptr<float>(), comb.data_ptr<float>(), sumsq.data_ptr<float>(),
                                 reinterpret_cast<uint32_t*>(err.data_ptr()), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "ar_hc_post failed ", rc);
}

void nvls_ar_norm(int64_t T, int64_t hidden, std::vector<int64_t> bases, int64_t rank, int64_t max_t, int64_t mc,
                  at::Tensor epoch, at::Tensor ticket, int64_t expected, at::Tensor residual, const at::Tensor& w,
                  double eps, c10::optional<at::Tensor> y, c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf,
                  at::Tensor err) {
  TORCH_CHECK(residual.is_cuda() && residual.scalar_type() == at::kFloat && residual.is_contiguous(), "residual fp32");
  TORCH_CHECK(mc != 0, "nvls_ar_norm needs the multicast address");
  const c10::cuda::CUDAGuard g(residual.device());
  ArPeers p = make_peers(bases, rank, max_t, mc);
  const int rc = b200_nvls_ar_norm(T, hidden, &p, reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                   reinterpret_cast<uint32_t*>(ticket.data_ptr()), expected,
                                   reinterpret_cast<float*>(residual.data_ptr()),
                                   reinterpret_cast<const float*>(w.data_ptr()), eps, optr<void>(y), optr<uint8_t>(q),
                                   optr<uint8_t>(sf), reinterpret_cast<uint32_t*>(err.data_ptr()),
                                   at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "nvls_ar_norm failed ", rc);
}

// ---------------------------------------------------------------------------
// Expert-parallel dispatch / combine
EpPeers make_ep(const std::vector<int64_t>& bases, int64_t rank, int64_t max_t, int64_t hidden, int64_t K) {
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kArMaxRanks, "1..8 ranks");
  EpPeers p{};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  p.rank = rank;
  p.world = bases.size();
  p.max_t = max_t;
  p.hidden = hidden;
  p.K = K;
  ep_layout(p.world, max_t, hidden, K, &p.par_bytes, &p.off_sf, &p.off_ids, &p.off_w, &p.off_g);
  return p;
}

// (region offset, parity bytes, scale offset, global-scale offset) of the
// dispatch buffer: the fused expert GEMM reads received rows in place.
std::vector<int64_t> ep_region_layout(int64_t world, int64_t max_t, int64_t hidden, int64_t K) {
  int64_t pb, off_sf, off_ids, off_w, off_g;
  ep_layout(world, max_t, hidden, K, &pb, &off_sf, &off_ids, &off_w, &off_g);
  return {kEpRegionOff, pb, off_sf, off_g};
}

int64_t ep_buffer_size(int64_t world, int64_t max_t, int64_t hidden, int64_t K) {
  return ep_buffer_bytes(world, max_t, hidden, K);
}

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }

void ep_dispatch(const at::Tensor& q, const at::Tensor& sf, c10::optional<at::Tensor> gs, int64_t hidden,
                 const at::Tensor& ids, const at::Tensor& w, int64_t T_step, int64_t experts_per_rank,
                 std::vector<int64_t> bases, int64_t rank, int64_t max_t, const at::Tensor& epoch, at::Tensor ticket,
                 bool peer_pull) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 2 && q.is_contiguous(), "q [T, hidden] e4m3 or [T, hidden/2] e2m1 pairs");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && w.scalar_type() == at::kFloat && w.is_contiguous(),
              "ids int32 / w fp32 [T, K]");
  const bool fp4 = gs.has_value() && gs->defined();
  TORCH_CHECK(q.size(1) == (fp4 ? hidden / 2 : hidden), "row bytes");
  const c10::cuda::CUDAGuard g(q.device());
  EpPeers p = make_ep(bases, rank, max_t, hidden, ids.size(1));
  const int rc = b200_ep_dispatch(reinterpret_cast<const uint8_t*>(q.data_ptr()),
                                  reinterpret_cast<const uint8_t*>(sf.data_ptr()), optr<float>(gs), fp4 ? 1 : 0,
                                  ids.data_ptr<int>(),
                                  w.data_ptr<float>(), ids.size(0), T_step, experts_per_rank, &p,
                                  reinterpret_cast<const uint32_t*>(epoch.data_ptr()),
                                  reinterpret_cast<uint32_t*>(ticket.data_ptr()), cur(), peer_pull ? 1 : 0);
  TORCH_CHECK(rc == 0, "ep_dispatch failed ", rc);
}

void ep_align(std::vector<int64_t> bases, int64_t rank, int64_t max_t, int64_t hidden, int64_t K, int64_t T_step,
              int64_t first, int64_t E, at::Tensor seg_start, at::Tensor seg_count, at::Tensor row_token,
              at::Tensor row_weight, at::Tensor pair_row, at::Tensor total_rows, int64_t bn1, at::Tensor ttile1,
              int64_t bn2, at::Tensor ttile2, const at::Tensor& epoch, at::Tensor err, bool release,
              c10::optional<at::Tensor> row_pair) {
  const c10::cuda::CUDAGuard g(pair_row.device());
  EpPeers p = make_ep(bases, rank, max_t, hidden, K);
  TORCH_CHECK(pair_row.numel() == p.world * T_step * K, "pair_row [world*T_step, K]");
  if (row_pair.has_value()) TORCH_CHECK(row_pair->numel() >= row_token.numel(), "row_pair as long as row_token");
  const int rc = b200_ep_align(&p, T_step, first, E, seg_start.data_ptr<int>(), seg_count.data_ptr<int>(),
                               row_token.data_ptr<int>(), row_weight.data_ptr<float>(), pair_row.data_ptr<int>(),
                               total_rows.data_ptr<int>(), bn1, ttile1.data_ptr<int>(), bn2, ttile2.data_ptr<int>(),
                               reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                               reinterpret_cast<uint32_t*>(err.data_ptr()), release ? 1 : 0, cur(),
                               optr<int>(row_pair));
  TORCH_CHECK(rc == 0, "ep_align failed ", rc);
}

void ep_gather(std::vector<int64_t> bases, int64_t rank, int64_t max_t, int64_t hidden, int64_t K, int64_t T_step,
               const at::Tensor& pair_row, at::Tensor dq, at::Tensor dsf, c10::optional<at::Tensor> dg,
               at::Tensor epoch, at::Tensor ticket) {
  const c10::cuda::CUDAGuard g(pair_row.device());
  EpPeers p = make_ep(bases, rank, max_t, hidden, K);
  const bool fp4 = dg.has_value() && dg->defined();
  const int rc = b200_ep_gather(&p, T_step, pair_row.data_ptr<int>(), fp4 ? 1 : 0,
                                reinterpret_cast<uint8_t*>(dq.data_ptr()), reinterpret_cast<uint8_t*>(dsf.data_ptr()),
                                optr<float>(dg), reinterpret_cast<uint32_t*>(epoch.data_ptr()),
                                reinterpret_cast<uint32_t*>(ticket.data_ptr()), cur());
  TORCH_CHECK(rc == 0, "ep_gather failed ", rc);
}

void ep_combine_rs(const at::Tensor& y, const at::Tensor& pair_row, int64_t T_step, int64_t T_r,
                   c10::optional<at::Tensor> add, std::vector<int64_t> bases, int64_t rank, int64_t max_t,
                   const at::Tensor& epoch, at::Tensor ticket, int64_t nctas) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.is_contiguous(), "y bf16");
  TORCH_CHECK(pair_row.scalar_type() == at::kInt && pair_row.is_contiguous(), "pair_row int32");
  if (add.has_value() && add->defined())
    TORCH_CHECK(add->scalar_type() == at::kBFloat16 && add->is_contiguous(), "add bf16 [T_r, hidden]");
  const c10::cuda::CUDAGuard g(y.device());
  ArPeers p = make_peers(bases, rank, max_t);
  const int rc = b200_ep_combine_rs(y.data_ptr(), pair_row.data_ptr<int>(), T_step, T_r, pair_row.size(1), y.size(1),
                                    optr<void>(add), &p, reinterpret_cast<const uint32_t*>(epoch.data_ptr()),
                                    reinterpret_cast<uint32_t*>(ticket.data_ptr()), nctas, cur());
  TORCH_CHECK(rc == 0, "ep_combine_rs failed ", rc);
}

// ---------------------------------------------------------------------------
// Vocab-parallel sampling.  bases empty: local candidate buffers; else the
// candidates travel through the fused all-reduce slots of those ranks.
void lm_candidates(const at::Tensor& logits, int64_t Kc, int64_t vocab_off, const at::Tensor& temperature,
                   c10::optional<at::Tensor> out, std::vector<int64_t> bases, int64_t rank, int64_t max_t,
                   int64_t hidden, c10::optional<at::Tensor> epoch, c10::optional<at::Tensor> ticket) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.stride(1) == 1, "logits [B, n]");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16, "logits fp32/bf16");
  const c10::cuda::CUDAGuard g(logits.device());
  ArPeers p{};
  const bool fused = !bases.empty();
  if (fused) {
    p = make_peers(bases, rank, max_t);
    p.hidden = hidden;
  }
  const int rc = b200_lm_candidates(logits.data_ptr(), logits.scalar_type() == at::kFloat, logits.stride(0),
                                    logits.size(0), logits.size(1), Kc, vocab_off, temperature.data_ptr<float>(),
                                    optr<void>(out), fused ? &p : nullptr,
                                    fused ? reinterpret_cast<const uint32_t*>(epoch->data_ptr()) : nullptr,
                                    fused ? reinterpret_cast<uint32_t*>(ticket->data_ptr()) : nullptr, cur());
  TORCH_CHECK(rc == 0, "lm_candidates failed ", rc);
}

void sample_final(c10::optional<at::Tensor> cand, int64_t B, int64_t Kc, int64_t world, std::vector<int64_t> bases,
                  int64_t rank, int64_t max_t, int64_t hidden, c10::optional<at::Tensor> epoch,
                  c10::optional<at::Tensor> ticket, const at::Tensor& temperature, const at::Tensor& top_p,
                  const at::Tensor& top_k, const at::Tensor& uniform, at::Tensor tokens, at::Tensor err) {
  TORCH_CHECK(tokens.scalar_type() == at::kLong && top_k.scalar_type() == at::kInt, "tokens int64, top_k int32");
  const c10::cuda::CUDAGuard g(tokens.device());
  ArPeers p{};
  const bool fused = !bases.empty();
  if (fused) {
    p = make_peers(bases, rank, max_t);
    p.hidden = hidden;
  }
  const int rc = b200_sample_final(optr<void>(cand), B, Kc, world, fused ? &p : nullptr,
                                   fused ? reinterpret_cast<uint32_t*>(epoch->data_ptr()) : nullptr,
                                   fused ? reinterpret_cast<uint32_t*>(ticket->data_ptr()) : nullptr,
                                   temperature.data_ptr<float>(), top_p.data_ptr<float>(), top_k.data_ptr<int>(),
                                   uniform.data_ptr<float>(), tokens.data_ptr<int64_t>(),
                                   reinterpret_cast<uint32_t*>(err.data_ptr()), cur());
  TORCH_CHECK(rc == 0, "sample_final failed ", rc);
}

}  // namespace

void register_comm(pybind11::module& m) {
  m.def("ar_push", &ar_push, pybind11::arg("x"), pybind11::arg("bases"), pybind11::arg("rank"), pybind11::arg("max_t"),
        pybind11::arg("epoch"), pybind11::arg("ticket"), pybind11::arg("nctas"), pybind11::arg("mc") = 0);
  m.def("ar_reduce_norm", &ar_reduce_norm);
  m.def("ar_fused_norm", &ar_fused_norm, pybind11::arg("x"), pybind11::arg("pair_row"), pybind11::arg("add"),
        pybind11::arg("T"), pybind11::arg("bases"), pybind11::arg("rank"), pybind11::arg("max_t"),
        pybind11::arg("epoch"), pybind11::arg("ticket"), pybind11::arg("residual"), pybind11::arg("w"),
        pybind11::arg("eps"), pybind11::arg("y"), pybind11::arg("q"), pybind11::arg("sf"), pybind11::arg("err"),
        pybind11::arg("mc") = 0, pybind11::arg("chunks") = 1);
  m.def("ar_buffer_size", &ar_buffer_size);
  m.def("nvls_buffer_size", &nvls_buffer_size);
  m.def("nvls_ar_norm", &nvls_ar_norm);
  m.def("ar_hc_post", &ar_hc_post);
  m.def("ep_ar_buffer_size", &ep_ar_buffer_size);
  m.def("ep_combine_offset", &ep_combine_offset);
  m.def("ep_comb_reduce_norm", &ep_comb_reduce_norm);
  m.def("moe_combine_push", &moe_combine_push, pybind11::arg("y"), pybind11::arg("pair_row"), pybind11::arg("add"),
        pybind11::arg("bases"), pybind11::arg("rank"), pybind11::arg("max_t"), pybind11::arg("epoch"),
        pybind11::arg("ticket"), pybind11::arg("nctas"), pybind11::arg("mc") = 0);
  m.def("ep_buffer_size", &ep_buffer_size);
  m.def("ep_region_layout", &ep_region_layout);
  m.def("ep_dispatch", &ep_dispatch, pybind11::arg("q"), pybind11::arg("sf"), pybind11::arg("gs"),
        pybind11::arg("hidden"), pybind11::arg("ids"), pybind11::arg("w"), pybind11::arg("T_step"),
        pybind11::arg("experts_per_rank"), pybind11::arg("bases"), pybind11::arg("rank"), pybind11::arg("max_t"),
        pybind11::arg("epoch"), pybind11::arg("ticket"), pybind11::arg("peer_pull") = false);
  m.def("ep_align", &ep_align, pybind11::arg("bases"), pybind11::arg("rank"), pybind11::arg("max_t"),
        pybind11::arg("hidden"), pybind11::arg("K"), pybind11::arg("T_step"), pybind11::arg("first"), pybind11::arg("E"),
        pybind11::arg("seg_start"), pybind11::arg("seg_count"), pybind11::arg("row_token"), pybind11::arg("row_weight"),
        pybind11::arg("pair_row"), pybind11::arg("total_rows"), pybind11::arg("bn1"), pybind11::arg("ttile1"),
        pybind11::arg("bn2"), pybind11::arg("ttile2"), pybind11::arg("epoch"), pybind11::arg("err"),
        pybind11::arg("release") = false, pybind11::arg("row_pair") = pybind11::none());
  m.def("ep_gather", &ep_gather);
  m.def("ep_combine_rs", &ep_combine_rs);
  m.def("lm_candidates", &lm_candidates);
  m.def("sample_final", &sample_final);
}
