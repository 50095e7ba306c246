// Python bindings of the native kernels (module b200ds._C).
// Every entry point validates devices / dtypes / alignment and launches on
// the current CUDA stream; kernels never allocate.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <algorithm>

#include <cstring>
#include <vector>

#include "attn/attn.h"
#include "comm/comm.h"
#include "elementwise/elementwise.h"
#include "gemm/gemm_mxf8.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
T* ptr(const at::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* optr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void check(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }

void check_cuda(const at::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda(), n, " must be a CUDA tensor");
}

// ---------------------------------------------------------------------------
void rmsnorm(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, double eps,
             c10::optional<at::Tensor> y, c10::optional<at::Tensor> q, c10::optional<at::Tensor> sf) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be 2-D row-major");
  TORCH_CHECK(w.scalar_type() == at::kFloat, "w must be fp32");
  const int rows = x.size(0), K = x.size(1);
  if (residual.has_value()) TORCH_CHECK(residual->scalar_type() == at::kFloat && residual->is_contiguous(), "residual fp32");
  const int ldy = y.has_value() ? y->stride(0) : 0;
  check(b200_rmsnorm(x.data_ptr(), x.scalar_type() == at::kFloat, x.stride(0), optr<float>(residual), ptr<float>(w),
                     float(eps), rows, K, optr<void>(y), ldy, optr<uint8_t>(q), optr<uint8_t>(sf), cur_stream()),
        "rmsnorm");
}

void quant(const at::Tensor& x, at::Tensor q, at::Tensor sf) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be 2-D row-major");
  check(b200_quant_mxfp8(x.data_ptr(), x.scalar_type() == at::kFloat, x.stride(0), x.size(0), x.size(1), ptr<uint8_t>(q),
                         ptr<uint8_t>(sf), cur_stream()),
        "quant");
}

// Batched bf16 GEMM for the MLA absorptions (csrc/gemm/gemm_bf16.cu).
//   x: [T, B, K] view (unit inner stride), w: [B, M, K] contiguous bf16.
void bf16_absorb(const at::Tensor& w, const at::Tensor& x, int64_t epi, c10::optional<at::Tensor> out,
                 c10::optional<at::Tensor> q_pe, c10::optional<at::Tensor> pos, c10::optional<at::Tensor> table,
                 c10::optional<at::Tensor> q8, c10::optional<at::Tensor> qs, c10::optional<at::Tensor> q,
                 c10::optional<at::Tensor> sf, int64_t splits) {
  check_cuda(w, "w");
  const c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w.scalar_type() == at::kBFloat16, "w bf16 [B, M, K]");
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.scalar_type() == at::kBFloat16, "x bf16 [T, B, K]");
  Bf16GemmArgs a{};
  a.w = w.data_ptr();
  a.x = x.data_ptr();
  a.x_ts = x.stride(0);
  a.x_bs = x.stride(1);
  a.T = x.size(0);
  a.B = x.size(1);
  a.K = x.size(2);
  a.M = w.size(1);
  TORCH_CHECK(w.size(0) == a.B && w.size(2) == a.K, "shapes");
  a.epi = epi;
  a.splits = splits;
  if (out.has_value()) {
    a.out = out->data_ptr();
    a.out_ts = out->stride(0);
    a.out_bs = out->stride(1);
  }
  if (q_pe.has_value()) {
    a.q_pe = q_pe->data_ptr();
    a.pe_ts = q_pe->stride(0);
    a.pe_bs = q_pe->stride(1);
  }
  a.pos = optr<int>(pos);
  a.table = optr<float>(table);
  a.q8 = optr<uint8_t>(q8);
  a.qs = optr<float>(qs);
  a.q = optr<uint8_t>(q);
  a.sf = optr<uint8_t>(sf);
  check(b200_bf16_gemm(&a, cur_stream()), "bf16_absorb");
}

// x [H, T, v] (contiguous, head-major) -> MXFP8 rows [T, H * v].
void quant_heads(const at::Tensor& x, at::Tensor q, at::Tensor sf) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 3 && x.is_contiguous(), "x [H, T, v] contiguous");
  const int H = x.size(0), T = x.size(1), v = x.size(2);
  check(b200_quant_mxfp8_seg(x.data_ptr(), x.scalar_type() == at::kFloat, v, T, H * v, v, (int64_t)T * v,
                             ptr<uint8_t>(q), ptr<uint8_t>(sf), cur_stream()),
        "quant_heads");
}

void gemm(const at::Tensor& w, const at::Tensor& w_sf, int64_t w_sf_estride, const at::Tensor& x,
          const at::Tensor& x_sf, int64_t nw, int64_t t, int64_t k, int64_t epi, int64_t splits,
          c10::optional<at::Tensor> out, int64_t ldo, c10::optional<at::Tensor> q_out, c10::optional<at::Tensor> sf_out,
          int64_t ldq, int64_t inter, int64_t num_experts, c10::optional<at::Tensor> seg_start,
          c10::optional<at::Tensor> seg_count, int64_t max_rows, c10::optional<at::Tensor> row_weight,
          c10::optional<at::Tensor> err, bool pdl) {
  check_cuda(w, "w");
  const c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(k % 128 == 0, "K must be a multiple of 128");
  TORCH_CHECK(nw % 128 == 0, "weight rows must be a multiple of 128");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "operands must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x_sf.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w_sf.data_ptr()) % 16 == 0,
              "scales must be 16-byte aligned");
  GemmArgs a{};
  a.w = ptr<uint8_t>(w);
  a.w_sf = ptr<uint8_t>(w_sf);
  a.w_sf_estride = w_sf_estride;
  a.x = ptr<uint8_t>(x);
  a.x_sf = ptr<uint8_t>(x_sf);
  a.x_rows = x.size(0);
  a.nw = nw;
  a.nw_total = num_experts > 0 ? nw * num_experts : w.numel() / k;
  a.t = t;
  a.k = k;
  a.splits = splits;
  a.num_experts = num_experts;
  a.seg_start = optr<int>(seg_start);
  a.seg_count = optr<int>(seg_count);
  a.max_rows_per_expert = max_rows;
  a.epi = epi;
  a.out = optr<void>(out);
  a.ldo = ldo;
  a.q_out = optr<uint8_t>(q_out);
  a.sf_out = optr<uint8_t>(sf_out);
  a.ldq = ldq;
  a.inter = inter;
  a.row_weight = optr<float>(row_weight);
  a.err = optr<uint32_t>(err);
  a.pdl = pdl ? 1 : 0;
  check(b200_gemm_mxf8(&a, cur_stream()), "gemm_mxf8");
}

// Fused GEMM + all-reduce push: out tile rows go to every rank's receive slot.
// Returns the number of CTAs that publish (the reduce kernel's expected count).
int64_t gemm_push(const at::Tensor& w, const at::Tensor& w_sf, const at::Tensor& x, const at::Tensor& x_sf,
                  int64_t nw, int64_t t, int64_t k, int64_t splits, std::vector<int64_t> bases, int64_t rank,
                  int64_t max_t, const at::Tensor& epoch, at::Tensor ticket, int64_t mc) {
  check_cuda(w, "w");
  const c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(k % 128 == 0 && nw % 128 == 0, "k, nw multiples of 128");
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= (size_t)kArMaxRanks, "1..8 ranks");
  ArPeers pe{};
  for (size_t i = 0; i < bases.size(); ++i) pe.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  pe.rank = rank;
  pe.world = bases.size();
  pe.max_t = max_t;
  pe.mc = reinterpret_cast<uint8_t*>(mc);
  GemmArgs a{};
  a.w = ptr<uint8_t>(w);
  a.w_sf = ptr<uint8_t>(w_sf);
  a.x = ptr<uint8_t>(x);
  a.x_sf = ptr<uint8_t>(x_sf);
  a.x_rows = x.size(0);
  a.nw = nw;
  a.nw_total = w.numel() / k;
  a.t = t;
  a.k = k;
  a.splits = splits;
  a.epi = kEpiClusterPush;
  a.ldo = nw;
  a.ar_peers = &pe;
  a.ar_epoch = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  a.ar_ticket = reinterpret_cast<uint32_t*>(ticket.data_ptr());
  a.pdl = 1;
  check(b200_gemm_mxf8(&a, cur_stream()), "gemm_push");
  return 1;   // arrivals per source rank
}

void rope(at::Tensor x, const at::Tensor& pos, const at::Tensor& table) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1, "x must be [T, H, d] with unit inner stride");
  TORCH_CHECK(pos.scalar_type() == at::kInt, "pos int32");
  check(b200_rope(x.data_ptr(), x.scalar_type() == at::kFloat, x.stride(0), x.stride(1), x.size(0), x.size(1), x.size(2),
                  ptr<int>(pos), ptr<float>(table), cur_stream()),
        "rope");
}

void kv_store(const at::Tensor& kv, const at::Tensor& w, double eps, const at::Tensor& pos, const at::Tensor& table,
              const at::Tensor& slots, at::Tensor cache, double kv_scale, int64_t L) {
  check_cuda(kv, "kv");
  const c10::cuda::CUDAGuard g(kv.device());
  TORCH_CHECK(kv.dim() == 2 && kv.stride(1) == 1, "kv 2-D");
  TORCH_CHECK(slots.scalar_type() == at::kLong, "slots int64");
  const int R = kv.size(1) - L;
  TORCH_CHECK(cache.size(1) == L + R, "cache width");
  check(b200_kv_store(kv.data_ptr(), kv.scalar_type() == at::kFloat, kv.stride(0), kv.size(0), L, R, ptr<float>(w),
                      float(eps), ptr<int>(pos), ptr<float>(table), ptr<int64_t>(slots), ptr<uint8_t>(cache),
                      float(kv_scale), cur_stream()),
        "kv_store");
}

void router(const at::Tensor& logits, const at::Tensor& bias, int64_t G, int64_t topk_group, int64_t K, double scaling,
            bool renorm, at::Tensor w_out, at::Tensor id_out, int64_t scoring) {
  check_cuda(logits, "logits");
  const c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "logits fp32 contiguous");
  check(b200_router(ptr<float>(logits), ptr<float>(bias), logits.size(0), logits.size(1), G, topk_group, K, float(scaling),
                    renorm ? 1 : 0, int(scoring), ptr<float>(w_out), ptr<int>(id_out), cur_stream()),
        "router");
}

void moe_align(const at::Tensor& ids, const at::Tensor& w, int64_t first, int64_t E, at::Tensor seg_start,
               at::Tensor seg_count, at::Tensor row_token, at::Tensor row_weight, at::Tensor pair_row,
               at::Tensor total_rows, int64_t bn1, c10::optional<at::Tensor> ttile1, int64_t bn2,
               c10::optional<at::Tensor> ttile2) {
  check_cuda(ids, "ids");
  const c10::cuda::CUDAGuard g(ids.device());
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "ids int32");
  check(b200_moe_align(ptr<int>(ids), ptr<float>(w), ids.size(0), ids.size(1), first, E, ptr<int>(seg_start),
                       ptr<int>(seg_count), ptr<int>(row_token), ptr<float>(row_weight), ptr<int>(pair_row),
                       ptr<int>(total_rows), bn1, optr<int>(ttile1), bn2, optr<int>(ttile2), cur_stream()),
        "moe_align");
}

void moe_gather(const at::Tensor& xq, const at::Tensor& xsf, const at::Tensor& pair_row, at::Tensor dq, at::Tensor dsf) {
  check_cuda(xq, "xq");
  const c10::cuda::CUDAGuard g(xq.device());
  check(b200_moe_gather(ptr<uint8_t>(xq), ptr<uint8_t>(xsf), ptr<int>(pair_row), pair_row.numel(), pair_row.size(1),
                        xq.size(1), ptr<uint8_t>(dq), ptr<uint8_t>(dsf), cur_stream()),
        "moe_gather");
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

void gemm_grouped(const at::Tensor& w, const at::Tensor& w_sf, const at::Tensor& x, const at::Tensor& x_sf,
                  int64_t nw, int64_t k, int64_t E, int64_t inter, int64_t bn, const at::Tensor& seg_start,
                  const at::Tensor& seg_count, const at::Tensor& ttile_off, int64_t epi, c10::optional<at::Tensor> out,
                  int64_t ldo, c10::optional<at::Tensor> q_out, c10::optional<at::Tensor> sf_out, int64_t ldq,
                  c10::optional<at::Tensor> row_weight, int64_t num_ctas, bool pdl, c10::optional<at::Tensor> w_g,
                  c10::optional<at::Tensor> x_g, double x_g_const, double out_g, bool a_tiled) {
  check_cuda(w, "w");
  const c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(k % 128 == 0 && nw % 128 == 0, "k and nw must be multiples of 128");
  GroupedArgs a{};
  a.w = ptr<uint8_t>(w);
  a.w_sf = ptr<uint8_t>(w_sf);
  a.w_sf_estride = w_sf.dim() > 1 ? w_sf.stride(0) : 0;
  a.x = ptr<uint8_t>(x);
  a.x_sf = ptr<uint8_t>(x_sf);
  a.x_rows = x.size(0);
  a.nw = nw;
  a.k = k;
  a.E = E;
  a.inter = inter;
  a.bn = bn;
  a.seg_start = ptr<int>(seg_start);
  a.seg_count = ptr<int>(seg_count);
  a.ttile_off = ptr<int>(ttile_off);
  a.epi = epi;
  a.out = optr<void>(out);
  a.ldo = ldo;
  a.q_out = optr<uint8_t>(q_out);
  a.sf_out = optr<uint8_t>(sf_out);
  a.ldq = ldq;
  a.row_weight = optr<float>(row_weight);
  a.num_ctas = num_ctas > 0 ? num_ctas : num_sms();
  a.pdl = pdl ? 1 : 0;
  a.fp4 = (w_g.has_value() && w_g->defined()) ? 1 : 0;
  a.w_g = optr<float>(w_g);
  a.x_g = optr<float>(x_g);
  a.x_g_const = float(x_g_const);
  a.out_g = float(out_g);
  a.a_tiled = a_tiled ? 1 : 0;
  check(b200_gemm_grouped(&a, cur_stream()), "gemm_grouped");
}

void moe_fused(const at::Tensor& w13, const at::Tensor& w13_sf, const at::Tensor& w2, const at::Tensor& w2_sf,
               const at::Tensor& x, const at::Tensor& x_sf, at::Tensor hq, at::Tensor hq_sf, at::Tensor y, int64_t E,
               int64_t hidden, int64_t inter, int64_t bn, const at::Tensor& seg_start, const at::Tensor& seg_count,
               const at::Tensor& ttile_off, const at::Tensor& row_weight, at::Tensor ws, at::Tensor err,
               int64_t num_ctas, bool pdl, bool a_tiled, c10::optional<at::Tensor> x_g, c10::optional<at::Tensor> w1_g,
               c10::optional<at::Tensor> w2_g, double out_g, c10::optional<at::Tensor> row_token,
               std::vector<int64_t> src_q, std::vector<int64_t> src_sf, std::vector<int64_t> src_g, int64_t src_rows,
               c10::optional<at::Tensor> src_epoch, int64_t src_epoch_add, int64_t src_par_bytes,
               c10::optional<at::Tensor> c_row_pair, int64_t c_K, int64_t c_T_step, std::vector<int64_t> c_bases,
               int64_t c_rank, int64_t c_max_t, int64_t c_off, c10::optional<at::Tensor> c_epoch) {
  check_cuda(w13, "w13");
  const c10::cuda::CUDAGuard gd(w13.device());
  TORCH_CHECK(ws.scalar_type() == at::kInt && ws.numel() >= 2 + E, "workspace int32 [2 + E]");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.is_contiguous(), "y bf16");
  MoeFusedArgs a{};
  a.w13 = ptr<uint8_t>(w13);
  a.w13_sf = ptr<uint8_t>(w13_sf);
  a.w13_sf_estride = w13_sf.dim() > 1 ? w13_sf.stride(0) : 0;
  a.w2 = ptr<uint8_t>(w2);
  a.w2_sf = ptr<uint8_t>(w2_sf);
  a.w2_sf_estride = w2_sf.dim() > 1 ? w2_sf.stride(0) : 0;
  a.x = ptr<uint8_t>(x);
  a.x_sf = ptr<uint8_t>(x_sf);
  a.hq = ptr<uint8_t>(hq);
  a.hq_sf = ptr<uint8_t>(hq_sf);
  a.y = y.data_ptr();
  a.ldy = y.stride(0);
  a.rows = std::min<int64_t>(x.size(0), hq.size(0));
  a.hidden = hidden;
  a.inter = inter;
  a.E = E;
  a.bn = bn;
  a.seg_start = ptr<int>(seg_start);
  a.seg_count = ptr<int>(seg_count);
  a.ttile_off = ptr<int>(ttile_off);
  a.row_weight = ptr<float>(row_weight);
  a.work = ptr<int>(ws);
  a.fc1_done = ptr<int>(ws) + 2;
  a.err = reinterpret_cast<uint32_t*>(err.data_ptr());
  a.num_ctas = num_ctas > 0 ? num_ctas : num_sms();
  a.pdl = pdl ? 1 : 0;
  a.a_tiled = a_tiled ? 1 : 0;
  a.fp4 = (w1_g.has_value() && w1_g->defined()) ? 1 : 0;
  a.x_g = optr<float>(x_g);
  a.w1_g = optr<float>(w1_g);
  a.w2_g = optr<float>(w2_g);
  a.out_g = float(out_g);
  // pull mode: FC1 rows read from up to 8 source buffers (raw device
  // addresses: this GPU's activations or peers' symmetric buffers)
  a.pull = src_q.empty() ? 0 : 1;
  if (a.pull) {
    TORCH_CHECK(src_q.size() <= 8 && src_sf.size() == src_q.size() && row_token.has_value() && src_rows > 0,
                "pull: <= 8 sources with scales, row_token, src_rows");
    TORCH_CHECK(!a.fp4 || src_g.size() == src_q.size(), "pull nvfp4: per-source global scales");
    for (size_t i = 0; i < src_q.size(); ++i) {
      a.src_q[i] = reinterpret_cast<const uint8_t*>(src_q[i]);
      a.src_sf[i] = reinterpret_cast<const uint8_t*>(src_sf[i]);
      a.src_g[i] = i < src_g.size() ? reinterpret_cast<const float*>(src_g[i]) : nullptr;
    }
    a.src_rows = src_rows;
    a.row_token = ptr<int>(*row_token);
    if (src_epoch.has_value() && src_epoch->defined()) {
      a.src_epoch = reinterpret_cast<const uint32_t*>(src_epoch->data_ptr());
      a.src_epoch_add = int(src_epoch_add);
      a.src_par_bytes = src_par_bytes;
    }
    a.rows = hq.size(0);
  }
  // expert-parallel combine stored by the FC2 epilogue into the owners' slots
  if (c_row_pair.has_value() && c_row_pair->defined()) {
    TORCH_CHECK(!c_bases.empty() && c_bases.size() <= 8 && c_epoch.has_value(), "combine: 1..8 rank bases + epoch");
    a.c_row_pair = ptr<int>(*c_row_pair);
    a.c_K = int(c_K);
    a.c_T_step = int(c_T_step);
    for (size_t i = 0; i < c_bases.size(); ++i) a.c_base[i] = reinterpret_cast<uint8_t*>(c_bases[i]);
    a.c_rank = int(c_rank);
    a.c_world = int(c_bases.size());
    a.c_max_t = int(c_max_t);
    a.c_off = c_off;
    a.c_epoch = reinterpret_cast<const uint32_t*>(c_epoch->data_ptr());
  }
  check(b200_moe_fused(&a, cur_stream()), "moe_fused");
}

void nvfp4_quant(const at::Tensor& x, at::Tensor q, at::Tensor sf, at::Tensor g) {
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard gd(x.device());
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x [T, K] unit inner stride");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat, "x bf16/fp32");
  TORCH_CHECK(q.is_contiguous() && q.size(1) * 2 == x.size(1), "q [T, K/2] uint8");
  check(b200_nvfp4_quant(x.data_ptr(), x.scalar_type() == at::kFloat, x.stride(0), x.size(0), x.size(1),
                         ptr<uint8_t>(q), ptr<uint8_t>(sf), ptr<float>(g), cur_stream()),
        "nvfp4_quant");
}

void moe_gather4(const at::Tensor& xq, const at::Tensor& xsf, const at::Tensor& xg, const at::Tensor& pair_row,
                 at::Tensor dq, at::Tensor dsf, at::Tensor dg) {
  check_cuda(xq, "xq");
  const c10::cuda::CUDAGuard gd(xq.device());
  check(b200_moe_gather4(ptr<uint8_t>(xq), ptr<uint8_t>(xsf), ptr<float>(xg), ptr<int>(pair_row), pair_row.numel(),
                         pair_row.size(1), xq.size(1) * 2, ptr<uint8_t>(dq), ptr<uint8_t>(dsf), ptr<float>(dg),
                         cur_stream()),
        "moe_gather4");
}

void moe_combine(const at::Tensor& y, const at::Tensor& pair_row, c10::optional<at::Tensor> add, at::Tensor out) {
  check_cuda(y, "y");
  const c10::cuda::CUDAGuard g(y.device());
  TORCH_CHECK(y.scalar_type() == at::kBFloat16, "y bf16");
  const int T = pair_row.size(0), K = pair_row.size(1), D = y.size(1);
  check(b200_moe_combine(y.data_ptr(), ptr<int>(pair_row), T, K, D, optr<void>(add),
                         add.has_value() && add->scalar_type() == at::kFloat, out.data_ptr(),
                         out.scalar_type() == at::kFloat, cur_stream()),
        "moe_combine");
}

void fill_bytes(at::Tensor t, int64_t seed, int64_t and_mask, int64_t or_mask) {
  check_cuda(t, "t");
  const c10::cuda::CUDAGuard g(t.device());
  TORCH_CHECK(t.is_contiguous(), "contiguous");
  check(b200_fill_bytes(t.data_ptr(), t.numel() * t.element_size(), (uint64_t)seed, (uint8_t)and_mask, (uint8_t)or_mask,
                        cur_stream()),
        "fill_bytes");
}

// Kernel nodes of a captured CUDA graph: (all kernels, kernels of this
// extension).  Used by the benchmark to report its launches per step.
std::vector<int64_t> graph_kernel_count(int64_t raw_graph) {
  cudaGraph_t g = reinterpret_cast<cudaGraph_t>(raw_graph);
  size_t n = 0;
  TORCH_CHECK(cudaGraphGetNodes(g, nullptr, &n) == cudaSuccess, "cudaGraphGetNodes");
  std::vector<cudaGraphNode_t> nodes(n);
  TORCH_CHECK(cudaGraphGetNodes(g, nodes.data(), &n) == cudaSuccess, "cudaGraphGetNodes");
  int64_t total = 0, ours = 0;
  for (auto nd : nodes) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nd, &t) != cudaSuccess || t != cudaGraphNodeTypeKernel) continue;
    ++total;
    cudaKernelNodeParams kp;
    if (cudaGraphKernelNodeGetParams(nd, &kp) != cudaSuccess) continue;
    const char* name = nullptr;
    if (cudaFuncGetName(&name, kp.func) == cudaSuccess && name && std::strstr(name, "b200")) ++ours;
  }
  return {total, ours};
}

}  // namespace

void register_attn(pybind11::module& m);
void register_comm(pybind11::module& m);
void register_v4(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "b200ds native sm_100a kernels";
  m.def("rmsnorm", &rmsnorm);
  m.def("quant", &quant);
  m.def("quant_heads", &quant_heads);
  m.def("bf16_absorb", &bf16_absorb, pybind11::arg("w"), pybind11::arg("x"), pybind11::arg("epi"),
        pybind11::arg("out"), pybind11::arg("q_pe"), pybind11::arg("pos"), pybind11::arg("table"),
        pybind11::arg("q8"), pybind11::arg("qs"), pybind11::arg("q"), pybind11::arg("sf"),
        pybind11::arg("splits") = 1);
  m.def("gemm", &gemm);
  m.def("gemm_push", &gemm_push, pybind11::arg("w"), pybind11::arg("w_sf"), pybind11::arg("x"), pybind11::arg("x_sf"),
        pybind11::arg("nw"), pybind11::arg("t"), pybind11::arg("k"), pybind11::arg("splits"), pybind11::arg("bases"),
        pybind11::arg("rank"), pybind11::arg("max_t"), pybind11::arg("epoch"), pybind11::arg("ticket"),
        pybind11::arg("mc") = 0);
  m.def("rope", &rope);
  m.def("kv_store", &kv_store);
  m.def("router", &router, pybind11::arg("logits"), pybind11::arg("bias"), pybind11::arg("G"),
        pybind11::arg("topk_group"), pybind11::arg("K"), pybind11::arg("scaling"), pybind11::arg("renorm"),
        pybind11::arg("w_out"), pybind11::arg("id_out"), pybind11::arg("scoring") = 0);
  m.def("moe_align", &moe_align);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("gemm_grouped", &gemm_grouped, pybind11::arg("w"), pybind11::arg("w_sf"), pybind11::arg("x"), pybind11::arg("x_sf"), pybind11::arg("nw"), pybind11::arg("k"), pybind11::arg("E"), pybind11::arg("inter"), pybind11::arg("bn"), pybind11::arg("seg_start"), pybind11::arg("seg_count"), pybind11::arg("ttile_off"), pybind11::arg("epi"), pybind11::arg("out"), pybind11::arg("ldo"), pybind11::arg("q_out"), pybind11::arg("sf_out"), pybind11::arg("ldq"), pybind11::arg("row_weight"), pybind11::arg("num_ctas"), pybind11::arg("pdl"),
        pybind11::arg("w_g") = pybind11::none(), pybind11::arg("x_g") = pybind11::none(),
        pybind11::arg("x_g_const") = 1.0, pybind11::arg("out_g") = 1.0, pybind11::arg("a_tiled") = false);
  m.def("nvfp4_quant", &nvfp4_quant);
  m.def("moe_fused", &moe_fused, pybind11::arg("w13"), pybind11::arg("w13_sf"), pybind11::arg("w2"), pybind11::arg("w2_sf"),
        pybind11::arg("x"), pybind11::arg("x_sf"), pybind11::arg("hq"), pybind11::arg("hq_sf"), pybind11::arg("y"),
        pybind11::arg("E"), pybind11::arg("hidden"), pybind11::arg("inter"), pybind11::arg("bn"),
        pybind11::arg("seg_start"), pybind11::arg("seg_count"), pybind11::arg("ttile_off"), pybind11::arg("row_weight"),
        pybind11::arg("ws"), pybind11::arg("err"), pybind11::arg("num_ctas"), pybind11::arg("pdl"),
        pybind11::arg("a_tiled"), pybind11::arg("x_g"), pybind11::arg("w1_g"), pybind11::arg("w2_g"),
        pybind11::arg("out_g"), pybind11::arg("row_token") = pybind11::none(),
        pybind11::arg("src_q") = std::vector<int64_t>{}, pybind11::arg("src_sf") = std::vector<int64_t>{},
        pybind11::arg("src_g") = std::vector<int64_t>{}, pybind11::arg("src_rows") = 0,
        pybind11::arg("src_epoch") = pybind11::none(), pybind11::arg("src_epoch_add") = 0,
        pybind11::arg("src_par_bytes") = 0, pybind11::arg("c_row_pair") = pybind11::none(), pybind11::arg("c_K") = 0,
        pybind11::arg("c_T_step") = 0, pybind11::arg("c_bases") = std::vector<int64_t>{}, pybind11::arg("c_rank") = 0,
        pybind11::arg("c_max_t") = 0, pybind11::arg("c_off") = 0, pybind11::arg("c_epoch") = pybind11::none());
  m.def("moe_gather4", &moe_gather4);
  m.def("num_sms", &num_sms);
  m.def("graph_kernel_count", &graph_kernel_count);
  m.def("fill_bytes", &fill_bytes);
  register_attn(m);
  register_v4(m);
  register_comm(m);
}
