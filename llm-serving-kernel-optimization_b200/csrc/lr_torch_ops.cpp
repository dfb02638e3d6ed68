// lr_torch_ops.cpp -- registers the C-ABI entry points of liblr_kernels.so as
// torch custom ops (namespace `lightning_router`).  Tensors are validated here,
// outputs and workspaces come from the caching allocator on the current
// stream, and a non-zero LR_* status raises a RuntimeError.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <cstring>
#include <tuple>
#include <vector>

#include "../../include/lightning_router.h"

namespace {

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == LR_OK, "lightning_router.", what, " failed: ", lr_status_string(rc), " (",
              rc, ")");
}

lr_stream_t cur_stream() {
  return reinterpret_cast<lr_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

int32_t* err_ptr(const c10::optional<at::Tensor>& err) {
  if (!err.has_value() || !err->defined()) return nullptr;
  TORCH_CHECK(err->is_cuda() && err->scalar_type() == at::kInt && err->numel() >= 1,
              "err must be a CUDA int32 tensor");
  return err->data_ptr<int32_t>();
}

at::Tensor workspace(size_t bytes, const at::Tensor& like) {
  return at::empty({static_cast<int64_t>(bytes < 16 ? 16 : bytes)},
                   like.options().dtype(at::kByte));
}

// ---------------------------------------------------------------------------
at::Tensor gate_logits(const at::Tensor& h, const at::Tensor& wg,
                       const c10::optional<at::Tensor>& bias) {
  check_cuda(h, "h");
  check_cuda(wg, "wg");
  TORCH_CHECK(h.dim() == 2 && wg.dim() == 2 && h.size(1) == wg.size(1), "gate_logits: shapes");
  TORCH_CHECK(h.scalar_type() == at::kHalf && wg.scalar_type() == at::kHalf,
              "gate_logits: fp16 inputs expected");
  const float* b = nullptr;
  if (bias.has_value() && bias->defined()) {
    check_cuda(*bias, "bias");
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == wg.size(0), "bias");
    b = bias->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(h.device());
  auto out = at::empty({h.size(0), wg.size(0)}, h.options().dtype(at::kFloat));
  check_status(lr_gate_logits(h.data_ptr(), wg.data_ptr(), b, int(h.size(0)), int(h.size(1)),
                              int(wg.size(0)), out.data_ptr<float>(), cur_stream()),
               "gate_logits");
  return out;
}

std::vector<at::Tensor> topk_gating_dispatch(const c10::optional<at::Tensor>& x,
                                             const at::Tensor& logits, int64_t k,
                                             int64_t capacity, double lbw, bool fill_dropped,
                                             bool with_aux, const c10::optional<at::Tensor>& err) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == at::kFloat, "logits: (T,E) fp32");
  const int64_t T = logits.size(0), E = logits.size(1), S = T * k;
  c10::cuda::CUDAGuard g(logits.device());
  auto iopt = logits.options().dtype(at::kInt);
  auto fopt = logits.options().dtype(at::kFloat);
  auto ids = at::empty({S}, iopt);
  auto gw = at::empty({S}, fopt);
  auto tok = at::empty({S}, iopt);
  auto offsets = at::empty({E + 1}, iopt);
  auto kept = at::empty({E}, iopt);
  auto aux = with_aux ? at::empty({}, fopt) : at::zeros({}, fopt);  // the kernel writes it
  auto rw = at::empty({S}, fopt);
  auto src = at::empty({S}, iopt);
  auto pos = at::empty({S}, iopt);
  at::Tensor permuted;
  int64_t d = 0;
  if (x.has_value() && x->defined()) {
    check_cuda(*x, "x");
    TORCH_CHECK(x->dim() == 2 && x->size(0) == T && x->scalar_type() == at::kHalf,
                "x: (T,d) fp16");
    d = x->size(1);
    permuted = fill_dropped ? at::empty({S, d}, x->options()) : at::empty({S, d}, x->options());
  } else {
    permuted = at::empty({0}, logits.options().dtype(at::kHalf));
  }
  auto ws = workspace(lr_route_workspace_bytes(int(T), int(k), int(E)), logits);
  check_status(
      lr_topk_gating_dispatch(permuted.numel() ? x->data_ptr() : nullptr, logits.data_ptr<float>(),
                              int(T), int(d), int(E), int(k), int(capacity), float(lbw),
                              fill_dropped ? 1 : 0, ids.data_ptr<int32_t>(), gw.data_ptr<float>(),
                              tok.data_ptr<int32_t>(), offsets.data_ptr<int32_t>(),
                              kept.data_ptr<int32_t>(), with_aux ? aux.data_ptr<float>() : nullptr,
                              permuted.numel() ? permuted.data_ptr() : nullptr,
                              rw.data_ptr<float>(), src.data_ptr<int32_t>(),
                              pos.data_ptr<int32_t>(), ws.data_ptr(), size_t(ws.numel()),
                              err_ptr(err), cur_stream()),
      "topk_gating_dispatch");
  return {ids, gw, tok, offsets, kept, aux, permuted, rw, src, pos};
}

// Gate projection + gating dispatch; returns {logits, then topk_gating_dispatch's outputs}.
std::vector<at::Tensor> gate_topk_gating_dispatch(const at::Tensor& x, const at::Tensor& wg,
                                                  const c10::optional<at::Tensor>& bias,
                                                  int64_t k, int64_t capacity, double lbw,
                                                  bool fill_dropped, bool permute,
                                                  const c10::optional<at::Tensor>& err) {
  check_cuda(x, "x");
  check_cuda(wg, "wg");
  TORCH_CHECK(x.dim() == 2 && wg.dim() == 2 && x.size(1) == wg.size(1), "x (T,d), wg (E,d)");
  TORCH_CHECK(x.scalar_type() == at::kHalf && wg.scalar_type() == at::kHalf,
              "gate_topk_gating_dispatch: fp16 x and wg expected");
  const float* b = nullptr;
  if (bias.has_value() && bias->defined()) {
    check_cuda(*bias, "bias");
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == wg.size(0), "bias");
    b = bias->data_ptr<float>();
  }
  const int64_t T = x.size(0), d = x.size(1), E = wg.size(0), S = T * k;
  c10::cuda::CUDAGuard g(x.device());
  auto iopt = x.options().dtype(at::kInt);
  auto fopt = x.options().dtype(at::kFloat);
  auto logits = at::empty({T, E}, fopt);
  auto ids = at::empty({S}, iopt);
  auto gw = at::empty({S}, fopt);
  auto tok = at::empty({S}, iopt);
  auto offsets = at::empty({E + 1}, iopt);
  auto kept = at::empty({E}, iopt);
  auto aux = at::empty({}, fopt);
  auto rw = at::empty({S}, fopt);
  auto src = at::empty({S}, iopt);
  auto pos = at::empty({S}, iopt);
  auto permuted = permute ? at::empty({S, d}, x.options()) : at::empty({0}, x.options());
  auto ws = workspace(lr_gate_dispatch_workspace_bytes(int(T), int(k), int(E)), x);
  check_status(lr_gate_topk_gating_dispatch(
                   x.data_ptr(), wg.data_ptr(), b, int(T), int(d), int(E), int(k), int(capacity),
                   float(lbw), fill_dropped ? 1 : 0, logits.data_ptr<float>(),
                   ids.data_ptr<int32_t>(), gw.data_ptr<float>(), tok.data_ptr<int32_t>(),
                   offsets.data_ptr<int32_t>(), kept.data_ptr<int32_t>(), aux.data_ptr<float>(),
                   permute ? permuted.data_ptr() : nullptr, rw.data_ptr<float>(),
                   src.data_ptr<int32_t>(), pos.data_ptr<int32_t>(), ws.data_ptr(),
                   size_t(ws.numel()), err_ptr(err), cur_stream()),
               "gate_topk_gating_dispatch");
  return {logits, ids, gw, tok, offsets, kept, aux, permuted, rw, src, pos};
}

// Phase 1 of the fused dispatch; the returned workspace must be passed to permute_tokens.
std::vector<at::Tensor> topk_route(const at::Tensor& logits, int64_t k, int64_t capacity,
                                   double lbw, const c10::optional<at::Tensor>& err) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == at::kFloat, "logits: (T,E) fp32");
  const int64_t T = logits.size(0), E = logits.size(1), S = T * k;
  c10::cuda::CUDAGuard g(logits.device());
  auto iopt = logits.options().dtype(at::kInt);
  auto fopt = logits.options().dtype(at::kFloat);
  auto ids = at::empty({S}, iopt);
  auto gw = at::empty({S}, fopt);
  auto tok = at::empty({S}, iopt);
  auto offsets = at::empty({E + 1}, iopt);
  auto kept = at::empty({E}, iopt);
  auto aux = at::empty({}, fopt);
  auto psum = at::empty({E}, logits.options().dtype(at::kDouble));
  auto pos = at::empty({S}, iopt);
  auto ws = workspace(lr_route_workspace_bytes(int(T), int(k), int(E)), logits);
  check_status(lr_topk_route(logits.data_ptr<float>(), int(T), int(E), int(k), int(capacity),
                             float(lbw), ids.data_ptr<int32_t>(), gw.data_ptr<float>(),
                             tok.data_ptr<int32_t>(), offsets.data_ptr<int32_t>(),
                             kept.data_ptr<int32_t>(), aux.data_ptr<float>(),
                             psum.data_ptr<double>(), pos.data_ptr<int32_t>(), ws.data_ptr(),
                             size_t(ws.numel()), err_ptr(err), cur_stream()),
               "topk_route");
  return {ids, gw, tok, offsets, kept, aux, psum, pos, ws};
}

// Phase 2: rows for kept slots (rank_base / compact as in lr_permute_tokens).
// slot_pos is updated in place from block ranks to rows.
std::vector<at::Tensor> permute_tokens(const at::Tensor& x, const at::Tensor& expert_ids,
                                       const at::Tensor& gate_weights,
                                       const at::Tensor& row_offsets,
                                       const c10::optional<at::Tensor>& rank_base,
                                       int64_t capacity, bool compact, bool fill_dropped,
                                       at::Tensor slot_pos, const at::Tensor& ws,
                                       int64_t num_rows, int64_t num_experts) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 2 && x.scalar_type() == at::kHalf, "x: (T,d) fp16");
  const int64_t T = x.size(0), S = expert_ids.numel(), k = S / std::max<int64_t>(T, 1);
  TORCH_CHECK(k * T == S, "slot count must be T*k");
  TORCH_CHECK(row_offsets.numel() == num_experts + 1, "row_offsets: (E+1,)");
  c10::cuda::CUDAGuard g(x.device());
  auto iopt = x.options().dtype(at::kInt);
  auto permuted = at::empty({num_rows, x.size(1)}, x.options());
  auto rw = at::empty({std::max<int64_t>(num_rows, 1)}, x.options().dtype(at::kFloat));
  auto src = at::empty({std::max<int64_t>(num_rows, 1)}, iopt);
  const int32_t* rb = nullptr;
  if (rank_base.has_value() && rank_base->defined()) {
    check_cuda(*rank_base, "rank_base");
    TORCH_CHECK(rank_base->numel() == num_experts, "rank_base: (E,)");
    rb = rank_base->data_ptr<int32_t>();
  }
  check_status(lr_permute_tokens(x.data_ptr(), int(T), int(x.size(1)), int(num_experts), int(k),
                                 int(capacity), expert_ids.data_ptr<int32_t>(),
                                 gate_weights.data_ptr<float>(), row_offsets.data_ptr<int32_t>(),
                                 rb, compact ? 1 : 0, fill_dropped ? 1 : 0,
                                 slot_pos.data_ptr<int32_t>(),
                                 num_rows ? permuted.data_ptr() : nullptr, rw.data_ptr<float>(),
                                 src.data_ptr<int32_t>(), ws.data_ptr(), size_t(ws.numel()),
                                 cur_stream()),
               "permute_tokens");
  return {permuted, rw, src};
}

std::vector<at::Tensor> expert_routing_forward(const at::Tensor& tokens,
                                               const at::Tensor& expert_ids,
                                               const at::Tensor& gate_weights,
                                               const at::Tensor& token_indices,
                                               int64_t num_experts, int64_t capacity,
                                               bool fill_dropped,
                                               const c10::optional<at::Tensor>& err) {
  check_cuda(tokens, "tokens");
  check_cuda(expert_ids, "expert_ids");
  check_cuda(gate_weights, "gate_weights");
  check_cuda(token_indices, "token_indices");
  TORCH_CHECK(tokens.dim() == 2 && tokens.scalar_type() == at::kHalf, "tokens: (T,d) fp16");
  TORCH_CHECK(expert_ids.scalar_type() == at::kInt && token_indices.scalar_type() == at::kInt,
              "expert_ids / token_indices: int32");
  TORCH_CHECK(gate_weights.scalar_type() == at::kFloat, "gate_weights: fp32");
  const int64_t S = expert_ids.numel(), T = tokens.size(0), d = tokens.size(1);
  TORCH_CHECK(gate_weights.numel() == S && token_indices.numel() == S, "slot counts differ");
  c10::cuda::CUDAGuard g(tokens.device());
  auto iopt = tokens.options().dtype(at::kInt);
  auto permuted = at::empty({S, d}, tokens.options());
  auto offsets = at::empty({num_experts + 1}, iopt);
  auto rw = at::empty({S}, tokens.options().dtype(at::kFloat));
  auto src = at::empty({S}, iopt);
  auto kept = at::empty({num_experts}, iopt);
  auto pos = at::empty({S}, iopt);
  auto ws = workspace(lr_dispatch_workspace_bytes(int(S), int(num_experts)), tokens);
  check_status(lr_expert_routing_forward(
                   tokens.data_ptr(), expert_ids.data_ptr<int32_t>(), gate_weights.data_ptr<float>(),
                   token_indices.data_ptr<int32_t>(), int(T), int(d), int(S), int(num_experts),
                   int(capacity), fill_dropped ? 1 : 0, permuted.data_ptr(),
                   offsets.data_ptr<int32_t>(), rw.data_ptr<float>(), src.data_ptr<int32_t>(),
                   kept.data_ptr<int32_t>(), pos.data_ptr<int32_t>(), ws.data_ptr(),
                   size_t(ws.numel()), err_ptr(err), cur_stream()),
               "expert_routing_forward");
  return {permuted, offsets, rw, src, kept, pos};
}

at::Tensor combine(const at::Tensor& y, const at::Tensor& gate_weights, const at::Tensor& slot_pos,
                   int64_t num_tokens, int64_t k) {
  check_cuda(y, "y");
  check_cuda(gate_weights, "gate_weights");
  check_cuda(slot_pos, "slot_pos");
  TORCH_CHECK(y.dim() == 2 && y.scalar_type() == at::kHalf, "y: (R,d) fp16");
  TORCH_CHECK(slot_pos.numel() == num_tokens * k && gate_weights.numel() == num_tokens * k,
              "slot counts");
  c10::cuda::CUDAGuard g(y.device());
  auto out = at::empty({num_tokens, y.size(1)}, y.options());
  check_status(lr_combine(y.data_ptr(), gate_weights.data_ptr<float>(), slot_pos.data_ptr<int32_t>(),
                          int(num_tokens), int(k), int(y.size(1)), out.data_ptr(), cur_stream()),
               "combine");
  return out;
}

at::Tensor expert_routing_gather(const at::Tensor& y, const at::Tensor& routing_w,
                                 const at::Tensor& source_idx, int64_t num_tokens,
                                 const c10::optional<at::Tensor>& err) {
  check_cuda(y, "expert_output");
  check_cuda(routing_w, "routing_weights");
  check_cuda(source_idx, "source_indices");
  TORCH_CHECK(y.dim() == 2 && y.scalar_type() == at::kHalf, "expert_output: (R,d) fp16");
  TORCH_CHECK(routing_w.scalar_type() == at::kFloat && source_idx.scalar_type() == at::kInt,
              "routing_weights fp32 / source_indices int32");
  const int64_t R = y.size(0);
  TORCH_CHECK(routing_w.numel() == R && source_idx.numel() == R, "row counts differ");
  c10::cuda::CUDAGuard g(y.device());
  auto out = at::empty({num_tokens, y.size(1)}, y.options());
  auto ws = workspace(lr_gather_workspace_bytes(int(R), int(num_tokens)), y);
  check_status(lr_expert_routing_gather(y.data_ptr(), routing_w.data_ptr<float>(),
                                        source_idx.data_ptr<int32_t>(), int(R), int(y.size(1)),
                                        int(num_tokens), out.data_ptr(), ws.data_ptr(),
                                        size_t(ws.numel()), err_ptr(err), cur_stream()),
               "expert_routing_gather");
  return out;
}

// Host-side encoding of the per-expert weight table; returns a CPU uint8 tensor.
at::Tensor encode_weight_table(const std::vector<c10::optional<at::Tensor>>& qweights,
                               const std::vector<c10::optional<at::Tensor>>& scales,
                               const std::vector<c10::optional<at::Tensor>>& zeros,
                               int64_t num_experts, int64_t d_model, int64_t d_ff,
                               int64_t group_size, bool gated) {
  TORCH_CHECK(int64_t(qweights.size()) == 3 * num_experts &&
                  int64_t(scales.size()) == 3 * num_experts &&
                  int64_t(zeros.size()) == 3 * num_experts,
              "encode_weight_table: expected 3 entries per expert");
  std::vector<lr_expert_weights> ex(num_experts);
  std::memset(ex.data(), 0, sizeof(lr_expert_weights) * ex.size());
  c10::optional<c10::Device> dev;
  for (int64_t e = 0; e < num_experts; ++e) {
    for (int m = 0; m < 3; ++m) {
      const auto& q = qweights[e * 3 + m];
      if (!q.has_value() || !q->defined()) continue;
      const auto& s = scales[e * 3 + m];
      const auto& z = zeros[e * 3 + m];
      TORCH_CHECK(s.has_value() && z.has_value(), "scales/zeros missing for a present matrix");
      check_cuda(*q, "qweight");
      check_cuda(*s, "scales");
      check_cuda(*z, "zeros");
      TORCH_CHECK(q->scalar_type() == at::kInt && z->scalar_type() == at::kInt &&
                      s->scalar_type() == at::kHalf,
                  "qweight/zeros int32, scales fp16");
      const int64_t K = (m < 2) ? d_model : d_ff, N = (m < 2) ? d_ff : d_model;
      TORCH_CHECK(q->size(0) == K && q->size(1) == N / 8, "qweight shape");
      TORCH_CHECK(s->size(0) == K / group_size && s->size(1) == N, "scales shape");
      TORCH_CHECK(z->size(0) == K / group_size && z->size(1) == N / 8, "zeros shape");
      if (!dev) dev = q->device();
      ex[e].qweight[m] = q->data_ptr<int32_t>();
      ex[e].scales[m] = s->data_ptr();
      ex[e].zeros[m] = z->data_ptr<int32_t>();
    }
  }
  TORCH_CHECK(dev.has_value(), "encode_weight_table: no matrices");
  c10::cuda::CUDAGuard g(*dev);
  const size_t bytes = lr_weight_table_bytes(int(num_experts));
  // 128-byte aligned host staging
  auto host = at::empty({int64_t(bytes + 128)}, at::TensorOptions().dtype(at::kByte));
  const uintptr_t base = reinterpret_cast<uintptr_t>(host.data_ptr());
  const int64_t off = int64_t((128 - (base & 127)) & 127);
  auto view = host.narrow(0, off, int64_t(bytes));
  check_status(lr_encode_weight_table(ex.data(), int(num_experts), int(d_model), int(d_ff),
                                      int(group_size), gated ? 1 : 0, view.data_ptr(), bytes),
               "encode_weight_table");
  return view.clone();
}

at::Tensor grouped_w4a16_gemm(const at::Tensor& table, int64_t num_experts, int64_t mode,
                              int64_t mat, const at::Tensor& A, int64_t N, int64_t group_size,
                              const c10::optional<at::Tensor>& seg_start,
                              const c10::optional<at::Tensor>& seg_len, int64_t max_rows,
                              const c10::optional<at::Tensor>& out,
                              const c10::optional<at::Tensor>& err, bool int8_operands) {
  check_cuda(table, "table");
  check_cuda(A, "A");
  TORCH_CHECK(A.dim() == 2 && A.scalar_type() == at::kHalf, "A: (R,K) fp16");
  c10::cuda::CUDAGuard g(A.device());
  at::Tensor C;
  if (out.has_value() && out->defined()) {
    C = *out;
    check_cuda(C, "out");
    TORCH_CHECK(C.scalar_type() == at::kHalf && C.dim() == 2 && C.size(0) == A.size(0) &&
                    C.size(1) == N,
                "out: (R,N) fp16");
  } else {
    C = at::empty({A.size(0), N}, A.options());
  }
  const int32_t* ss = nullptr;
  const int32_t* sl = nullptr;
  if (seg_start.has_value() && seg_start->defined()) {
    check_cuda(*seg_start, "seg_start");
    check_cuda(*seg_len, "seg_len");
    ss = seg_start->data_ptr<int32_t>();
    sl = seg_len->data_ptr<int32_t>();
  }
  // the 8-bit path (short segments) writes the token terms into a workspace
  const size_t wsb = int8_operands
                         ? lr_grouped_w4a16_workspace_bytes(int(num_experts), int(A.size(0)),
                                                            int(A.size(1)), int(N),
                                                            int(group_size), int(max_rows))
                         : 0;
  at::Tensor ws;
  if (wsb) ws = workspace(wsb, A);
  check_status(lr_grouped_w4a16_gemm(table.data_ptr(), int(num_experts), int(mode), int(mat),
                                     A.data_ptr(), int(A.size(0)), int(A.size(1)), int(N),
                                     int(group_size), ss, sl, int(max_rows), C.data_ptr(),
                                     wsb ? ws.data_ptr() : nullptr, wsb, err_ptr(err),
                                     cur_stream()),
               "grouped_w4a16_gemm");
  return C;
}

// Routing without rows: every slot's uncapped local row (slot_pos) and the
// row -> token map (source_idx, S entries) of this shard's expert segments.
at::Tensor route_rows(const at::Tensor& expert_ids, const at::Tensor& gate_weights,
                      const at::Tensor& row_offsets, at::Tensor slot_pos, const at::Tensor& ws,
                      int64_t num_tokens, int64_t num_experts, at::Tensor source_idx) {
  check_cuda(expert_ids, "expert_ids");
  const int64_t S = expert_ids.numel();
  TORCH_CHECK(num_tokens > 0 && S % num_tokens == 0, "slot count must be T*k");
  TORCH_CHECK(row_offsets.numel() == num_experts + 1, "row_offsets: (E+1,)");
  TORCH_CHECK(source_idx.scalar_type() == at::kInt && source_idx.numel() >= S &&
                  source_idx.is_contiguous(),
              "source_idx: >= S contiguous int32");
  c10::cuda::CUDAGuard g(expert_ids.device());
  auto rw = at::empty({S}, expert_ids.options().dtype(at::kFloat));
  check_status(lr_permute_tokens(nullptr, int(num_tokens), 0, int(num_experts),
                                 int(S / num_tokens), int(S), expert_ids.data_ptr<int32_t>(),
                                 gate_weights.data_ptr<float>(), row_offsets.data_ptr<int32_t>(),
                                 nullptr, 0, 0, slot_pos.data_ptr<int32_t>(), nullptr,
                                 rw.data_ptr<float>(), source_idx.data_ptr<int32_t>(),
                                 ws.data_ptr(), size_t(ws.numel()), cur_stream()),
               "route_rows");
  return rw;
}

at::Tensor ep_plan(const at::Tensor& counts, int64_t rank, int64_t capacity,
                   const c10::optional<at::Tensor>& err) {
  check_cuda(counts, "counts");
  TORCH_CHECK(counts.dim() == 2 && counts.scalar_type() == at::kInt && counts.is_contiguous(),
              "counts: contiguous (G, E) int32");
  c10::cuda::CUDAGuard g(counts.device());
  const int G = int(counts.size(0)), E = int(counts.size(1));
  const int n = lr_ep_plan_size(G, E);
  TORCH_CHECK(n > 0, "ep_plan: E must be a multiple of G");
  auto plan = at::empty({n}, counts.options());
  check_status(lr_ep_plan(counts.data_ptr<int32_t>(), G, E, int(rank), int(capacity),
                          plan.data_ptr<int32_t>(), err_ptr(err), cur_stream()),
               "ep_plan");
  return plan;
}

// Plan with the capacity from the all-gathered shard sizes (int32 [G]).
at::Tensor ep_plan_tokens(const at::Tensor& counts, const at::Tensor& shard_tokens, int64_t rank,
                          int64_t top_k, double capacity_factor, int64_t max_capacity,
                          const c10::optional<at::Tensor>& err) {
  check_cuda(counts, "counts");
  check_cuda(shard_tokens, "shard_tokens");
  TORCH_CHECK(counts.dim() == 2 && counts.scalar_type() == at::kInt && counts.is_contiguous(),
              "counts: contiguous (G, E) int32");
  TORCH_CHECK(shard_tokens.scalar_type() == at::kInt && shard_tokens.is_contiguous() &&
                  shard_tokens.numel() == counts.size(0),
              "shard_tokens: contiguous (G,) int32");
  c10::cuda::CUDAGuard g(counts.device());
  const int G = int(counts.size(0)), E = int(counts.size(1));
  const int n = lr_ep_plan_size(G, E);
  TORCH_CHECK(n > 0, "ep_plan_tokens: E must be a multiple of G");
  auto plan = at::empty({n}, counts.options());
  check_status(lr_ep_plan_tokens(counts.data_ptr<int32_t>(), shard_tokens.data_ptr<int32_t>(), G,
                                 E, int(top_k), capacity_factor, int(rank), int(max_capacity),
                                 plan.data_ptr<int32_t>(), err_ptr(err), cur_stream()),
               "ep_plan_tokens");
  return plan;
}

at::Tensor ep_gather(const at::Tensor& peer_tokens, const at::Tensor& peer_source_idx,
                     const at::Tensor& plan, int64_t num_experts, int64_t rank,
                     int64_t max_tokens, int64_t max_slots, int64_t d, at::Tensor out,
                     const c10::optional<at::Tensor>& err) {
  check_cuda(plan, "plan");
  check_cuda(out, "out");
  TORCH_CHECK(peer_tokens.scalar_type() == at::kLong && peer_source_idx.scalar_type() == at::kLong,
              "peer address arrays: int64");
  TORCH_CHECK(out.scalar_type() == at::kHalf && out.dim() == 2 && out.size(1) == d &&
                  out.is_contiguous(),
              "out: contiguous (rows, d) fp16");
  c10::cuda::CUDAGuard g(out.device());
  check_status(lr_ep_gather(reinterpret_cast<const uint64_t*>(peer_tokens.data_ptr()),
                            reinterpret_cast<const uint64_t*>(peer_source_idx.data_ptr()),
                            plan.data_ptr<int32_t>(), int(peer_tokens.numel()), int(num_experts),
                            int(rank), int(max_tokens), int(max_slots), int(d),
                            int(out.size(0)), out.data_ptr(), err_ptr(err), cur_stream()),
               "ep_gather");
  return out;
}

void ep_publish(const at::Tensor& peer_stats, const at::Tensor& peer_flags,
                const c10::optional<at::Tensor>& offsets,
                const c10::optional<at::Tensor>& prob_sums, int64_t num_tokens,
                int64_t num_experts, int64_t rank, int64_t epoch) {
  check_cuda(peer_stats, "peer_stats");
  TORCH_CHECK(peer_stats.scalar_type() == at::kLong && peer_flags.scalar_type() == at::kLong,
              "peer address arrays: int64");
  c10::cuda::CUDAGuard g(peer_stats.device());
  const int32_t* offs = nullptr;
  const double* ps = nullptr;
  if (num_tokens > 0) {
    TORCH_CHECK(offsets.has_value() && prob_sums.has_value(), "offsets / prob_sums needed");
    TORCH_CHECK(offsets->scalar_type() == at::kInt && offsets->numel() == num_experts + 1,
                "offsets: (E+1,) int32");
    TORCH_CHECK(prob_sums->scalar_type() == at::kDouble && prob_sums->numel() == num_experts,
                "prob_sums: (E,) float64");
    offs = offsets->data_ptr<int32_t>();
    ps = prob_sums->data_ptr<double>();
  }
  check_status(lr_ep_publish(reinterpret_cast<const uint64_t*>(peer_stats.data_ptr()),
                             reinterpret_cast<const uint64_t*>(peer_flags.data_ptr()), offs, ps,
                             int(num_tokens), int(peer_stats.numel()), int(num_experts),
                             int(rank), int(epoch), cur_stream()),
               "ep_publish");
}

std::vector<at::Tensor> ep_plan_wait(const at::Tensor& stats, const at::Tensor& flags,
                                     int64_t num_experts, int64_t rank, int64_t top_k,
                                     double capacity_factor, int64_t max_capacity,
                                     double load_balance_weight, int64_t epoch,
                                     const c10::optional<at::Tensor>& err) {
  check_cuda(stats, "stats");
  check_cuda(flags, "flags");
  TORCH_CHECK(stats.scalar_type() == at::kDouble && stats.dim() == 2 &&
                  stats.size(1) == 1 + 2 * num_experts && stats.is_contiguous(),
              "stats: contiguous (G, 1 + 2E) float64");
  TORCH_CHECK(flags.scalar_type() == at::kInt && flags.numel() >= 2 * stats.size(0),
              "flags: (2G,) int32");
  c10::cuda::CUDAGuard g(stats.device());
  const int G = int(stats.size(0));
  const int n = lr_ep_plan_size(G, int(num_experts));
  TORCH_CHECK(n > 0, "ep_plan_wait: E must be a multiple of G");
  auto plan = at::empty({n}, stats.options().dtype(at::kInt));
  auto aux = at::empty({}, stats.options().dtype(at::kFloat));
  check_status(lr_ep_plan_wait(stats.data_ptr<double>(), flags.data_ptr<int32_t>(), G,
                               int(num_experts), int(rank), int(top_k), capacity_factor,
                               int(max_capacity), float(load_balance_weight), int(epoch),
                               plan.data_ptr<int32_t>(), aux.data_ptr<float>(), err_ptr(err),
                               cur_stream()),
               "ep_plan_wait");
  return {plan, aux};
}

void ep_signal(const at::Tensor& peer_flags, int64_t rank, int64_t epoch) {
  check_cuda(peer_flags, "peer_flags");
  TORCH_CHECK(peer_flags.scalar_type() == at::kLong, "peer address array: int64");
  c10::cuda::CUDAGuard g(peer_flags.device());
  check_status(lr_ep_signal(reinterpret_cast<const uint64_t*>(peer_flags.data_ptr()),
                            int(peer_flags.numel()), int(rank), int(epoch), cur_stream()),
               "ep_signal");
}

at::Tensor ep_combine(const at::Tensor& peer_outputs, const at::Tensor& plan,
                      const at::Tensor& expert_ids, const at::Tensor& gate_weights,
                      const at::Tensor& slot_pos, int64_t num_tokens, int64_t num_experts,
                      int64_t rows_max, int64_t d, const c10::optional<at::Tensor>& err,
                      const c10::optional<at::Tensor>& ready_flags, int64_t epoch) {
  check_cuda(plan, "plan");
  TORCH_CHECK(peer_outputs.scalar_type() == at::kLong, "peer address array: int64");
  const int64_t S = expert_ids.numel();
  TORCH_CHECK(num_tokens >= 0 && (num_tokens == 0 || S % num_tokens == 0), "slot count");
  c10::cuda::CUDAGuard g(plan.device());
  auto out = at::empty({num_tokens, d}, plan.options().dtype(at::kHalf));
  const int k = num_tokens ? int(S / num_tokens) : 1;
  check_status(lr_ep_combine(reinterpret_cast<const uint64_t*>(peer_outputs.data_ptr()),
                             plan.data_ptr<int32_t>(), expert_ids.data_ptr<int32_t>(),
                             gate_weights.data_ptr<float>(), slot_pos.data_ptr<int32_t>(),
                             int(num_tokens), k, int(peer_outputs.numel()), int(num_experts),
                             int(d), int(rows_max), out.data_ptr(),
                             ready_flags.has_value() && ready_flags->defined()
                                 ? ready_flags->data_ptr<int32_t>()
                                 : nullptr,
                             int(epoch), err_ptr(err), cur_stream()),
               "ep_combine");
  return out;
}

}  // namespace

TORCH_LIBRARY(lightning_router, m) {
  m.def("gate_logits(Tensor h, Tensor wg, Tensor? bias) -> Tensor");
  m.def(
      "topk_gating_dispatch(Tensor? x, Tensor logits, int k, int capacity, float lbw, "
      "bool fill_dropped, bool with_aux, Tensor? err) -> Tensor[]");
  m.def(
      "gate_topk_gating_dispatch(Tensor x, Tensor wg, Tensor? bias, int k, int capacity, "
      "float lbw, bool fill_dropped, bool permute, Tensor? err) -> Tensor[]");
  m.def(
      "expert_routing_forward(Tensor tokens, Tensor expert_ids, Tensor gate_weights, "
      "Tensor token_indices, int num_experts, int capacity, bool fill_dropped, Tensor? err) -> "
      "Tensor[]");
  m.def(
      "topk_route(Tensor logits, int k, int capacity, float lbw, Tensor? err) -> Tensor[]");
  m.def(
      "permute_tokens(Tensor x, Tensor expert_ids, Tensor gate_weights, Tensor row_offsets, "
      "Tensor? rank_base, int capacity, bool compact, bool fill_dropped, Tensor(a!) slot_pos, "
      "Tensor ws, int num_rows, int num_experts) -> Tensor[]");
  m.def("combine(Tensor y, Tensor gate_weights, Tensor slot_pos, int num_tokens, int k) -> Tensor");
  m.def(
      "expert_routing_gather(Tensor expert_output, Tensor routing_weights, Tensor "
      "source_indices, int num_tokens, Tensor? err) -> Tensor");
  m.def(
      "encode_weight_table(Tensor?[] qweights, Tensor?[] scales, Tensor?[] zeros, int "
      "num_experts, int d_model, int d_ff, int group_size, bool gated) -> Tensor");
  m.def(
      "grouped_w4a16_gemm(Tensor table, int num_experts, int mode, int mat, Tensor A, int N, "
      "int group_size, Tensor? seg_start, Tensor? seg_len, int max_rows, Tensor? out, "
      "Tensor? err, bool int8_operands=True) -> Tensor");
  m.def(
      "route_rows(Tensor expert_ids, Tensor gate_weights, Tensor row_offsets, Tensor(a!) "
      "slot_pos, Tensor ws, int num_tokens, int num_experts, Tensor(b!) source_idx) -> Tensor");
  m.def("ep_plan(Tensor counts, int rank, int capacity, Tensor? err) -> Tensor");
  m.def(
      "ep_plan_tokens(Tensor counts, Tensor shard_tokens, int rank, int top_k, float cf, "
      "int max_capacity, Tensor? err) -> Tensor");
  m.def(
      "ep_gather(Tensor peer_tokens, Tensor peer_source_idx, Tensor plan, int num_experts, "
      "int rank, int max_tokens, int max_slots, int d, Tensor(a!) out, Tensor? err) -> Tensor");
  m.def(
      "ep_combine(Tensor peer_outputs, Tensor plan, Tensor expert_ids, Tensor gate_weights, "
      "Tensor slot_pos, int num_tokens, int num_experts, int rows_max, int d, Tensor? err, "
      "Tensor? ready_flags=None, int epoch=0) -> Tensor");
  m.def(
      "ep_publish(Tensor peer_stats, Tensor peer_flags, Tensor? offsets, Tensor? prob_sums, "
      "int num_tokens, int num_experts, int rank, int epoch) -> ()");
  m.def(
      "ep_plan_wait(Tensor stats, Tensor flags, int num_experts, int rank, int top_k, float cf, "
      "int max_capacity, float lbw, int epoch, Tensor? err) -> Tensor[]");
  m.def("ep_signal(Tensor peer_flags, int rank, int epoch) -> ()");
}

TORCH_LIBRARY_IMPL(lightning_router, CUDA, m) {
  m.impl("gate_logits", &gate_logits);
  m.impl("topk_gating_dispatch", &topk_gating_dispatch);
  m.impl("gate_topk_gating_dispatch", &gate_topk_gating_dispatch);
  m.impl("expert_routing_forward", &expert_routing_forward);
  m.impl("combine", &combine);
  m.impl("topk_route", &topk_route);
  m.impl("permute_tokens", &permute_tokens);
  m.impl("expert_routing_gather", &expert_routing_gather);
  m.impl("grouped_w4a16_gemm", &grouped_w4a16_gemm);
  m.impl("route_rows", &route_rows);
  m.impl("ep_plan", &ep_plan);
  m.impl("ep_plan_tokens", &ep_plan_tokens);
  m.impl("ep_gather", &ep_gather);
  m.impl("ep_combine", &ep_combine);
  m.impl("ep_publish", &ep_publish);
  m.impl("ep_plan_wait", &ep_plan_wait);
  m.impl("ep_signal", &ep_signal);
}

TORCH_LIBRARY_IMPL(lightning_router, CompositeExplicitAutograd, m) {
  m.impl("encode_weight_table", &encode_weight_table);
}
