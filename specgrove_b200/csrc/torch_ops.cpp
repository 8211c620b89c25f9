// PyTorch custom operators over the C ABI (torch.ops.specgrove_b200.*).
//
// The reference binds its native sampler as a pybind extension taking
// torch::Tensor arguments: contiguous CUDA tensors with checked dtypes,
// outputs allocated inside, launches on the current CUDA stream under a
// device guard, errors raised as RuntimeError (fused_tree_sampling.py:153-191,
// 2061-2086).  These operators give the same contract to the B200 kernels, as
// registered torch operators (schemas, CUDA kernels and Meta shape functions)
// so they compose with the dispatcher, torch.compile tracing and CUDA graphs.
// Every operator is a thin shim: checks, then one C-ABI call on the current
// stream.  Built with g++ against torch's headers (no CUDA code here).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>
#include <vector>

#include "specgrove_b200.h"

namespace {

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

void check_status(int st, const char* where) {
  TORCH_CHECK(st == SG_OK, where, ": ", sg_status_string(st), " (status ", st, "): ", sg_last_error());
}

void expect(const at::Tensor& t, at::ScalarType dtype, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == dtype, name, " must be a contiguous CUDA ",
              dtype, " tensor (got ", t.scalar_type(), t.is_cuda() ? "" : " on the host",
              t.is_contiguous() ? "" : ", non-contiguous", ")");
}

template <typename T>
T* data_or_null(const std::optional<at::Tensor>& t) {
  return t.has_value() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

// ---------------------------------------------------------------- acceptance

void tree_accept_out(const at::Tensor& probs, const at::Tensor& row_offsets, const at::Tensor& parents,
                     const at::Tensor& tokens, int64_t max_nodes, int64_t max_depth, int64_t rule,
                     const std::optional<at::Tensor>& uniforms, int64_t seed,
                     const std::optional<at::Tensor>& request_ids, const std::optional<at::Tensor>& status,
                     at::Tensor& out) {
  expect(probs, at::kFloat, "probs");
  TORCH_CHECK(probs.dim() == 2, "probs must be [rows, vocab]");
  expect(row_offsets, at::kLong, "row_offsets");
  expect(parents, at::kLong, "parents");
  expect(tokens, at::kLong, "tokens");
  const int64_t trees = row_offsets.numel() - 1;
  TORCH_CHECK(trees >= 1 && max_depth >= 0 && max_nodes >= 1, "tree_accept: bad tree counts");
  expect(out, at::kLong, "out");
  TORCH_CHECK(out.numel() == trees * (max_depth + 2), "out must be [trees, max_depth + 2]");
  int32_t stride = 0;
  if (uniforms.has_value()) {
    expect(*uniforms, at::kDouble, "uniforms");
    TORCH_CHECK(uniforms->numel() % trees == 0, "uniforms must be [trees, stride]");
    stride = static_cast<int32_t>(uniforms->numel() / trees);
  }
  if (request_ids.has_value()) expect(*request_ids, at::kLong, "request_ids");
  if (status.has_value()) expect(*status, at::kInt, "status");
  c10::cuda::CUDAGuard guard(probs.device());
  check_status(sg_tree_accept_probs(probs.data_ptr<float>(), probs.size(1), row_offsets.data_ptr<int64_t>(),
                                    parents.data_ptr<int64_t>(), tokens.data_ptr<int64_t>(),
                                    static_cast<int32_t>(trees), static_cast<int32_t>(max_nodes),
                                    static_cast<int32_t>(max_depth), static_cast<int32_t>(rule),
                                    data_or_null<double>(uniforms), stride, static_cast<uint64_t>(seed),
                                    data_or_null<int64_t>(request_ids), out.data_ptr<int64_t>(),
                                    data_or_null<int32_t>(status), stream_of(probs)),
               "specgrove_b200::tree_accept");
}

at::Tensor tree_accept(const at::Tensor& probs, const at::Tensor& row_offsets, const at::Tensor& parents,
                       const at::Tensor& tokens, int64_t max_nodes, int64_t max_depth, int64_t rule,
                       const std::optional<at::Tensor>& uniforms, int64_t seed,
                       const std::optional<at::Tensor>& request_ids, const std::optional<at::Tensor>& status) {
  at::Tensor out = at::empty({row_offsets.numel() - 1, max_depth + 2}, probs.options().dtype(at::kLong));
  tree_accept_out(probs, row_offsets, parents, tokens, max_nodes, max_depth, rule, uniforms, seed, request_ids,
                  status, out);
  return out;
}

void tree_accept_logits_out(const at::Tensor& logits, const at::Tensor& row_offsets, const at::Tensor& parents,
                            const at::Tensor& tokens, int64_t max_nodes, int64_t max_depth, double temperature,
                            const std::optional<at::Tensor>& uniforms, int64_t seed,
                            const std::optional<at::Tensor>& request_ids, const std::optional<at::Tensor>& status,
                            at::Tensor& out) {
  TORCH_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.dim() == 2 &&
                  (logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16),
              "logits must be a contiguous CUDA float32 or bfloat16 [rows, vocab] tensor");
  expect(row_offsets, at::kLong, "row_offsets");
  expect(parents, at::kLong, "parents");
  expect(tokens, at::kLong, "tokens");
  expect(out, at::kLong, "out");
  const int64_t trees = row_offsets.numel() - 1;
  TORCH_CHECK(trees >= 1 && max_depth >= 0 && max_nodes >= 1, "tree_accept_logits: bad tree counts");
  TORCH_CHECK(out.numel() == trees * (max_depth + 2), "out must be [trees, max_depth + 2]");
  int32_t stride = 0;
  if (uniforms.has_value()) {
    expect(*uniforms, at::kDouble, "uniforms");
    TORCH_CHECK(uniforms->numel() % trees == 0, "uniforms must be [trees, stride]");
    stride = static_cast<int32_t>(uniforms->numel() / trees);
  }
  if (request_ids.has_value()) expect(*request_ids, at::kLong, "request_ids");
  if (status.has_value()) expect(*status, at::kInt, "status");
  c10::cuda::CUDAGuard guard(logits.device());
  check_status(sg_tree_accept_logits(logits.data_ptr(), logits.scalar_type() == at::kBFloat16 ? SG_DTYPE_BF16
                                                                                               : SG_DTYPE_F32,
                                     logits.size(1), row_offsets.data_ptr<int64_t>(), parents.data_ptr<int64_t>(),
                                     tokens.data_ptr<int64_t>(), static_cast<int32_t>(trees),
                                     static_cast<int32_t>(max_nodes), static_cast<int32_t>(max_depth), temperature,
                                     data_or_null<double>(uniforms), stride, static_cast<uint64_t>(seed),
                                     data_or_null<int64_t>(request_ids), out.data_ptr<int64_t>(),
                                     data_or_null<int32_t>(status), stream_of(logits)),
               "specgrove_b200::tree_accept_logits");
}

void tree_follow_out(const at::Tensor& posterior, const at::Tensor& row_offsets, const at::Tensor& parents,
                     const at::Tensor& tokens, int64_t max_nodes, int64_t max_depth,
                     const std::optional<at::Tensor>& status, at::Tensor& out) {
  expect(posterior, at::kLong, "posterior");
  expect(row_offsets, at::kLong, "row_offsets");
  expect(parents, at::kLong, "parents");
  expect(tokens, at::kLong, "tokens");
  expect(out, at::kLong, "out");
  if (status.has_value()) expect(*status, at::kInt, "status");
  const int64_t trees = row_offsets.numel() - 1;
  TORCH_CHECK(trees >= 1 && max_depth >= 0, "tree_follow: bad tree counts");
  TORCH_CHECK(out.numel() == trees * (max_depth + 2), "out must be [trees, max_depth + 2]");
  c10::cuda::CUDAGuard guard(posterior.device());
  check_status(sg_tree_follow(posterior.data_ptr<int64_t>(), row_offsets.data_ptr<int64_t>(),
                              parents.data_ptr<int64_t>(), tokens.data_ptr<int64_t>(), static_cast<int32_t>(trees),
                              static_cast<int32_t>(max_nodes), static_cast<int32_t>(max_depth),
                              out.data_ptr<int64_t>(), data_or_null<int32_t>(status), stream_of(posterior)),
               "specgrove_b200::tree_follow");
}

at::Tensor tree_follow(const at::Tensor& posterior, const at::Tensor& row_offsets, const at::Tensor& parents,
                       const at::Tensor& tokens, int64_t max_nodes, int64_t max_depth,
                       const std::optional<at::Tensor>& status) {
  at::Tensor out = at::empty({row_offsets.numel() - 1, max_depth + 2}, posterior.options());
  tree_follow_out(posterior, row_offsets, parents, tokens, max_nodes, max_depth, status, out);
  return out;
}

// ----------------------------------------------------------------- KV commit

void kv_commit_accepted(at::Tensor& arena, int64_t capacity, const at::Tensor& slots, const at::Tensor& lengths_in,
                        at::Tensor& lengths_out, const at::Tensor& accept_out, int64_t max_depth,
                        const std::optional<at::Tensor>& status) {
  TORCH_CHECK(arena.is_cuda() && arena.is_contiguous() && arena.dim() >= 3, "arena must be a contiguous CUDA "
              "[..., slots * capacity, head_dim] tensor");
  expect(slots, at::kLong, "slots");
  expect(lengths_in, at::kLong, "lengths_in");
  expect(lengths_out, at::kLong, "lengths_out");
  expect(accept_out, at::kLong, "accept_out");
  if (status.has_value()) expect(*status, at::kInt, "status");
  const int64_t plane_rows = arena.size(-2);
  const int64_t row_bytes = arena.size(-1) * arena.element_size();
  const int64_t planes = arena.numel() / (plane_rows * arena.size(-1));
  c10::cuda::CUDAGuard guard(arena.device());
  check_status(sg_kv_commit_accepted(arena.data_ptr(), plane_rows, planes, row_bytes, capacity,
                                     slots.data_ptr<int64_t>(), lengths_in.data_ptr<int64_t>(),
                                     lengths_out.data_ptr<int64_t>(), accept_out.data_ptr<int64_t>(),
                                     static_cast<int32_t>(slots.numel()), static_cast<int32_t>(max_depth),
                                     data_or_null<int32_t>(status), stream_of(arena)),
               "specgrove_b200::kv_commit_accepted");
}

void kv_commit(at::Tensor& dst, const at::Tensor& src, const at::Tensor& src_rows, const at::Tensor& dst_rows,
               const at::Tensor& group_offsets, int64_t max_group_rows, const std::optional<at::Tensor>& status) {
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous() && src.is_cuda() && src.is_contiguous() && dst.dim() >= 2 &&
                  src.dim() >= 2 && dst.size(-1) == src.size(-1) && dst.scalar_type() == src.scalar_type(),
              "kv_commit: dst and src must be contiguous CUDA [planes..., rows, row] tensors of one dtype");
  expect(src_rows, at::kLong, "src_rows");
  expect(dst_rows, at::kLong, "dst_rows");
  expect(group_offsets, at::kLong, "group_offsets");
  if (status.has_value()) expect(*status, at::kInt, "status");
  const int64_t dst_plane_rows = dst.size(-2), src_plane_rows = src.size(-2);
  const int64_t planes = dst.numel() / (dst_plane_rows * dst.size(-1));
  TORCH_CHECK(src.numel() / (src_plane_rows * src.size(-1)) == planes, "kv_commit: plane counts differ");
  c10::cuda::CUDAGuard guard(dst.device());
  check_status(sg_kv_commit(dst.data_ptr(), dst_plane_rows, src.data_ptr(), src_plane_rows, planes,
                            dst.size(-1) * dst.element_size(), src_rows.data_ptr<int64_t>(),
                            dst_rows.data_ptr<int64_t>(), group_offsets.data_ptr<int64_t>(),
                            static_cast<int32_t>(group_offsets.numel() - 1), static_cast<int32_t>(max_group_rows),
                            data_or_null<int32_t>(status), stream_of(dst)),
               "specgrove_b200::kv_commit");
}

// ------------------------------------------------------- LM head + sampling

std::tuple<at::Tensor, at::Tensor> lm_head_sample(const at::Tensor& x, const at::Tensor& final_norm,
                                                  const at::Tensor& lm_head, const at::Tensor& row_node,
                                                  const at::Tensor& row_request, int64_t seed, double temperature,
                                                  double rms_eps) {
  expect(x, at::kFloat, "x");
  expect(final_norm, at::kBFloat16, "final_norm");
  expect(lm_head, at::kBFloat16, "lm_head");
  expect(row_node, at::kInt, "row_node");
  expect(row_request, at::kLong, "row_request");
  TORCH_CHECK(x.dim() == 2 && lm_head.dim() == 2 && lm_head.size(1) == x.size(1), "x [rows, hidden] and lm_head "
              "[vocab, hidden] disagree");
  const int64_t rows = x.size(0), hidden = x.size(1), vocab = lm_head.size(0);
  TORCH_CHECK(row_node.numel() == rows && row_request.numel() == rows, "one node and request key per row");
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor lse = at::empty({rows}, x.options());
  at::Tensor posterior = at::empty({rows}, x.options().dtype(at::kLong));
  const size_t bytes = sg_lm_head_sample_workspace_bytes(static_cast<int32_t>(rows), static_cast<int32_t>(hidden),
                                                         static_cast<int32_t>(vocab));
  at::Tensor ws = at::empty({static_cast<int64_t>(bytes) + 256}, x.options().dtype(at::kByte));
  uint8_t* base = ws.data_ptr<uint8_t>();
  uint8_t* aligned = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
  check_status(sg_lm_head_sample(x.data_ptr<float>(), final_norm.data_ptr(), lm_head.data_ptr(),
                                 static_cast<int32_t>(rows), static_cast<int32_t>(hidden),
                                 static_cast<int32_t>(vocab), static_cast<float>(rms_eps),
                                 row_node.data_ptr<int32_t>(), row_request.data_ptr<int64_t>(),
                                 static_cast<uint64_t>(seed), static_cast<float>(temperature),
                                 lse.data_ptr<float>(), posterior.data_ptr<int64_t>(), aligned, bytes, stream_of(x)),
               "specgrove_b200::lm_head_sample");
  return {lse, posterior};
}

std::tuple<at::Tensor, at::Tensor> lm_head_sample_normed(const at::Tensor& xn, const at::Tensor& lm_head,
                                                         const at::Tensor& row_node, const at::Tensor& row_request,
                                                         int64_t seed, double temperature) {
  expect(xn, at::kBFloat16, "xn");
  expect(lm_head, at::kBFloat16, "lm_head");
  expect(row_node, at::kInt, "row_node");
  expect(row_request, at::kLong, "row_request");
  TORCH_CHECK(xn.dim() == 2 && lm_head.dim() == 2 && lm_head.size(1) == xn.size(1), "xn [rows, hidden] and "
              "lm_head [vocab, hidden] disagree");
  const int64_t rows = xn.size(0), hidden = xn.size(1), vocab = lm_head.size(0);
  TORCH_CHECK(row_node.numel() == rows && row_request.numel() == rows, "one node and request key per row");
  c10::cuda::CUDAGuard guard(xn.device());
  at::Tensor lse = at::empty({rows}, xn.options().dtype(at::kFloat));
  at::Tensor posterior = at::empty({rows}, xn.options().dtype(at::kLong));
  const size_t bytes = sg_lm_head_sample_workspace_bytes(static_cast<int32_t>(rows), static_cast<int32_t>(hidden),
                                                         static_cast<int32_t>(vocab));
  at::Tensor ws = at::empty({static_cast<int64_t>(bytes) + 256}, xn.options().dtype(at::kByte));
  uint8_t* base = ws.data_ptr<uint8_t>();
  uint8_t* aligned = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255));
  check_status(sg_lm_head_sample_bf16(xn.data_ptr(), lm_head.data_ptr(), static_cast<int32_t>(rows),
                                      static_cast<int32_t>(hidden), static_cast<int32_t>(vocab),
                                      row_node.data_ptr<int32_t>(), row_request.data_ptr<int64_t>(),
                                      static_cast<uint64_t>(seed), static_cast<float>(temperature),
                                      lse.data_ptr<float>(), posterior.data_ptr<int64_t>(), aligned, bytes,
                                      stream_of(xn)),
               "specgrove_b200::lm_head_sample_normed");
  return {lse, posterior};
}

// --------------------------------------------------------- the verify pass

// `wave` is the int64 wave buffer of specgrove_b200.engine.Wave: row offsets
// [R + 1], parents [Q], tokens [Q], slots [R], cache lengths [R], position
// bases [R], request ids [R], back to back.
void verify_pass(int64_t engine, const at::Tensor& wave, int64_t num_requests, int64_t num_rows,
                 int64_t max_rows_per_request, int64_t max_depth, int64_t seed, double temperature, bool commit,
                 at::Tensor& accept_out, const std::optional<at::Tensor>& lengths_out,
                 const std::optional<at::Tensor>& posterior, const std::optional<at::Tensor>& lse,
                 const std::optional<at::Tensor>& child_logprob, const std::optional<at::Tensor>& hidden_out,
                 at::Tensor& status, at::IntArrayRef feature_layers, const std::optional<at::Tensor>& features_out,
                 const std::optional<at::Tensor>& features_kept,
                 const std::optional<at::Tensor>& features_kept_offsets) {
  TORCH_CHECK(engine != 0, "verify_pass: null engine handle");
  expect(wave, at::kLong, "wave");
  const int64_t R = num_requests, Q = num_rows;
  TORCH_CHECK(wave.numel() == (R + 1) + 2 * Q + 4 * R, "verify_pass: wave buffer size disagrees with R and Q");
  expect(accept_out, at::kLong, "accept_out");
  TORCH_CHECK(accept_out.numel() == R * (max_depth + 2), "accept_out must be [requests, max_depth + 2]");
  expect(status, at::kInt, "status");
  if (lengths_out.has_value()) expect(*lengths_out, at::kLong, "lengths_out");
  if (posterior.has_value()) expect(*posterior, at::kLong, "posterior");
  if (lse.has_value()) expect(*lse, at::kFloat, "lse");
  if (child_logprob.has_value()) expect(*child_logprob, at::kFloat, "child_logprob");
  if (hidden_out.has_value()) expect(*hidden_out, at::kFloat, "hidden_out");
  if (features_out.has_value()) expect(*features_out, at::kBFloat16, "features_out");
  if (features_kept.has_value()) expect(*features_kept, at::kBFloat16, "features_kept");
  if (features_kept_offsets.has_value()) expect(*features_kept_offsets, at::kLong, "features_kept_offsets");
  const int64_t* w = wave.data_ptr<int64_t>();
  std::vector<int32_t> layers(feature_layers.begin(), feature_layers.end());
  sg_wave_desc d{};
  d.num_requests = static_cast<int32_t>(R);
  d.num_rows = static_cast<int32_t>(Q);
  d.max_rows_per_request = static_cast<int32_t>(max_rows_per_request);
  d.max_depth = static_cast<int32_t>(max_depth);
  d.row_offsets = w;
  d.parents = w + (R + 1);
  d.tokens = w + (R + 1) + Q;
  d.slots = w + (R + 1) + 2 * Q;
  d.cache_lengths = d.slots + R;
  d.position_base = d.cache_lengths + R;
  d.request_ids = d.position_base + R;
  d.seed = static_cast<uint64_t>(seed);
  d.temperature = static_cast<float>(temperature);
  d.commit = commit ? 1 : 0;
  d.accept_out = accept_out.data_ptr<int64_t>();
  d.lengths_out = data_or_null<int64_t>(lengths_out);
  d.posterior = data_or_null<int64_t>(posterior);
  d.lse = data_or_null<float>(lse);
  d.child_logprob = data_or_null<float>(child_logprob);
  d.hidden_out = data_or_null<float>(hidden_out);
  d.status = status.data_ptr<int32_t>();
  d.num_feature_layers = static_cast<int32_t>(layers.size());
  d.feature_layers = layers.empty() ? nullptr : layers.data();
  d.features_out = data_or_null<void>(features_out);
  d.features_kept = data_or_null<void>(features_kept);
  d.features_kept_offsets = data_or_null<int64_t>(features_kept_offsets);
  c10::cuda::CUDAGuard guard(wave.device());
  check_status(sg_verify_pass(reinterpret_cast<void*>(engine), &d, stream_of(wave)), "specgrove_b200::verify_pass");
}

// --------------------------------------------------------- Meta (shapes only)

at::Tensor tree_accept_meta(const at::Tensor& probs, const at::Tensor& row_offsets, const at::Tensor&,
                            const at::Tensor&, int64_t, int64_t max_depth, int64_t, const std::optional<at::Tensor>&,
                            int64_t, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&) {
  return at::empty({row_offsets.size(0) - 1, max_depth + 2}, probs.options().dtype(at::kLong));
}

at::Tensor tree_follow_meta(const at::Tensor& posterior, const at::Tensor& row_offsets, const at::Tensor&,
                            const at::Tensor&, int64_t, int64_t max_depth, const std::optional<at::Tensor>&) {
  return at::empty({row_offsets.size(0) - 1, max_depth + 2}, posterior.options());
}

std::tuple<at::Tensor, at::Tensor> lm_head_sample_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&,
                                                       const at::Tensor&, const at::Tensor&, int64_t, double,
                                                       double) {
  return {at::empty({x.size(0)}, x.options()), at::empty({x.size(0)}, x.options().dtype(at::kLong))};
}

std::tuple<at::Tensor, at::Tensor> lm_head_sample_normed_meta(const at::Tensor& xn, const at::Tensor&,
                                                              const at::Tensor&, const at::Tensor&, int64_t, double) {
  return {at::empty({xn.size(0)}, xn.options().dtype(at::kFloat)),
          at::empty({xn.size(0)}, xn.options().dtype(at::kLong))};
}

void tree_accept_out_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                          int64_t, int64_t, const std::optional<at::Tensor>&, int64_t,
                          const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, at::Tensor&) {}

void tree_follow_out_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                          int64_t, const std::optional<at::Tensor>&, at::Tensor&) {}

void tree_accept_logits_out_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                                 int64_t, double, const std::optional<at::Tensor>&, int64_t,
                                 const std::optional<at::Tensor>&, const std::optional<at::Tensor>&, at::Tensor&) {}

void kv_commit_meta(at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                    const std::optional<at::Tensor>&) {}

void kv_commit_accepted_meta(at::Tensor&, int64_t, const at::Tensor&, const at::Tensor&, at::Tensor&,
                             const at::Tensor&, int64_t, const std::optional<at::Tensor>&) {}

void verify_pass_meta(int64_t, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, int64_t, double, bool,
                      at::Tensor&, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                      const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                      const std::optional<at::Tensor>&, at::Tensor&, at::IntArrayRef,
                      const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                      const std::optional<at::Tensor>&) {}

}  // namespace

TORCH_LIBRARY(specgrove_b200, m) {
  m.def("tree_accept(Tensor probs, Tensor row_offsets, Tensor parents, Tensor tokens, int max_nodes, "
        "int max_depth, int rule, Tensor? uniforms, int seed, Tensor? request_ids, Tensor(a!)? status) -> Tensor");
  m.def("tree_accept_out(Tensor probs, Tensor row_offsets, Tensor parents, Tensor tokens, int max_nodes, "
        "int max_depth, int rule, Tensor? uniforms, int seed, Tensor? request_ids, Tensor(a!)? status, "
        "Tensor(b!) out) -> ()");
  m.def("tree_accept_logits_out(Tensor logits, Tensor row_offsets, Tensor parents, Tensor tokens, int max_nodes, "
        "int max_depth, float temperature, Tensor? uniforms, int seed, Tensor? request_ids, Tensor(a!)? status, "
        "Tensor(b!) out) -> ()");
  m.def("tree_follow(Tensor posterior, Tensor row_offsets, Tensor parents, Tensor tokens, int max_nodes, "
        "int max_depth, Tensor(a!)? status) -> Tensor");
  m.def("tree_follow_out(Tensor posterior, Tensor row_offsets, Tensor parents, Tensor tokens, int max_nodes, "
        "int max_depth, Tensor(a!)? status, Tensor(b!) out) -> ()");
  m.def("kv_commit(Tensor(a!) dst, Tensor src, Tensor src_rows, Tensor dst_rows, Tensor group_offsets, "
        "int max_group_rows, Tensor(b!)? status) -> ()");
  m.def("kv_commit_accepted(Tensor(a!) arena, int capacity, Tensor slots, Tensor lengths_in, "
        "Tensor(b!) lengths_out, Tensor accept_out, int max_depth, Tensor(c!)? status) -> ()");
  m.def("lm_head_sample(Tensor x, Tensor final_norm, Tensor lm_head, Tensor row_node, Tensor row_request, "
        "int seed, float temperature, float rms_eps) -> (Tensor, Tensor)");
  m.def("lm_head_sample_normed(Tensor xn, Tensor lm_head, Tensor row_node, Tensor row_request, int seed, "
        "float temperature) -> (Tensor, Tensor)");
  m.def("verify_pass(int engine, Tensor wave, int num_requests, int num_rows, int max_rows_per_request, "
        "int max_depth, int seed, float temperature, bool commit, Tensor(a!) accept_out, "
        "Tensor(b!)? lengths_out, Tensor(c!)? posterior, Tensor(d!)? lse, Tensor(e!)? child_logprob, "
        "Tensor(f!)? hidden_out, Tensor(g!) status, int[] feature_layers, Tensor(h!)? features_out, "
        "Tensor(i!)? features_kept, Tensor(j!)? features_kept_offsets) -> ()");
}

TORCH_LIBRARY_IMPL(specgrove_b200, CUDA, m) {
  m.impl("tree_accept", &tree_accept);
  m.impl("tree_accept_out", &tree_accept_out);
  m.impl("tree_accept_logits_out", &tree_accept_logits_out);
  m.impl("tree_follow", &tree_follow);
  m.impl("tree_follow_out", &tree_follow_out);
  m.impl("kv_commit", &kv_commit);
  m.impl("kv_commit_accepted", &kv_commit_accepted);
  m.impl("lm_head_sample", &lm_head_sample);
  m.impl("lm_head_sample_normed", &lm_head_sample_normed);
  m.impl("verify_pass", &verify_pass);
}

TORCH_LIBRARY_IMPL(specgrove_b200, Meta, m) {
  m.impl("tree_accept", &tree_accept_meta);
  m.impl("tree_accept_out", &tree_accept_out_meta);
  m.impl("tree_accept_logits_out", &tree_accept_logits_out_meta);
  m.impl("tree_follow", &tree_follow_meta);
  m.impl("tree_follow_out", &tree_follow_out_meta);
  m.impl("kv_commit", &kv_commit_meta);
  m.impl("kv_commit_accepted", &kv_commit_accepted_meta);
  m.impl("lm_head_sample", &lm_head_sample_meta);
  m.impl("lm_head_sample_normed", &lm_head_sample_normed_meta);
  m.impl("verify_pass", &verify_pass_meta);
}
