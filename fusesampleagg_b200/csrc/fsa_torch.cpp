// fsa_torch.cpp - PyTorch binding of libfsa_sm100.so: the operator's
// autograd functions and output allocation in C++, the counterpart of the
// reference's torch extension (fuseop/binding.cpp:74-231) and of its Python
// autograd functions (fuseop/__init__.py:32-72, :108-161).
//
// Every kernel launch goes through the C ABI (include/fsa_sm100.h); this
// file only checks arguments, allocates outputs with ATen on the input's
// device and passes the current CUDA stream.  Keeping the autograd glue in
// C++ takes the per-call host cost off the Python interpreter (the backward
// runs on the autograd engine's device thread without the GIL).
//
// Argument checks and their messages follow fuseop/binding.cpp:16-53 (graph
// inputs), :119-135 and :200-218 (backward); the Python layer keeps the
// reference's ValueError / TypeError checks (fuseop/__init__.py:15-29).

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/custom_function.h>
#include <torch/python.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "fsa_sm100.h"

namespace {

using at::Tensor;
using torch::autograd::AutogradContext;
using torch::autograd::variable_list;

void check_status(int status, const char* what) {
  if (status == FSA_OK) return;
  const char* text = fsa_status_string(status);
  if (status == FSA_ERR_CUDA) {
    TORCH_CHECK(false, what, " failed: ", text, " (cudaError ", fsa_last_cuda_error(), ")");
  }
  TORCH_CHECK(false, what, " failed: ", text);
}

void* stream_of(const Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// fuseop/binding.cpp:16-53
void check_graph_inputs(const Tensor& rowptr, const Tensor& col, const Tensor& x,
                        const Tensor& frontier) {
  TORCH_CHECK(x.is_cuda() && rowptr.is_cuda() && col.is_cuda() && frontier.is_cuda(),
              "all inputs must be CUDA tensors");
  const auto dev = x.device();
  TORCH_CHECK(rowptr.device() == dev && col.device() == dev && frontier.device() == dev,
              "all inputs must be on the same CUDA device");
  TORCH_CHECK(rowptr.scalar_type() == at::kInt && col.scalar_type() == at::kInt &&
                  frontier.scalar_type() == at::kInt,
              "rowptr, col, and frontier must be int32");
  TORCH_CHECK(x.scalar_type() == at::kFloat, "x must be float32");
  TORCH_CHECK(rowptr.dim() == 1 && col.dim() == 1 && x.dim() == 2 && frontier.dim() == 1,
              "expected rowptr[N+1], col[E], x[N,D], and frontier[B]");
  TORCH_CHECK(x.is_contiguous() && rowptr.is_contiguous() && col.is_contiguous() &&
                  frontier.is_contiguous(),
              "all inputs must be contiguous");
  TORCH_CHECK(rowptr.numel() == x.size(0) + 1, "rowptr length must equal N+1");
}

void check_fanout_1hop(int64_t fanout) {
  TORCH_CHECK(fanout >= 0, "fanout must be non-negative");
  TORCH_CHECK(fanout <= FSA_MAX_FANOUT_1HOP, "fanout exceeds the supported maximum of ",
              FSA_MAX_FANOUT_1HOP);
}

void check_fanout_2hop(int64_t f1, int64_t f2) {
  TORCH_CHECK(f1 >= 0 && f2 >= 0, "fanouts must be non-negative");
  TORCH_CHECK(f1 == 0 || f2 <= (INT64_MAX - f1) / f1, "fanout pair is too large");
  TORCH_CHECK(f1 + f1 * f2 <= FSA_MAX_2HOP_ENTRIES,
              "fanout pair requires too much shared memory; reduce fanout1 or fanout2");
}

void check_offset(int64_t batch_offset) {
  TORCH_CHECK(batch_offset >= 0, "batch_offset must be non-negative");
}

// The dense feature gradient, zero-filled by the library's fill kernel (the
// reference's at::zeros, fuseop/binding.cpp:137, :220).
Tensor zeroed(int64_t num_nodes, int64_t dim, const Tensor& like) {
  Tensor g = at::empty({num_nodes, dim}, like.options().dtype(at::kFloat));
  check_status(fsa_fill_zero_f32(g.data_ptr<float>(), g.numel(), stream_of(like)),
               "fsa_fill_zero_f32");
  return g;
}

// ---------------------------------------------------------------------------
// 1-hop
// ---------------------------------------------------------------------------

std::vector<Tensor> forward_1hop(const Tensor& rowptr_in, const Tensor& col_in,
                                 const Tensor& x_in, const Tensor& frontier_in, int64_t fanout,
                                 uint64_t seed, bool capture, int64_t batch_offset) {
  const Tensor rowptr = rowptr_in.contiguous();
  const Tensor col = col_in.contiguous();
  const Tensor x = x_in.contiguous();
  const Tensor frontier = frontier_in.contiguous();
  check_graph_inputs(rowptr, col, x, frontier);
  check_fanout_1hop(fanout);
  check_offset(batch_offset);
  const int64_t B = frontier.size(0);
  const int64_t D = x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  auto f32 = x.options();
  auto i32 = x.options().dtype(at::kInt);
  if (B == 0 || fanout == 0) {
    return {at::zeros({B, D}, f32), at::full({B, fanout}, -1, i32), at::zeros({B}, i32)};
  }
  Tensor out = at::empty({B, D}, f32);
  Tensor samples, takes;
  if (capture) {
    samples = at::empty({B, fanout}, i32);
    takes = at::empty({B}, i32);
  }
  check_status(
      fsa_sample_agg_forward(rowptr.data_ptr<int32_t>(), col.data_ptr<int32_t>(), x.size(0),
                             col.numel(), x.data_ptr<float>(), D, frontier.data_ptr<int32_t>(),
                             B, batch_offset, static_cast<int32_t>(fanout), seed,
                             out.data_ptr<float>(),
                             capture ? samples.data_ptr<int32_t>() : nullptr,
                             capture ? takes.data_ptr<int32_t>() : nullptr, stream_of(x)),
      "fsa_sample_agg_forward");
  return {out, samples, takes};
}

// fuseop/binding.cpp:119-145
Tensor backward_1hop(const Tensor& samples, const Tensor& takes, const Tensor& grad_out,
                     int64_t num_nodes) {
  TORCH_CHECK(samples.is_cuda() && takes.is_cuda() && grad_out.is_cuda(),
              "backward inputs must be CUDA tensors");
  TORCH_CHECK(samples.scalar_type() == at::kInt && takes.scalar_type() == at::kInt,
              "samples and takes must be int32");
  TORCH_CHECK(samples.device() == takes.device() && takes.device() == grad_out.device(),
              "backward inputs must be on the same CUDA device");
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && grad_out.dim() == 2,
              "grad_out must be a float32 matrix");
  TORCH_CHECK(samples.dim() == 2 && takes.dim() == 1 && samples.size(0) == grad_out.size(0) &&
                  takes.size(0) == grad_out.size(0),
              "saved sample shapes do not match grad_out");
  TORCH_CHECK(samples.is_contiguous() && takes.is_contiguous() && grad_out.is_contiguous(),
              "backward inputs must be contiguous");
  TORCH_CHECK(num_nodes >= 0, "num_nodes must be non-negative");
  const int64_t B = grad_out.size(0);
  const int64_t D = grad_out.size(1);
  const c10::cuda::CUDAGuard guard(grad_out.device());
  Tensor grad_x = zeroed(num_nodes, D, grad_out);
  if (B == 0 || samples.size(1) == 0) return grad_x;
  check_status(fsa_sample_agg_backward(samples.data_ptr<int32_t>(), takes.data_ptr<int32_t>(),
                                       grad_out.data_ptr<float>(), B, D,
                                       static_cast<int32_t>(samples.size(1)),
                                       grad_x.data_ptr<float>(), num_nodes, stream_of(grad_out)),
               "fsa_sample_agg_backward");
  return grad_x;
}

// fuseop/__init__.py:32-72
struct SampleAgg1Hop : public torch::autograd::Function<SampleAgg1Hop> {
  static Tensor forward(AutogradContext* ctx, const Tensor& rowptr, const Tensor& col,
                        const Tensor& x, const Tensor& frontier, int64_t fanout, uint64_t seed,
                        bool capture, bool grad_needed, int64_t batch_offset) {
    auto r = forward_1hop(rowptr, col, x, frontier, fanout, seed, capture, batch_offset);
    if (capture) ctx->save_for_backward({r[1], r[2]});
    ctx->saved_data["capture"] = capture;
    ctx->saved_data["grad_needed"] = grad_needed;
    ctx->saved_data["num_nodes"] = x.size(0);
    return r[0];
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    Tensor grad_x;
    if (ctx->saved_data["capture"].toBool() && ctx->saved_data["grad_needed"].toBool()) {
      auto saved = ctx->get_saved_variables();
      grad_x = backward_1hop(saved[0], saved[1], grads[0].contiguous(),
                             ctx->saved_data["num_nodes"].toInt());
    }
    return {Tensor(), Tensor(), grad_x, Tensor(), Tensor(), Tensor(), Tensor(), Tensor(),
            Tensor()};
  }
};

Tensor sample_agg(const Tensor& rowptr, const Tensor& col, const Tensor& x,
                  const Tensor& frontier, int64_t fanout, uint64_t seed, bool save_indices,
                  int64_t batch_offset) {
  const bool grad_needed = at::GradMode::is_enabled() && x.requires_grad();
  const bool capture = save_indices || x.requires_grad();
  return SampleAgg1Hop::apply(rowptr, col, x, frontier, fanout, seed, capture, grad_needed,
                              batch_offset);
}

std::vector<Tensor> sample_agg_with_samples(const Tensor& rowptr, const Tensor& col,
                                            const Tensor& x, const Tensor& frontier,
                                            int64_t fanout, uint64_t seed,
                                            int64_t batch_offset) {
  const at::AutoGradMode no_grad(false);
  return forward_1hop(rowptr, col, x, frontier, fanout, seed, true, batch_offset);
}

// ---------------------------------------------------------------------------
// 2-hop
// ---------------------------------------------------------------------------

// `zero`: the dense gradient buffer to zero inside the forward (undefined =
// none).  samples1, samples2 and the workspace share one allocation, each
// part on a 256-byte boundary.
std::tuple<Tensor, Tensor, Tensor> forward_2hop(const Tensor& rowptr_in, const Tensor& col_in,
                                                const Tensor& x_in, const Tensor& frontier_in,
                                                int64_t f1, int64_t f2, uint64_t seed,
                                                bool capture, int64_t batch_offset,
                                                const Tensor& zero,
                                                const Tensor& clear_table = Tensor(),
                                                const Tensor& clear_rows = Tensor()) {
  const Tensor rowptr = rowptr_in.contiguous();
  const Tensor col = col_in.contiguous();
  const Tensor x = x_in.contiguous();
  const Tensor frontier = frontier_in.contiguous();
  check_graph_inputs(rowptr, col, x, frontier);
  check_fanout_2hop(f1, f2);
  check_offset(batch_offset);
  const int64_t B = frontier.size(0);
  const int64_t D = x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  auto f32 = x.options();
  auto i32 = x.options().dtype(at::kInt);
  const bool clearing = clear_rows.defined() && clear_rows.numel() > 0;
  if (B == 0 || f1 == 0 || f2 == 0) {
    if (zero.defined()) zero.zero_();
    if (clearing) {
      check_status(fsa_zero_rows_f32(clear_table.data_ptr<float>(), clear_table.size(0),
                                     clear_table.size(1), clear_rows.data_ptr<int32_t>(),
                                     clear_rows.numel(), stream_of(x)),
                   "fsa_zero_rows_f32");
    }
    return {at::zeros({B, D}, f32), at::full({B, f1}, -1, i32), at::full({B, f1, f2}, -1, i32)};
  }
  const size_t ws_bytes = fsa_sample_agg_2hop_workspace_size(
      B, static_cast<int32_t>(f1), static_cast<int32_t>(f2), capture ? 1 : 0, capture ? 1 : 0);
  Tensor out = at::empty({B, D}, f32);
  Tensor s1, s2, ws;
  void* ws_ptr = nullptr;
  if (capture) {
    const int64_t n1 = B * f1;
    const int64_t n2 = n1 * f2;
    const int64_t o2 = (n1 + 63) / 64 * 64;
    const int64_t ow = (o2 + n2 + 63) / 64 * 64;
    Tensor buf = at::empty({ow + static_cast<int64_t>((ws_bytes + 3) / 4)}, i32);
    s1 = buf.narrow(0, 0, n1).view({B, f1});
    s2 = buf.narrow(0, o2, n2).view({B, f1, f2});
    ws_ptr = buf.data_ptr<int32_t>() + ow;
  } else {
    ws = at::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(at::kByte));
    ws_ptr = ws.data_ptr();
  }
  if (clearing) {
    check_status(fsa_sample_agg_2hop_forward_zero_rows(
                     rowptr.data_ptr<int32_t>(), col.data_ptr<int32_t>(), x.size(0),
                     col.numel(), x.data_ptr<float>(), D, frontier.data_ptr<int32_t>(), B,
                     batch_offset, static_cast<int32_t>(f1), static_cast<int32_t>(f2), seed,
                     out.data_ptr<float>(), capture ? s1.data_ptr<int32_t>() : nullptr,
                     capture ? s2.data_ptr<int32_t>() : nullptr, ws_ptr, ws_bytes,
                     clear_table.data_ptr<float>(), clear_rows.data_ptr<int32_t>(),
                     clear_rows.numel(), stream_of(x)),
                 "fsa_sample_agg_2hop_forward_zero_rows");
    return {out, s1, s2};
  }
  check_status(fsa_sample_agg_2hop_forward(
                   rowptr.data_ptr<int32_t>(), col.data_ptr<int32_t>(), x.size(0), col.numel(),
                   x.data_ptr<float>(), D, frontier.data_ptr<int32_t>(), B, batch_offset,
                   static_cast<int32_t>(f1), static_cast<int32_t>(f2), seed,
                   out.data_ptr<float>(), capture ? s1.data_ptr<int32_t>() : nullptr,
                   capture ? s2.data_ptr<int32_t>() : nullptr, ws_ptr, ws_bytes,
                   zero.defined() ? zero.data_ptr<float>() : nullptr,
                   zero.defined() ? zero.numel() : 0, stream_of(x)),
               "fsa_sample_agg_2hop_forward");
  return {out, s1, s2};
}

// fuseop/binding.cpp:200-231; `zeroed` is the buffer the forward zeroed.
Tensor backward_2hop(const Tensor& grad_out, const Tensor& s1, const Tensor& s2,
                     int64_t num_nodes, const Tensor& zeroed_buf) {
  TORCH_CHECK(grad_out.is_cuda() && s1.is_cuda() && s2.is_cuda(),
              "backward inputs must be CUDA tensors");
  TORCH_CHECK(grad_out.scalar_type() == at::kFloat && s1.scalar_type() == at::kInt &&
                  s2.scalar_type() == at::kInt,
              "invalid backward input dtypes");
  TORCH_CHECK(grad_out.dim() == 2 && s1.dim() == 2 && s2.dim() == 3 &&
                  s1.size(0) == grad_out.size(0) && s2.size(0) == grad_out.size(0) &&
                  s2.size(1) == s1.size(1),
              "saved sample shapes do not match grad_out");
  TORCH_CHECK(grad_out.device() == s1.device() && s1.device() == s2.device(),
              "backward inputs must be on the same CUDA device");
  TORCH_CHECK(grad_out.is_contiguous() && s1.is_contiguous() && s2.is_contiguous(),
              "backward inputs must be contiguous");
  TORCH_CHECK(num_nodes >= 0, "num_nodes must be non-negative");
  const int64_t B = grad_out.size(0);
  const int64_t D = grad_out.size(1);
  const c10::cuda::CUDAGuard guard(grad_out.device());
  Tensor grad_x;
  if (zeroed_buf.defined() && zeroed_buf.size(0) == num_nodes && zeroed_buf.size(1) == D &&
      zeroed_buf.device() == grad_out.device()) {
    grad_x = zeroed_buf;
  } else {
    grad_x = zeroed(num_nodes, D, grad_out);
  }
  const int64_t f1 = s1.size(1);
  const int64_t f2 = s2.size(2);
  if (B == 0 || f1 == 0 || f2 == 0) return grad_x;
  check_status(fsa_sample_agg_2hop_backward(grad_out.data_ptr<float>(), s1.data_ptr<int32_t>(),
                                            s2.data_ptr<int32_t>(), B, D,
                                            static_cast<int32_t>(f1), static_cast<int32_t>(f2),
                                            grad_x.data_ptr<float>(), num_nodes,
                                            stream_of(grad_out)),
               "fsa_sample_agg_2hop_backward");
  return grad_x;
}

// Dense gradient buffers that 2-hop forwards allocated (and zeroed) ahead of
// their backward, one per feature table at most.  A forward allocates one
// only when no other forward over the same table holds one that its
// backward has not taken yet; later forwards leave the fill to their own
// backward, as the reference does for every call (fuseop/binding.cpp:220).
// So k forwards before their backwards (gradient accumulation, several
// encoder calls per step) hold at most one extra N x D buffer, not k.  The
// table is keyed by the feature tensor's TensorImpl and holds weak
// references: a buffer whose graph was dropped without a backward is freed
// with it and no longer counts.
class ForwardBuffers {
 public:
  using Weak = c10::weak_intrusive_ptr<c10::TensorImpl, c10::UndefinedTensorImpl>;

  // A new zeroing target for a forward over `x`, or an undefined tensor when
  // another forward over x still holds one.
  Tensor claim(const Tensor& x) {
    const std::lock_guard<std::mutex> lock(mu_);
    for (auto it = held_.begin(); it != held_.end();) {
      it = it->second.expired() ? held_.erase(it) : std::next(it);
    }
    const auto* key = x.unsafeGetTensorImpl();
    if (held_.count(key) != 0) return Tensor();
    Tensor buf = at::empty({x.size(0), x.size(1)}, x.options().dtype(at::kFloat));
    held_.emplace(key, Weak(buf.getIntrusivePtr()));
    return buf;
  }

  // The backward of the forward over the table `key` took `buf`.
  void release(int64_t key, const Tensor& buf) {
    const std::lock_guard<std::mutex> lock(mu_);
    auto it = held_.find(reinterpret_cast<const c10::TensorImpl*>(key));
    if (it != held_.end() && it->second.lock().get() == buf.unsafeGetTensorImpl()) {
      held_.erase(it);
    }
  }

 private:
  std::mutex mu_;
  std::unordered_map<const c10::TensorImpl*, Weak> held_;
};

ForwardBuffers& forward_buffers() {
  static ForwardBuffers* b = new ForwardBuffers();  // never destroyed: used at exit
  return *b;
}

// fuseop/__init__.py:108-161.  When the backward will need the dense feature
// gradient, the forward allocates it (at most one pending per table, see
// ForwardBuffers) and the library's draw kernel zeroes it (bound by integer
// issue, it leaves HBM bandwidth idle that the fill uses); the reference
// zero-fills inside the backward (fuseop/binding.cpp:220), as this backward
// does when the forward held no buffer.
struct SampleAgg2Hop : public torch::autograd::Function<SampleAgg2Hop> {
  static Tensor forward(AutogradContext* ctx, const Tensor& rowptr, const Tensor& col,
                        const Tensor& x, const Tensor& frontier, int64_t f1, int64_t f2,
                        uint64_t seed, bool capture, bool grad_needed, int64_t batch_offset) {
    Tensor grad_buffer;
    if (capture && grad_needed) {
      TORCH_CHECK(x.is_cuda() && x.dim() == 2, "expected x[N,D] on a CUDA device");
      grad_buffer = forward_buffers().claim(x);
    }
    auto [out, s1, s2] =
        forward_2hop(rowptr, col, x, frontier, f1, f2, seed, capture, batch_offset, grad_buffer);
    if (capture) ctx->save_for_backward({s1, s2});
    ctx->saved_data["capture"] = capture;
    ctx->saved_data["grad_needed"] = grad_needed;
    ctx->saved_data["num_nodes"] = x.size(0);
    if (grad_buffer.defined()) {
      ctx->saved_data["grad_buffer"] = grad_buffer;
      ctx->saved_data["table"] = reinterpret_cast<int64_t>(x.unsafeGetTensorImpl());
    }
    return out;
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    Tensor grad_x;
    if (ctx->saved_data["capture"].toBool() && ctx->saved_data["grad_needed"].toBool()) {
      auto saved = ctx->get_saved_variables();
      Tensor buf;
      auto it = ctx->saved_data.find("grad_buffer");
      if (it != ctx->saved_data.end()) {
        buf = it->second.toTensor();
        ctx->saved_data.erase(it);
        forward_buffers().release(ctx->saved_data["table"].toInt(), buf);
      }
      grad_x = backward_2hop(grads[0].contiguous(), saved[0], saved[1],
                             ctx->saved_data["num_nodes"].toInt(), buf);
    }
    return {Tensor(), Tensor(), grad_x, Tensor(), Tensor(), Tensor(), Tensor(), Tensor(),
            Tensor(), Tensor()};
  }
};

// ---------------------------------------------------------------------------
// Persistent gradient buffer (opt-in; no counterpart in the reference)
//
// The reference's backward returns a fresh dense N x D gradient every call
// (at::zeros, fuseop/binding.cpp:137, :220) -- 4 N D bytes of fill per step
// for a sparse update.  With a caller-held buffer the backward instead adds
// into that buffer and returns no gradient for x; the forward returns its
// saved ids and a host flag as well, so that the caller can clear exactly
// the rows the backward will touch (fsa_zero_rows_f32) instead of all N.
// The flag is 1 until the backward has added into the buffer.
// ---------------------------------------------------------------------------

void check_grad_into(const Tensor& into, const Tensor& x) {
  TORCH_CHECK(into.sizes() == x.sizes(), "grad_buffer shape must equal the features' shape (",
              into.sizes(), " vs ", x.sizes(), ")");
  TORCH_CHECK(into.is_cuda() && into.device() == x.device(),
              "grad_buffer must be on the features' CUDA device");
  TORCH_CHECK(into.scalar_type() == at::kFloat && into.dim() == 2 && into.is_contiguous(),
              "grad_buffer must be a contiguous float32 matrix");
}

Tensor pending_flag() { return at::ones({1}, at::TensorOptions().dtype(at::kInt)); }

struct SampleAgg2HopInto : public torch::autograd::Function<SampleAgg2HopInto> {
  static variable_list forward(AutogradContext* ctx, const Tensor& rowptr, const Tensor& col,
                               const Tensor& x, const Tensor& frontier, int64_t f1, int64_t f2,
                               uint64_t seed, int64_t batch_offset, const Tensor& into,
                               const Tensor& clear_rows) {
    auto [out, s1, s2] = forward_2hop(rowptr, col, x, frontier, f1, f2, seed, true,
                                      batch_offset, Tensor(), into, clear_rows);
    Tensor flag = pending_flag();
    ctx->save_for_backward({s1, s2});
    ctx->saved_data["into"] = into;
    ctx->saved_data["flag"] = flag;
    ctx->mark_non_differentiable({s2, flag});
    return {out, s2, flag};
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    auto saved = ctx->get_saved_variables();
    Tensor into = ctx->saved_data["into"].toTensor();
    if (grads[0].defined()) {
      const Tensor g = grads[0].contiguous();
      const c10::cuda::CUDAGuard guard(g.device());
      check_status(fsa_sample_agg_2hop_backward(
                       g.data_ptr<float>(), saved[0].data_ptr<int32_t>(),
                       saved[1].data_ptr<int32_t>(), g.size(0), g.size(1),
                       static_cast<int32_t>(saved[0].size(1)),
                       static_cast<int32_t>(saved[1].size(2)), into.data_ptr<float>(),
                       into.size(0), stream_of(g)),
                   "fsa_sample_agg_2hop_backward");
    }
    ctx->saved_data["flag"].toTensor().data_ptr<int32_t>()[0] = 0;
    return variable_list(10);
  }
};

// `clear_rows` (optional): saved ids whose rows of `into` are zeroed as part
// of this call (inside the sampling kernel when the row width allows).
std::vector<Tensor> sample_agg_2hop_into(const Tensor& rowptr, const Tensor& col,
                                         const Tensor& x, const Tensor& frontier, int64_t f1,
                                         int64_t f2, uint64_t seed, int64_t batch_offset,
                                         const Tensor& into,
                                         const c10::optional<Tensor>& clear_rows) {
  check_grad_into(into, x);
  // an empty list rather than an undefined tensor: autograd's apply needs a
  // device for every tensor argument
  Tensor rows = at::empty({0}, into.options().dtype(at::kInt));
  if (clear_rows.has_value() && clear_rows->defined()) {
    rows = *clear_rows;
    TORCH_CHECK(rows.is_cuda() && rows.device() == into.device() &&
                    rows.scalar_type() == at::kInt && rows.is_contiguous(),
                "clear_rows must be contiguous int32 on the buffer's device");
  }
  if (!(at::GradMode::is_enabled() && x.requires_grad())) {
    auto r = forward_2hop(rowptr, col, x, frontier, f1, f2, seed, false, batch_offset, Tensor(),
                          into, rows);
    return {std::get<0>(r), Tensor(), Tensor()};
  }
  return SampleAgg2HopInto::apply(rowptr, col, x, frontier, f1, f2, seed, batch_offset, into,
                                  rows);
}

struct SampleAgg1HopInto : public torch::autograd::Function<SampleAgg1HopInto> {
  static variable_list forward(AutogradContext* ctx, const Tensor& rowptr, const Tensor& col,
                               const Tensor& x, const Tensor& frontier, int64_t fanout,
                               uint64_t seed, int64_t batch_offset, const Tensor& into) {
    auto r = forward_1hop(rowptr, col, x, frontier, fanout, seed, true, batch_offset);
    Tensor flag = pending_flag();
    ctx->save_for_backward({r[1], r[2]});
    ctx->saved_data["into"] = into;
    ctx->saved_data["flag"] = flag;
    ctx->mark_non_differentiable({r[1], flag});
    return {r[0], r[1], flag};
  }

  static variable_list backward(AutogradContext* ctx, variable_list grads) {
    auto saved = ctx->get_saved_variables();
    Tensor into = ctx->saved_data["into"].toTensor();
    if (grads[0].defined() && saved[0].numel() > 0) {
      const Tensor g = grads[0].contiguous();
      const c10::cuda::CUDAGuard guard(g.device());
      check_status(fsa_sample_agg_backward(saved[0].data_ptr<int32_t>(),
                                           saved[1].data_ptr<int32_t>(), g.data_ptr<float>(),
                                           g.size(0), g.size(1),
                                           static_cast<int32_t>(saved[0].size(1)),
                                           into.data_ptr<float>(), into.size(0), stream_of(g)),
                   "fsa_sample_agg_backward");
    }
    ctx->saved_data["flag"].toTensor().data_ptr<int32_t>()[0] = 0;
    return variable_list(8);
  }
};

std::vector<Tensor> sample_agg_into(const Tensor& rowptr, const Tensor& col, const Tensor& x,
                                    const Tensor& frontier, int64_t fanout, uint64_t seed,
                                    int64_t batch_offset, const Tensor& into) {
  check_grad_into(into, x);
  if (!(at::GradMode::is_enabled() && x.requires_grad())) {
    auto r = forward_1hop(rowptr, col, x, frontier, fanout, seed, false, batch_offset);
    return {r[0], Tensor(), Tensor()};
  }
  return SampleAgg1HopInto::apply(rowptr, col, x, frontier, fanout, seed, batch_offset, into);
}

// Clears rows `rows` (saved ids; -1 entries skipped) of a persistent buffer.
void zero_rows(const Tensor& table, const Tensor& rows) {
  TORCH_CHECK(table.is_cuda() && rows.is_cuda() && table.device() == rows.device(),
              "zero_rows: tensors must be on one CUDA device");
  TORCH_CHECK(table.scalar_type() == at::kFloat && table.dim() == 2 && table.is_contiguous(),
              "zero_rows: table must be a contiguous float32 matrix");
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous(),
              "zero_rows: rows must be contiguous int32");
  const c10::cuda::CUDAGuard guard(table.device());
  check_status(fsa_zero_rows_f32(table.data_ptr<float>(), table.size(0), table.size(1),
                                 rows.data_ptr<int32_t>(), rows.numel(), stream_of(table)),
               "fsa_zero_rows_f32");
}

// The reference binding's backward entry points (fuseop/binding.cpp:119-145,
// :200-231, exported at :236-242): a saved-index replay into a fresh
// zero-filled gradient.
Tensor replay_backward_1hop(const Tensor& samples, const Tensor& takes, const Tensor& grad_out,
                            int64_t num_nodes) {
  return backward_1hop(samples, takes, grad_out, num_nodes);
}

Tensor replay_backward_2hop(const Tensor& grad_out, const Tensor& s1, const Tensor& s2,
                            int64_t num_nodes) {
  return backward_2hop(grad_out, s1, s2, num_nodes, Tensor());
}

Tensor sample_agg_2hop(const Tensor& rowptr, const Tensor& col, const Tensor& x,
                       const Tensor& frontier, int64_t f1, int64_t f2, uint64_t seed,
                       bool save_indices, int64_t batch_offset) {
  const bool grad_needed = at::GradMode::is_enabled() && x.requires_grad();
  const bool capture = save_indices || x.requires_grad();
  return SampleAgg2Hop::apply(rowptr, col, x, frontier, f1, f2, seed, capture, grad_needed,
                              batch_offset);
}

std::tuple<Tensor, Tensor, Tensor> sample_agg_2hop_with_samples(
    const Tensor& rowptr, const Tensor& col, const Tensor& x, const Tensor& frontier, int64_t f1,
    int64_t f2, uint64_t seed, int64_t batch_offset) {
  const at::AutoGradMode no_grad(false);
  return forward_2hop(rowptr, col, x, frontier, f1, f2, seed, true, batch_offset, Tensor());
}

}  // namespace

PYBIND11_MODULE(_fsa_torch, m) {
  m.doc() = "PyTorch binding of libfsa_sm100.so (autograd functions in C++)";
  m.def("sample_agg", &sample_agg);
  m.def("sample_agg_with_samples", &sample_agg_with_samples);
  m.def("sample_agg_2hop", &sample_agg_2hop);
  m.def("sample_agg_2hop_with_samples", &sample_agg_2hop_with_samples);
  m.def("sample_agg_backward", &replay_backward_1hop);
  m.def("sample_agg_2hop_backward", &replay_backward_2hop);
  m.def("sample_agg_into", &sample_agg_into);
  m.def("sample_agg_2hop_into", &sample_agg_2hop_into);
  m.def("zero_rows", &zero_rows);
}
