// torch dispatcher ops over the C ABIs of include/kda_sm100.h and
// include/st_fused_ops.h:
//   kda_b200::chunk_fwd / chunk_bwd            -> kda_fwd_sm100 / kda_bwd_sm100
//   st_b200::silu_mul / silu_mul_bwd           -> st_silu_mul_fwd / _bwd
//   st_b200::rmsnorm_residual / _bwd           -> st_rmsnorm_residual_fwd / _bwd
//   st_b200::cross_entropy / cross_entropy_bwd -> st_cross_entropy_fwd / _bwd
//
// The schemas and CUDA implementations live here, in C++, so a call costs a
// dispatcher hop and a few caching-allocator allocations instead of a Python
// function; fake (meta) implementations and autograd are registered from
// Python (simpletrain_b200/ops.py).  Outputs and the workspace come from the
// caching allocator and the kernels run on the current stream, so the ops can
// be captured in CUDA graphs.  Layout rules follow the ABI: a tensor whose
// innermost stride is not 1, whose other strides are not multiples of 8
// elements, or whose base is not 16-byte aligned is made contiguous first.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/kda_sm100.h"
#include "../../include/st_fused_ops.h"

namespace {

using at::Tensor;
using c10::optional;

bool abi_layout_ok(const Tensor &t) {
  if (t.stride(-1) != 1 && t.size(-1) != 1) return false;
  if (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) return false;
  for (int64_t i = 0; i + 1 < t.dim(); ++i)
    if (t.size(i) != 1 && t.stride(i) % 8) return false;
  return true;
}

Tensor prep(const Tensor &t) { return abi_layout_ok(t) ? t : t.contiguous(); }

// New [B, H, T, D] tensor in the dimension order of `like`: its strides when
// they are dense, else [B, T, H, D] memory when `like` is time-major (the KDA
// layer's projection views, models/kimi_k3.py:99-102, dense or not), else
// contiguous.  Keeps the layer's transpose + contiguous() after the scan free.
Tensor empty_in_order_of(const Tensor &like) {
  if (like.is_non_overlapping_and_dense()) return at::empty_like(like);
  if (like.stride(1) < like.stride(2))
    return at::empty({like.size(0), like.size(2), like.size(1), like.size(3)}, like.options()).transpose(1, 2);
  return at::empty(like.sizes(), like.options());
}

optional<Tensor> prep(const optional<Tensor> &t) {
  if (!t.has_value()) return t;
  return prep(*t);
}

kda_tensor desc(const Tensor *t) {
  kda_tensor d{nullptr, 0, 0, 0, 0};
  if (t == nullptr) return d;
  int64_t st[4];
  for (int i = 0; i < 4; ++i) st[i] = t->size(i) == 1 ? 0 : t->stride(i);
  d.data = t->data_ptr();
  d.stride_b = st[0];
  d.stride_h = st[1];
  d.stride_t = st[2];
  d.stride_d = 1;
  return d;
}

void *ptr(const Tensor *t) { return (t == nullptr || t->numel() == 0) ? nullptr : t->data_ptr(); }

int32_t dtype_code(const Tensor &q) {
  if (q.scalar_type() == at::kBFloat16) return KDA_DTYPE_BF16;
  if (q.scalar_type() == at::kHalf) return KDA_DTYPE_F16;
  TORCH_CHECK(false, "KDA sm_100a kernels take bf16/fp16 inputs, got ", q.scalar_type());
}

// per-device int32 word the kernels OR device-side error bits into (shared with Python)
std::mutex g_status_mu;
std::vector<Tensor> g_status;

Tensor status_word(const at::Device &dev) {
  std::lock_guard<std::mutex> lock(g_status_mu);
  const int idx = dev.index();
  if ((int)g_status.size() <= idx) g_status.resize(idx + 1);
  if (!g_status[idx].defined())
    g_status[idx] = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, idx));
  return g_status[idx];
}

void decay_fields(const optional<Tensor> &decay, const float **p, int64_t *sb, int64_t *sh, int64_t *sd) {
  *p = nullptr;
  *sb = *sh = *sd = 0;
  if (!decay.has_value()) return;
  const Tensor &d = *decay;
  TORCH_CHECK(d.dim() == 3 && d.scalar_type() == at::kFloat, "decay must be a float32 [B, H, D] view");
  *p = d.data_ptr<float>();
  *sb = d.size(0) == 1 ? 0 : d.stride(0);
  *sh = d.size(1) == 1 ? 0 : d.stride(1);
  *sd = d.size(2) == 1 ? 0 : d.stride(2);
}

// state-update semantics of the ops: 0 = K^T V (chunk-constant decay), 1 = the
// reference's literal K V^T, 2 = per-token decay
// Error messages format integers with std::to_string, never by streaming them
// into a std::ostream (which TORCH_CHECK does with its arguments): with this
// toolchain and torch build, an integer streamed inside an extension module
// crashed the process (SIGSEGV) instead of raising.
uint32_t mode_flags(int64_t mode) {
  TORCH_CHECK(mode >= 0 && mode <= 2, "mode must be 0 (corrected), 1 (literal) or 2 (per-step), got ",
              std::to_string(mode));
  return mode == 1 ? KDA_FLAG_LITERAL : (mode == 2 ? KDA_FLAG_PER_STEP : 0u);
}

void check(int rc, const char *what) {
  TORCH_CHECK(rc == KDA_OK, what, " failed: ", kda_status_string(rc), " (status ", std::to_string(rc), ")");
}

void check_inputs(const Tensor &q, const Tensor &k, const Tensor &v, const optional<Tensor> &g) {
  TORCH_CHECK(q.is_cuda(), "the KDA sm_100a kernels need CUDA tensors (there is no CPU path)");
  TORCH_CHECK(q.dim() == 4, "q must be [B, H, T, D]");
  auto same = [&](const Tensor &t, const char *n) {
    TORCH_CHECK(t.sizes() == q.sizes(), n, " shape must match q");
    TORCH_CHECK(t.scalar_type() == q.scalar_type() && t.device() == q.device(), n,
                " must match q's dtype and device");
  };
  same(k, "k");
  same(v, "v");
  if (g.has_value()) same(*g, "gate");
}

std::tuple<Tensor, Tensor> chunk_fwd(const Tensor &q_, const Tensor &k_, const Tensor &v_,
                                     const optional<Tensor> &g_, const optional<Tensor> &decay,
                                     double decay_scalar, const optional<Tensor> &s0, int64_t chunk, int64_t mode,
                                     bool want_state) {
  check_inputs(q_, k_, v_, g_);
  c10::cuda::CUDAGuard guard(q_.device());
  const Tensor q = prep(q_), k = prep(k_), v = prep(v_);
  const optional<Tensor> g = prep(g_);
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), D = q.size(3);
  const Tensor y = prep(empty_in_order_of(q));  // like the reference: keeps q's memory order
  const auto f32 = q.options().dtype(at::kFloat);
  const Tensor s_out = want_state ? at::empty({B, H, D, D}, f32) : at::empty({0}, f32);
  const optional<Tensor> s_in = s0.has_value() ? optional<Tensor>(s0->contiguous().to(at::kFloat)) : c10::nullopt;
  const uint32_t flags = mode_flags(mode);
  const size_t ws_bytes = kda_fwd_workspace_bytes((int32_t)B, (int32_t)H, (int32_t)T, (int32_t)D, (int32_t)chunk, flags);
  const Tensor ws = at::empty({(int64_t)ws_bytes}, q.options().dtype(at::kByte));
  kda_fwd_params p{};
  p.B = (int32_t)B; p.H = (int32_t)H; p.T = (int32_t)T; p.D = (int32_t)D; p.chunk = (int32_t)chunk;
  p.dtype = dtype_code(q);
  p.flags = flags;
  p.q = desc(&q); p.k = desc(&k); p.v = desc(&v); p.g = desc(g.has_value() ? &*g : nullptr); p.y = desc(&y);
  decay_fields(decay, &p.decay, &p.decay_stride_b, &p.decay_stride_h, &p.decay_stride_d);
  p.decay_scalar = decay_scalar;
  p.state_in = s_in.has_value() ? static_cast<const float *>(ptr(&*s_in)) : nullptr;
  p.state_out = want_state ? static_cast<float *>(ptr(&s_out)) : nullptr;
  p.workspace = ptr(&ws);
  p.workspace_bytes = ws_bytes;
  p.status = status_word(q.device()).data_ptr<int32_t>();
  check(kda_fwd_sm100(&p, c10::cuda::getCurrentCUDAStream(q.device().index()).stream()), "kda_fwd_sm100");
  return {y, s_out};
}

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> chunk_bwd(
    const Tensor &q_, const Tensor &k_, const Tensor &v_, const optional<Tensor> &g_, const Tensor &dy_,
    const optional<Tensor> &decay, double decay_scalar, const optional<Tensor> &s0, const optional<Tensor> &s_T,
    const optional<Tensor> &ds_T, int64_t chunk, int64_t mode, bool need_ddecay_, bool need_ds0) {
  (void)s_T;
  check_inputs(q_, k_, v_, g_);
  c10::cuda::CUDAGuard guard(q_.device());
  const Tensor q = prep(q_), k = prep(k_), v = prep(v_), dy = prep(dy_);
  const optional<Tensor> g = prep(g_);
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), D = q.size(3);
  const Tensor dq = prep(empty_in_order_of(q)), dk = prep(empty_in_order_of(k)), dv = prep(empty_in_order_of(v));
  const Tensor dg = g.has_value() ? prep(empty_in_order_of(*g)) : at::empty({0}, q.options());
  const bool need_ddecay = need_ddecay_ && decay.has_value();
  const auto f32 = q.options().dtype(at::kFloat);
  const Tensor ddecay = need_ddecay ? at::empty({B, H, D}, f32) : at::empty({0}, f32);
  const Tensor ds0 = need_ds0 ? at::empty({B, H, D, D}, f32) : at::empty({0}, f32);
  const optional<Tensor> s_in = s0.has_value() ? optional<Tensor>(s0->contiguous().to(at::kFloat)) : c10::nullopt;
  const optional<Tensor> dsT = (ds_T.has_value() && ds_T->numel() > 0)
                                   ? optional<Tensor>(ds_T->contiguous().to(at::kFloat))
                                   : c10::nullopt;
  const uint32_t flags = mode_flags(mode);
  const size_t ws_bytes = kda_bwd_workspace_bytes((int32_t)B, (int32_t)H, (int32_t)T, (int32_t)D, (int32_t)chunk, flags);
  const Tensor ws = at::empty({(int64_t)ws_bytes}, q.options().dtype(at::kByte));
  kda_bwd_params p{};
  p.B = (int32_t)B; p.H = (int32_t)H; p.T = (int32_t)T; p.D = (int32_t)D; p.chunk = (int32_t)chunk;
  p.dtype = dtype_code(q);
  p.flags = flags;
  p.q = desc(&q); p.k = desc(&k); p.v = desc(&v); p.g = desc(g.has_value() ? &*g : nullptr); p.dy = desc(&dy);
  p.dq = desc(&dq); p.dk = desc(&dk); p.dv = desc(&dv); p.dg = desc(g.has_value() ? &dg : nullptr);
  decay_fields(decay, &p.decay, &p.decay_stride_b, &p.decay_stride_h, &p.decay_stride_d);
  p.decay_scalar = decay_scalar;
  p.state_in = s_in.has_value() ? static_cast<const float *>(ptr(&*s_in)) : nullptr;
  p.dstate_out = dsT.has_value() ? static_cast<const float *>(ptr(&*dsT)) : nullptr;
  p.dstate_in = need_ds0 ? static_cast<float *>(ptr(&ds0)) : nullptr;
  p.ddecay = need_ddecay ? static_cast<float *>(ptr(&ddecay)) : nullptr;
  p.workspace = ptr(&ws);
  p.workspace_bytes = ws_bytes;
  p.status = status_word(q.device()).data_ptr<int32_t>();
  check(kda_bwd_sm100(&p, c10::cuda::getCurrentCUDAStream(q.device().index()).stream()), "kda_bwd_sm100");
  return {dq, dk, dv, dg, ddecay, ds0};
}

// The status word the kernels write (Python reads and clears it).
Tensor status(int64_t device) { return status_word(at::Device(at::kCUDA, (c10::DeviceIndex)device)); }

// ------------------------------------------------ fused elementwise / row ops
int32_t dtype16(const Tensor &t) {
  TORCH_CHECK(t.is_cuda(), "the sm_100a fused ops need CUDA tensors (there is no CPU path)");
  return dtype_code(t);
}
cudaStream_t stream_of(const Tensor &t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

Tensor silu_mul(const Tensor &a_, const Tensor &b_) {
  TORCH_CHECK(a_.sizes() == b_.sizes() && a_.scalar_type() == b_.scalar_type(), "silu_mul: a and b must match");
  c10::cuda::CUDAGuard guard(a_.device());
  const Tensor a = a_.contiguous(), b = b_.contiguous();
  Tensor out = at::empty_like(a);
  check(st_silu_mul_fwd(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), dtype16(a), stream_of(a)),
        "st_silu_mul_fwd");
  return out;
}

std::tuple<Tensor, Tensor> silu_mul_bwd(const Tensor &a_, const Tensor &b_, const Tensor &g_) {
  c10::cuda::CUDAGuard guard(a_.device());
  const Tensor a = a_.contiguous(), b = b_.contiguous(), g = g_.contiguous().to(a.scalar_type());
  Tensor da = at::empty_like(a), db = at::empty_like(b);
  check(st_silu_mul_bwd(a.data_ptr(), b.data_ptr(), g.data_ptr(), da.data_ptr(), db.data_ptr(), a.numel(),
                        dtype16(a), stream_of(a)),
        "st_silu_mul_bwd");
  return {da, db};
}

std::tuple<Tensor, Tensor> rmsnorm_residual(const Tensor &x_, const Tensor &r_, const Tensor &w_, double eps) {
  TORCH_CHECK(x_.sizes() == r_.sizes(), "rmsnorm_residual: x and residual must match");
  TORCH_CHECK(w_.dim() == 1 && w_.size(0) == x_.size(-1), "rmsnorm_residual: weight must be [D]");
  c10::cuda::CUDAGuard guard(x_.device());
  const Tensor x = x_.contiguous(), r = r_.contiguous().to(x.scalar_type()), w = w_.contiguous().to(x.scalar_type());
  const int64_t D = x.size(-1), N = D ? x.numel() / D : 0;
  Tensor out = at::empty_like(x);
  Tensor rstd = at::empty(x.sizes().slice(0, x.dim() - 1), x.options().dtype(at::kFloat));
  check(st_rmsnorm_residual_fwd(x.data_ptr(), r.data_ptr(), w.data_ptr(), out.data_ptr(), rstd.data_ptr<float>(), N,
                                D, (float)eps, dtype16(x), stream_of(x)),
        "st_rmsnorm_residual_fwd");
  return {out, rstd};
}

std::tuple<Tensor, Tensor> rmsnorm_residual_bwd(const Tensor &x_, const Tensor &w_, const Tensor &rstd_,
                                                const Tensor &dy_) {
  c10::cuda::CUDAGuard guard(x_.device());
  const Tensor x = x_.contiguous(), w = w_.contiguous().to(x.scalar_type()), rstd = rstd_.contiguous(),
               dy = dy_.contiguous().to(x.scalar_type());
  const int64_t D = x.size(-1), N = D ? x.numel() / D : 0;
  Tensor dx = at::empty_like(x);
  Tensor dw = at::empty({D}, x.options().dtype(at::kFloat));
  Tensor scratch = at::empty({(int64_t)(st_rmsnorm_residual_bwd_scratch(N, D) / sizeof(float)) + 1},
                             x.options().dtype(at::kFloat));
  check(st_rmsnorm_residual_bwd(x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), dy.data_ptr(), dx.data_ptr(),
                                dw.data_ptr<float>(), scratch.data_ptr<float>(), N, D, dtype16(x), stream_of(x)),
        "st_rmsnorm_residual_bwd");
  return {dx, dw};
}

std::tuple<Tensor, Tensor, Tensor> cross_entropy(const Tensor &logits_, const Tensor &labels_, bool want_probs) {
  TORCH_CHECK(logits_.dim() == 2, "cross_entropy: logits must be [N, V]");
  TORCH_CHECK(labels_.dim() == 1 && labels_.size(0) == logits_.size(0), "cross_entropy: labels must be [N]");
  c10::cuda::CUDAGuard guard(logits_.device());
  const Tensor logits = logits_.contiguous(), labels = labels_.contiguous().to(at::kLong);
  const int64_t N = logits.size(0), V = logits.size(1);
  const auto f32 = logits.options().dtype(at::kFloat);
  Tensor loss = at::empty({N}, f32), lse = at::empty({N}, f32);
  Tensor probs = want_probs ? at::empty_like(logits) : at::empty({0}, logits.options());
  check(st_cross_entropy_fwd(logits.data_ptr(), labels.data_ptr<int64_t>(), loss.data_ptr<float>(),
                             lse.data_ptr<float>(), want_probs ? probs.data_ptr() : nullptr, N, V, dtype16(logits),
                             stream_of(logits)),
        "st_cross_entropy_fwd");
  return {loss, lse, probs};
}

Tensor cross_entropy_bwd(const Tensor &logits_, const Tensor &labels_, const Tensor &lse_, const Tensor &dloss_) {
  c10::cuda::CUDAGuard guard(logits_.device());
  const Tensor logits = logits_.contiguous(), labels = labels_.contiguous().to(at::kLong), lse = lse_.contiguous(),
               dloss = dloss_.contiguous().to(at::kFloat);
  const int64_t N = logits.size(0), V = logits.size(1);
  Tensor dlogits = at::empty_like(logits);
  check(st_cross_entropy_bwd(logits.data_ptr(), labels.data_ptr<int64_t>(), lse.data_ptr<float>(),
                             dloss.data_ptr<float>(), dlogits.data_ptr(), N, V, dtype16(logits), stream_of(logits)),
        "st_cross_entropy_bwd");
  return dlogits;
}

}  // namespace

TORCH_LIBRARY(st_b200, m) {
  m.def("silu_mul(Tensor a, Tensor b) -> Tensor");
  m.def("silu_mul_bwd(Tensor a, Tensor b, Tensor dout) -> (Tensor, Tensor)");
  m.def("rmsnorm_residual(Tensor x, Tensor residual, Tensor weight, float eps) -> (Tensor, Tensor)");
  m.def("rmsnorm_residual_bwd(Tensor x, Tensor weight, Tensor rstd, Tensor dy) -> (Tensor, Tensor)");
  m.def("cross_entropy(Tensor logits, Tensor labels, bool want_probs) -> (Tensor, Tensor, Tensor)");
  m.def("cross_entropy_bwd(Tensor logits, Tensor labels, Tensor lse, Tensor dloss) -> Tensor");
}

TORCH_LIBRARY_IMPL(st_b200, CUDA, m) {
  m.impl("silu_mul", &silu_mul);
  m.impl("silu_mul_bwd", &silu_mul_bwd);
  m.impl("rmsnorm_residual", &rmsnorm_residual);
  m.impl("rmsnorm_residual_bwd", &rmsnorm_residual_bwd);
  m.impl("cross_entropy", &cross_entropy);
  m.impl("cross_entropy_bwd", &cross_entropy_bwd);
}

TORCH_LIBRARY(kda_b200, m) {
  m.def(
      "chunk_fwd(Tensor q, Tensor k, Tensor v, Tensor? g, Tensor? decay, float decay_scalar, Tensor? s0, "
      "int chunk, int mode, bool want_state) -> (Tensor, Tensor)");
  m.def(
      "chunk_bwd(Tensor q, Tensor k, Tensor v, Tensor? g, Tensor dy, Tensor? decay, float decay_scalar, "
      "Tensor? s0, Tensor? s_T, Tensor? ds_T, int chunk, int mode, bool need_ddecay, bool need_ds0) "
      "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("status_word(int device) -> Tensor");
}

TORCH_LIBRARY_IMPL(kda_b200, CUDA, m) {
  m.impl("chunk_fwd", &chunk_fwd);
  m.impl("chunk_bwd", &chunk_bwd);
}

TORCH_LIBRARY_IMPL(kda_b200, CompositeExplicitAutograd, m) { m.impl("status_word", &status); }
