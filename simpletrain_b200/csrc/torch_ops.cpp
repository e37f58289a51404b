// torch dispatcher ops over the C ABI of include/kda_sm100.h:
//   kda_b200::chunk_fwd  -> kda_fwd_sm100
//   kda_b200::chunk_bwd  -> kda_bwd_sm100
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
#include <tuple>
#include <vector>

#include "../../include/kda_sm100.h"

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

void check(int rc, const char *what) {
  TORCH_CHECK(rc == KDA_OK, what, " failed: ", kda_status_string(rc), " (status ", rc, ")");
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
                                     double decay_scalar, const optional<Tensor> &s0, int64_t chunk, bool literal,
                                     bool want_state) {
  check_inputs(q_, k_, v_, g_);
  c10::cuda::CUDAGuard guard(q_.device());
  const Tensor q = prep(q_), k = prep(k_), v = prep(v_);
  const optional<Tensor> g = prep(g_);
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), D = q.size(3);
  const Tensor y = prep(at::empty_like(q));  // like the reference: keeps q's memory order
  const auto f32 = q.options().dtype(at::kFloat);
  const Tensor s_out = want_state ? at::empty({B, H, D, D}, f32) : at::empty({0}, f32);
  const optional<Tensor> s_in = s0.has_value() ? optional<Tensor>(s0->contiguous().to(at::kFloat)) : c10::nullopt;
  const uint32_t flags = literal ? KDA_FLAG_LITERAL : 0u;
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
    const optional<Tensor> &ds_T, int64_t chunk, bool literal, bool need_ddecay_, bool need_ds0) {
  (void)s_T;
  check_inputs(q_, k_, v_, g_);
  c10::cuda::CUDAGuard guard(q_.device());
  const Tensor q = prep(q_), k = prep(k_), v = prep(v_), dy = prep(dy_);
  const optional<Tensor> g = prep(g_);
  const int64_t B = q.size(0), H = q.size(1), T = q.size(2), D = q.size(3);
  const Tensor dq = prep(at::empty_like(q)), dk = prep(at::empty_like(k)), dv = prep(at::empty_like(v));
  const Tensor dg = g.has_value() ? prep(at::empty_like(*g)) : at::empty({0}, q.options());
  const bool need_ddecay = need_ddecay_ && decay.has_value();
  const auto f32 = q.options().dtype(at::kFloat);
  const Tensor ddecay = need_ddecay ? at::empty({B, H, D}, f32) : at::empty({0}, f32);
  const Tensor ds0 = need_ds0 ? at::empty({B, H, D, D}, f32) : at::empty({0}, f32);
  const optional<Tensor> s_in = s0.has_value() ? optional<Tensor>(s0->contiguous().to(at::kFloat)) : c10::nullopt;
  const optional<Tensor> dsT = (ds_T.has_value() && ds_T->numel() > 0)
                                   ? optional<Tensor>(ds_T->contiguous().to(at::kFloat))
                                   : c10::nullopt;
  const uint32_t flags = literal ? KDA_FLAG_LITERAL : 0u;
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

}  // namespace

TORCH_LIBRARY(kda_b200, m) {
  m.def(
      "chunk_fwd(Tensor q, Tensor k, Tensor v, Tensor? g, Tensor? decay, float decay_scalar, Tensor? s0, "
      "int chunk, bool literal, bool want_state) -> (Tensor, Tensor)");
  m.def(
      "chunk_bwd(Tensor q, Tensor k, Tensor v, Tensor? g, Tensor dy, Tensor? decay, float decay_scalar, "
      "Tensor? s0, Tensor? s_T, Tensor? ds_T, int chunk, bool literal, bool need_ddecay, bool need_ds0) "
      "-> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("status_word(int device) -> Tensor");
}

TORCH_LIBRARY_IMPL(kda_b200, CUDA, m) {
  m.impl("chunk_fwd", &chunk_fwd);
  m.impl("chunk_bwd", &chunk_bwd);
}

TORCH_LIBRARY_IMPL(kda_b200, CompositeExplicitAutograd, m) { m.impl("status_word", &status); }
