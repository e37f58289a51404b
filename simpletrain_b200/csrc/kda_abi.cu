// C-ABI entry points: argument validation and kernel dispatch.
//
// Mirrors the checks SimpleTrain's dispatch relies on (kernels/kda_kernel.py:
// the Triton wrapper's dtype assert at :204, the head-dim cap at :216-219 and
// the broadcast failure of the literal state update at :294-295) but reports
// them as status codes instead of exceptions or silent fallbacks.
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "kda_internal.h"
#include "kda_tc_epi.cuh"

namespace {
std::atomic<uint64_t> g_launches{0};

// Launch tracer: a CUDA event pair around each traced launch, on its stream.
struct Tracer {
  std::mutex mu;
  std::atomic<bool> on{false};
  int dev = -1;
  int used = 0;
  std::vector<cudaEvent_t> ev;  // 2 per slot: before, after
  std::vector<int> kernel;
};
Tracer g_trace;

// An event record on `st`: a plain record, or, while `st` is being captured
// into a CUDA graph, an event-record node of the graph (recorded at every
// replay).
void trace_record(cudaEvent_t ev, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, st);
}

// Elapsed times of the first min(used, cap) slots (the caller holds the lock).
int32_t trace_collect(float *ms, int32_t *kernel, int32_t cap) {
  const int n = g_trace.used;
  for (int i = 0; i < n && i < cap && ms != nullptr && kernel != nullptr; ++i) {
    float t = 0.f;
    if (g_trace.kernel[i] < 0) {  // the launch itself failed: nothing to time
      ms[i] = 0.f;
      kernel[i] = -1;
      continue;
    }
    if (cudaEventSynchronize(g_trace.ev[2 * i + 1]) != cudaSuccess ||
        cudaEventElapsedTime(&t, g_trace.ev[2 * i], g_trace.ev[2 * i + 1]) != cudaSuccess) {
      cudaGetLastError();
      return -KDA_ERR_CUDA;
    }
    ms[i] = t;
    kernel[i] = g_trace.kernel[i];
  }
  return n;
}

void trace_release() {
  for (cudaEvent_t e : g_trace.ev) cudaEventDestroy(e);
  g_trace.ev.clear();
  g_trace.kernel.clear();
  g_trace.used = 0;
}
}  // namespace

void kda::count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int kda::trace_before(cudaStream_t st) {
  if (!g_trace.on.load(std::memory_order_acquire)) return -1;
  std::lock_guard<std::mutex> lock(g_trace.mu);
  int dev = -1;
  if (!g_trace.on.load(std::memory_order_relaxed) || cudaGetDevice(&dev) != cudaSuccess || dev != g_trace.dev ||
      g_trace.used >= (int)g_trace.kernel.size())
    return -1;
  const int slot = g_trace.used++;
  g_trace.kernel[slot] = -1;
  trace_record(g_trace.ev[2 * slot], st);
  return slot;
}

void kda::trace_after(int slot, int kernel, cudaStream_t st) {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lock(g_trace.mu);
  if (slot >= (int)g_trace.kernel.size()) return;
  g_trace.kernel[slot] = kernel;
  trace_record(g_trace.ev[2 * slot + 1], st);
}

namespace {

using kda::View;

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_view(const kda_tensor &t, bool required) {
  if (t.data == nullptr) return required ? KDA_ERR_NULL_ARGUMENT : KDA_OK;
  if (t.stride_d != 1) return KDA_ERR_BAD_LAYOUT;
  if (!aligned16(t.data)) return KDA_ERR_BAD_LAYOUT;
  if ((t.stride_b % 8) || (t.stride_h % 8) || (t.stride_t % 8)) return KDA_ERR_BAD_LAYOUT;
  if (t.stride_b < 0 || t.stride_h < 0 || t.stride_t < 0) return KDA_ERR_BAD_LAYOUT;
  return KDA_OK;
}

View to_view(const kda_tensor &t) { return View{t.data, t.stride_b, t.stride_h, t.stride_t, t.stride_d}; }

int check_common(int32_t B, int32_t H, int32_t T, int32_t D, int32_t chunk, int32_t dtype, uint32_t flags) {
  if (B < 0 || H < 0 || T < 0 || D <= 0 || chunk <= 0) return KDA_ERR_BAD_SHAPE;
  if (dtype != KDA_DTYPE_BF16 && dtype != KDA_DTYPE_F16) return KDA_ERR_UNSUPPORTED;
  if (chunk != 64) return KDA_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return KDA_ERR_UNSUPPORTED;
  if (flags & ~uint32_t(KDA_FLAG_LITERAL | KDA_FLAG_PER_STEP)) return KDA_ERR_UNSUPPORTED;
  if ((flags & KDA_FLAG_LITERAL) && (flags & KDA_FLAG_PER_STEP)) return KDA_ERR_UNSUPPORTED;
  if ((flags & KDA_FLAG_LITERAL) && D != chunk) return KDA_ERR_BAD_SHAPE;
  return KDA_OK;
}

// Per-step mode: one decay per (batch, head) within the range the row scaling
// allows: powers a^-32 .. a^32 of it scale 16-bit operands, so bf16 takes
// 0.125 <= a <= 1 and fp16 (max 65504, normal above 6.1e-5) 0.9 <= a <= 1.
int check_per_step(uint32_t flags, int32_t dtype, const float *decay, int64_t stride_d, double scalar) {
  if (!(flags & KDA_FLAG_PER_STEP)) return KDA_OK;
  if (decay != nullptr) return stride_d == 0 ? KDA_OK : KDA_ERR_UNSUPPORTED;
  const double lo = dtype == KDA_DTYPE_F16 ? 0.9 : 0.125;
  return (scalar >= lo && scalar <= 1.0) ? KDA_OK : KDA_ERR_UNSUPPORTED;
}

kda::DecaySrc make_decay(const float *ptr, int64_t sb, int64_t sh, int64_t sd, double scalar, int T,
                         int C) {
  kda::DecaySrc s{};
  s.ptr = ptr;
  s.sb = sb;
  s.sh = sh;
  s.sd = sd;
  s.scalar = scalar;
  // python: (decay ** L) computed in double, then used as an fp32 scalar factor
  s.alpha_full = (float)std::pow(scalar, (double)C);
  s.alpha_tail = (float)std::pow(scalar, (double)(T % C == 0 ? C : T % C));
  return s;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? KDA_OK : KDA_ERR_CUDA; }

// ---- persistent work queue (see kda_tc_epi.cuh) ----------------------------
// float4 per epilogue thread of one fp32 D x D carry
int carry_f4(int D) { return D * D / (4 * kda::tc::kEpi); }

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// Tuning override: KDA_SM100_RANGES=<ranges per launch> (0 or unset: one per CTA slot).
int ranges_override() {
  static const int v = [] {
    const char *s = std::getenv("KDA_SM100_RANGES");
    return s ? std::atoi(s) : 0;
  }();
  return v;
}

// Ranges of one launch: one per resident CTA slot, at most one per chunk.  With
// fewer streams than slots but at least 3/5 as many, one range per stream
// instead: cutting streams there puts ranges inside streams, whose carries then
// need the range aggregates (a pass over k and v before the main kernel), and
// that costs more than the idle slots.  Measured on 148 slots, fwd+bwd per step,
// D=128, streams of 32 chunks, one range per stream against cut: 120 streams
// 0.293 / 0.350 ms, 104: 0.288 / 0.321, 96: 0.285 / 0.301, 88: 0.283 / 0.282,
// 80: 0.286 / 0.267; D=64, 80 streams: 0.188 / 0.164.
//
// Cut ranges hold at least KDA_SM100_MIN_CHUNKS chunks (default 4): a range's
// fixed cost (setting up its pipeline, the fold of its entry carry, its share
// of the decay gradient) is paid per range, so one short stream cut into one
// range per CTA slot (a stream split in time between GPUs) runs faster on
// fewer, longer ranges.
int min_chunks_per_range() {
  static const int v = [] {
    const char *s = std::getenv("KDA_SM100_MIN_CHUNKS");
    const int m = s ? std::atoi(s) : 4;
    return m > 0 ? m : 1;
  }();
  return v;
}

int n_ranges(int nstreams, int nchunks, int slots) {
  const long long n = (long long)nstreams * nchunks;
  long long want = slots;
  if (ranges_override() > 0) want = ranges_override();
  else if (nstreams < slots && 5LL * nstreams >= 3LL * slots) want = nstreams;
  else if (nstreams < slots) {
    const long long cap = (n + min_chunks_per_range() - 1) / min_chunks_per_range();
    if (cap < want) want = cap > nstreams ? cap : nstreams;
  }
  return (int)(n < want ? n : want);
}

// CTA slots of each kernel on the current device (the launch and the workspace
// query agree because both ask the same device).
int fwd_slots(int D, uint32_t flags) {
  const bool literal = (flags & KDA_FLAG_LITERAL) != 0, per_step = (flags & KDA_FLAG_PER_STEP) != 0;
  static std::atomic<int> cache[8];  // CTAs per SM by (D == 128, literal, per-step); 0 = not asked yet
  std::atomic<int> &c = cache[(D == 128 ? 4 : 0) + (literal ? 1 : 0) + (per_step ? 2 : 0)];
  int occ = c.load(std::memory_order_relaxed);
  if (occ == 0) {
    const int a = kda::fwd_tc_occupancy(D, KDA_DTYPE_BF16, literal, per_step);
    const int b = kda::fwd_tc_occupancy(D, KDA_DTYPE_F16, literal, per_step);
    occ = a > b ? a : b;
    c.store(occ, std::memory_order_relaxed);
  }
  return sm_count() * occ;
}
int bwd_slots() { return sm_count(); }

// workspace of one queue: [ticket][flags: nranges+1 ints][slots: (nranges+1) x slot_f4 x 256 float4]
size_t queue_header_bytes(int nranges) { return align256(16 + 4 * ((size_t)nranges + 1)); }
size_t queue_bytes(int nranges, int slot_f4) {
  if (nranges <= 0) return 0;
  return queue_header_bytes(nranges) + ((size_t)nranges + 1) * slot_f4 * kda::tc::kEpi * 16;
}

// Whether some range lies strictly inside one stream (starts and ends
// mid-stream): then the carry would pass through a chain of ranges, and the
// aggregates of every publishing piece are precomputed so each link costs
// only a combine.
bool has_middle(int nstreams, int nchunks, int nranges) {
  if (nchunks <= 0 || nranges <= 0) return false;
  const long long n = (long long)nstreams * nchunks;
  for (int r = 0; r < nranges; ++r) {
    const long long lo = n * r / nranges, hi = n * (r + 1) / nranges;
    const long long s0 = lo / nchunks, s1 = (hi - 1) / nchunks;
    if (s0 == s1 && lo - s0 * nchunks > 0 && hi - s1 * nchunks < nchunks) return true;
  }
  return false;
}

// aggregate buffer of one queue: nranges x agg_f4 x 256 float4 (only when some range is a middle range)
size_t agg_bytes(int nstreams, int nchunks, int nranges, int agg_f4) {
  return has_middle(nstreams, nchunks, nranges) ? (size_t)nranges * agg_f4 * kda::tc::kEpi * 16 : 0;
}

// Lay a queue (and its aggregates at `agg`, if any) over `ws` and clear its header on the stream.
cudaError_t make_queue(kda::tc::Queue &q, void *ws, int nstreams, int nchunks, int slot_f4, int nranges, void *agg,
                       int agg_f4, cudaStream_t st) {
  q.ticket = reinterpret_cast<int *>(ws);
  q.flags = reinterpret_cast<int *>(reinterpret_cast<char *>(ws) + 16);
  q.slots = reinterpret_cast<float4 *>(reinterpret_cast<char *>(ws) + queue_header_bytes(nranges));
  q.slot_f4 = slot_f4;
  q.nstreams = nstreams;
  q.nchunks = nchunks;
  q.nranges = nranges;
  q.agg = has_middle(nstreams, nchunks, nranges) ? reinterpret_cast<float4 *>(agg) : nullptr;
  q.agg_f4 = agg_f4;
  return cudaMemsetAsync(ws, 0, queue_header_bytes(nranges), st);
}

size_t do_bytes(int B, int H, int T, int D) {
  return T > 0 ? align256((size_t)B * H * T * D * 2) : 0;
}

int n_chunks(int T, int chunk) { return chunk > 0 && T > 0 ? (T + chunk - 1) / chunk : 0; }

}  // namespace

extern "C" {

int32_t kda_abi_version(void) { return KDA_ABI_VERSION; }

uint64_t kda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int kda_trace_start(int32_t max_launches) {
  if (max_launches <= 0) return KDA_ERR_BAD_SHAPE;
  std::lock_guard<std::mutex> lock(g_trace.mu);
  g_trace.on.store(false, std::memory_order_release);
  trace_release();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KDA_ERR_CUDA;
  g_trace.ev.reserve(2 * (size_t)max_launches);
  for (int i = 0; i < 2 * max_launches; ++i) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
      trace_release();
      cudaGetLastError();
      return KDA_ERR_CUDA;
    }
    g_trace.ev.push_back(e);
  }
  g_trace.kernel.assign((size_t)max_launches, -1);
  g_trace.dev = dev;
  g_trace.on.store(true, std::memory_order_release);
  return KDA_OK;
}

int32_t kda_trace_read(float *ms, int32_t *kernel, int32_t cap) {
  std::lock_guard<std::mutex> lock(g_trace.mu);
  return trace_collect(ms, kernel, cap);
}

int32_t kda_trace_stop(float *ms, int32_t *kernel, int32_t cap) {
  std::lock_guard<std::mutex> lock(g_trace.mu);
  g_trace.on.store(false, std::memory_order_release);
  const int32_t rc = trace_collect(ms, kernel, cap);
  trace_release();
  return rc;
}

const char *kda_kernel_name(int32_t kernel) {
  switch (kernel) {
    case kda::kTraceFwd: return "fwd_tc_kernel";
    case kda::kTraceBwdFwdDir: return "bwd_fwddir_tc_kernel";
    case kda::kTraceBwdRevDir: return "bwd_revdir_tc_kernel";
    case kda::kTraceAgg: return "agg_tc_kernel";
    case kda::kTraceFold: return "entry_fold_kernel";
    default: return "unknown";
  }
}

const char *kda_status_string(int32_t s) {
  switch (s) {
    case KDA_OK: return "ok";
    case KDA_ERR_NULL_ARGUMENT: return "a required pointer argument is NULL";
    case KDA_ERR_BAD_SHAPE: return "invalid shape (negative size, or literal mode with D != chunk)";
    case KDA_ERR_UNSUPPORTED:
      return "unsupported configuration (head dim 64 or 128, chunk 64, dtype bf16/f16; per-step mode: not literal, "
             "one decay per (batch, head) in [0.125, 1] (fp16: [0.9, 1]), no decay gradient)";
    case KDA_ERR_BAD_LAYOUT: return "bad layout (innermost stride must be 1, other strides multiples of 8 elements, base 16-byte aligned)";
    case KDA_ERR_WORKSPACE: return "workspace missing or too small";
    case KDA_ERR_CUDA: return "CUDA launch or runtime error";
    case KDA_ERR_DEVICE_TIMEOUT: return "device-side bounded wait expired";
    default: return "unknown kda status";
  }
}

size_t kda_fwd_workspace_bytes(int32_t B, int32_t H, int32_t T, int32_t D, int32_t chunk, uint32_t flags) {
  if (B <= 0 || H <= 0 || (D != 64 && D != 128)) return 0;
  const int nc = n_chunks(T, chunk), nr = n_ranges(B * H, nc, fwd_slots(D, flags));
  return queue_bytes(nr, carry_f4(D)) + agg_bytes(B * H, nc, nr, carry_f4(D));
}

size_t kda_bwd_workspace_bytes(int32_t B, int32_t H, int32_t T, int32_t D, int32_t chunk, uint32_t) {
  if (B <= 0 || H <= 0 || (D != 64 && D != 128)) return 0;
  const int nc = n_chunks(T, chunk), nr = n_ranges(B * H, nc, bwd_slots());
  // forward-direction pass: state, decay tangent, decay-gradient share; reverse pass: dS;
  // then dO = dy * g, [B][H][T][D] 16-bit, handed from the first pass to the second;
  // then the range aggregates of both passes (long streams)
  return queue_bytes(nr, 2 * carry_f4(D) + 1) + queue_bytes(nr, carry_f4(D)) + do_bytes(B, H, T, D) +
         agg_bytes(B * H, nc, nr, 2 * carry_f4(D)) + agg_bytes(B * H, nc, nr, carry_f4(D));
}

}  // extern "C"

// Every argument check of kda_fwd_sm100 except the workspace's (shared with
// kda_fwd_sm100_noalloc, which checks its scratch size only after these).
int kda::fwd_check_args(const kda_fwd_params *p) {
  if (p == nullptr) return KDA_ERR_NULL_ARGUMENT;
  int rc = check_common(p->B, p->H, p->T, p->D, p->chunk, p->dtype, p->flags);
  if (rc) return rc;
  const bool literal = (p->flags & KDA_FLAG_LITERAL) != 0;
  if (literal && p->state_out && (p->T % p->chunk) != 0) return KDA_ERR_BAD_SHAPE;
  if ((rc = check_per_step(p->flags, p->dtype, p->decay, p->decay_stride_d, p->decay_scalar))) return rc;
  if ((p->state_in && !aligned16(p->state_in)) || (p->state_out && !aligned16(p->state_out)))
    return KDA_ERR_BAD_LAYOUT;
  if (p->B == 0 || p->H == 0 || p->T == 0) return KDA_OK;  // no sequence is read or written
  if ((rc = check_view(p->q, true)) || (rc = check_view(p->k, true)) || (rc = check_view(p->v, true)) ||
      (rc = check_view(p->g, false)) || (rc = check_view(p->y, true)))
    return rc;
  return KDA_OK;
}

extern "C" {

int kda_fwd_sm100(const kda_fwd_params *p, kda_stream_t stream) {
  int rc = kda::fwd_check_args(p);
  if (rc) return rc;
  const bool literal = (p->flags & KDA_FLAG_LITERAL) != 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->H == 0) return KDA_OK;  // nothing to read or write
  if (p->T == 0) {
    // empty sequence: the final state is the initial one
    if (p->state_out) {
      const size_t n = (size_t)p->B * p->H * p->D * p->D * sizeof(float);
      cudaError_t e = p->state_in ? cudaMemcpyAsync(p->state_out, p->state_in, n, cudaMemcpyDeviceToDevice, st)
                                  : cudaMemsetAsync(p->state_out, 0, n, st);
      return cuda_status(e);
    }
    return KDA_OK;
  }
  const size_t need = kda_fwd_workspace_bytes(p->B, p->H, p->T, p->D, p->chunk, p->flags);
  if (need && (p->workspace == nullptr || p->workspace_bytes < need)) return KDA_ERR_WORKSPACE;
  kda::FwdArgs a{};
  a.B = p->B; a.H = p->H; a.T = p->T; a.D = p->D; a.C = p->chunk;
  a.literal = literal ? 1 : 0;
  a.per_step = (p->flags & KDA_FLAG_PER_STEP) ? 1 : 0;
  a.q = to_view(p->q); a.k = to_view(p->k); a.v = to_view(p->v); a.g = to_view(p->g); a.y = to_view(p->y);
  a.decay = make_decay(p->decay, p->decay_stride_b, p->decay_stride_h, p->decay_stride_d, p->decay_scalar,
                       p->T, p->chunk);
  a.s_in = p->state_in;
  a.s_out = p->state_out;
  a.status = p->status;
  const int ns = p->B * p->H, nchunks = n_chunks(p->T, p->chunk);
  const int nr = n_ranges(ns, nchunks, fwd_slots(p->D, p->flags));
  kda::tc::Queue q{};
  void *agg = reinterpret_cast<char *>(p->workspace) + queue_bytes(nr, carry_f4(p->D));
  cudaError_t e = make_queue(q, p->workspace, ns, nchunks, carry_f4(p->D), nr, agg, carry_f4(p->D), st);
  if (e != cudaSuccess) return cuda_status(e);
  const int slots = fwd_slots(p->D, p->flags);
  return cuda_status(kda::launch_fwd_tc(a, q, nr < slots ? nr : slots, p->dtype, st));
}

int kda_bwd_sm100(const kda_bwd_params *p, kda_stream_t stream) {
  if (p == nullptr) return KDA_ERR_NULL_ARGUMENT;
  int rc = check_common(p->B, p->H, p->T, p->D, p->chunk, p->dtype, p->flags);
  if (rc) return rc;
  const bool literal = (p->flags & KDA_FLAG_LITERAL) != 0;
  if (literal && (p->T % p->chunk) != 0 && p->dstate_out) return KDA_ERR_BAD_SHAPE;
  if ((rc = check_per_step(p->flags, p->dtype, p->decay, p->decay_stride_d, p->decay_scalar))) return rc;
  if ((p->flags & KDA_FLAG_PER_STEP) && p->ddecay) return KDA_ERR_UNSUPPORTED;
  const bool gate = p->g.data != nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->H == 0) return KDA_OK;
  if (p->T == 0) {
    const size_t n = (size_t)p->B * p->H * p->D * p->D * sizeof(float);
    cudaError_t e = cudaSuccess;
    if (p->dstate_in)
      e = p->dstate_out ? cudaMemcpyAsync(p->dstate_in, p->dstate_out, n, cudaMemcpyDeviceToDevice, st)
                        : cudaMemsetAsync(p->dstate_in, 0, n, st);
    if (e == cudaSuccess && p->ddecay)
      e = cudaMemsetAsync(p->ddecay, 0, (size_t)p->B * p->H * p->D * sizeof(float), st);
    return cuda_status(e);
  }
  if ((rc = check_view(p->q, true)) || (rc = check_view(p->k, true)) || (rc = check_view(p->v, true)) ||
      (rc = check_view(p->g, false)) || (rc = check_view(p->dy, true)) || (rc = check_view(p->dq, true)) ||
      (rc = check_view(p->dk, true)) || (rc = check_view(p->dv, true)) || (rc = check_view(p->dg, gate)))
    return rc;
  const size_t need = kda_bwd_workspace_bytes(p->B, p->H, p->T, p->D, p->chunk, p->flags);
  if (need && (p->workspace == nullptr || p->workspace_bytes < need)) return KDA_ERR_WORKSPACE;
  kda::BwdArgs a{};
  a.B = p->B; a.H = p->H; a.T = p->T; a.D = p->D; a.C = p->chunk;
  a.literal = literal ? 1 : 0;
  a.per_step = (p->flags & KDA_FLAG_PER_STEP) ? 1 : 0;
  a.q = to_view(p->q); a.k = to_view(p->k); a.v = to_view(p->v); a.g = to_view(p->g); a.dy = to_view(p->dy);
  a.dq = to_view(p->dq); a.dk = to_view(p->dk); a.dv = to_view(p->dv); a.dg = to_view(p->dg);
  a.decay = make_decay(p->decay, p->decay_stride_b, p->decay_stride_h, p->decay_stride_d, p->decay_scalar,
                       p->T, p->chunk);
  a.s_in = p->state_in;
  a.ds_out = p->dstate_out;
  a.ds_in = p->dstate_in;
  a.ddecay = p->ddecay;
  a.status = p->status;
  const int ns = p->B * p->H, nchunks = n_chunks(p->T, p->chunk);
  const int nr = n_ranges(ns, nchunks, bwd_slots());
  const int f1 = 2 * carry_f4(p->D) + 1, f2 = carry_f4(p->D);
  kda::tc::Queue q1{}, q2{};
  char *ws2 = reinterpret_cast<char *>(p->workspace) + queue_bytes(nr, f1);
  char *ws_do = ws2 + queue_bytes(nr, f2);
  char *agg1 = ws_do + do_bytes(p->B, p->H, p->T, p->D);
  char *agg2 = agg1 + agg_bytes(ns, nchunks, nr, 2 * carry_f4(p->D));
  a.dO = View{ws_do, (int64_t)p->H * p->T * p->D, (int64_t)p->T * p->D, p->D, 1};
  cudaError_t e = make_queue(q1, p->workspace, ns, nchunks, f1, nr, agg1, 2 * carry_f4(p->D), st);
  if (e == cudaSuccess) e = make_queue(q2, ws2, ns, nchunks, f2, nr, agg2, carry_f4(p->D), st);
  if (e != cudaSuccess) return cuda_status(e);
  const int grid = nr < bwd_slots() ? nr : bwd_slots();  // persistent CTAs; extra ranges are taken in turn
  return cuda_status(kda::launch_bwd_tc(a, q1, q2, grid, grid, p->dtype, st));
}

}  // extern "C"
