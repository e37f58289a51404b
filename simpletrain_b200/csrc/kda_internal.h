// Internal launch arguments shared by the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kda_sm100.h"

namespace kda {

// One [B,H,T,D] view (element strides).
struct View {
  void *data;
  int64_t sb, sh, st, sd;
};

// Per-channel chunk decay source.  alpha for a chunk of length L is
//   decay**L  (tensor decay: powf in-kernel; scalar: host-computed in double,
//   rounded once to fp32, matching `python_float ** L * fp32_state`).
struct DecaySrc {
  const float *ptr;  // nullptr -> scalar
  int64_t sb, sh, sd;
  float alpha_full;  // scalar decay**chunk
  float alpha_tail;  // scalar decay**(T % chunk) (unused when T % chunk == 0)
  double scalar;
};

struct FwdArgs {
  int B, H, T, D, C;
  int literal;
  int per_step;  // per-token decay (s_t = a s_{t-1} + k_t^T v_t), one decay per stream
  View q, k, v, g, y;  // g.data == nullptr -> no gate
  DecaySrc decay;
  const float *s_in;
  float *s_out;
  int32_t *status;
};

struct BwdArgs {
  int B, H, T, D, C;
  int literal;
  int per_step;
  View q, k, v, g, dy, dq, dk, dv, dg;
  View dO;  // workspace [B][H][T][D] 16-bit: dy * g, written by the forward-direction pass
  DecaySrc decay;
  const float *s_in;
  const float *ds_out;
  float *ds_in;
  float *ddecay;
  int32_t *status;
};

// Device-side alpha for channel d of (b, h) and a chunk of length L.
__device__ __forceinline__ float chunk_alpha(const DecaySrc &s, int b, int h, int d, int L, int C) {
  if (s.ptr == nullptr) return (L == C) ? s.alpha_full : s.alpha_tail;
  const float a = s.ptr[b * s.sb + h * s.sh + d * s.sd];
  return powf(a, (float)L);
}

__device__ __forceinline__ float decay_value(const DecaySrc &s, int b, int h, int d) {
  if (s.ptr == nullptr) return (float)s.scalar;
  return s.ptr[b * s.sb + h * s.sh + d * s.sd];
}

// chunk_alpha from a value decay_value() loaded earlier (the load's latency can then
// overlap other waits); the same result as chunk_alpha.
__device__ __forceinline__ float chunk_alpha_of(const DecaySrc &s, float dv, int L, int C) {
  if (s.ptr == nullptr) return (L == C) ? s.alpha_full : s.alpha_tail;
  return powf(dv, (float)L);
}

// Counts kernel launches for kda_launch_count().
void count_launches(int n);

// Launch `kern` on `st`.  With `early` the launch has a programmatic dependency
// on the kernel before it on the stream: it may start while that kernel is still
// running (once all of that kernel's CTAs have started or called
// pdl_launch_dependents), and its threads call pdl_wait() before they read what
// that kernel writes.
template <typename... P, typename... A>
cudaError_t launch_kernel(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool early,
                          A &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = early ? attr : nullptr;
  cfg.numAttrs = early ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<A &&>(args)...);
}

// kda_fwd_sm100's argument checks, all but the workspace's: KDA_OK or a kda_status.
int fwd_check_args(const kda_fwd_params *p);

// Kernel ids of the launch tracer (kda_trace_start / kda_trace_stop).
enum TraceKernel { kTraceFwd = 0, kTraceBwdFwdDir = 1, kTraceBwdRevDir = 2, kTraceAgg = 3, kTraceFold = 4 };
// Bracket one kernel launch on `st`: trace_before returns a slot (or -1 when
// the tracer is off or full), trace_after records the launch's end in it.
int trace_before(cudaStream_t st);
void trace_after(int slot, int kernel, cudaStream_t st);

namespace tc {
struct Queue;
}

// Range aggregates (kda_agg_tc.cu): the carry recurrence over the publishing
// piece of each range run from zero, stored thread-major at
// agg + r * agg_f4 * 256 float4.
struct AggArgs {
  int B, H, T, D;
  int literal;
  int per_step;
  DecaySrc decay;
  float4 *agg;
  int agg_f4;
  int32_t *status;
};

// Launchers (return cudaError_t of the launch).  `grid` persistent CTAs work
// through the queue's units.
cudaError_t launch_fwd_tc(const FwdArgs &a, const tc::Queue &q, int grid, int dtype, cudaStream_t st);
cudaError_t launch_bwd_tc(const BwdArgs &a, const tc::Queue &q1, const tc::Queue &q2, int grid1, int grid2,
                          int dtype, cudaStream_t st);
// mode 0: S from (k, v); 1: S and decay tangent from (k, v); 2: dS from (q, dO).
// a.per_step takes modes 0 and 2.
cudaError_t launch_agg_tc(int mode, const AggArgs &a, const View &va, const View &vb, const tc::Queue &q, int dtype,
                          const float *boundary, cudaStream_t st);
// CTAs of the forward kernel that fit on one SM.
int fwd_tc_occupancy(int D, int dtype, bool literal, bool per_step);

}  // namespace kda
