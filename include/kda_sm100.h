/*
 * kda_sm100.h -- C ABI of the B200 (sm_100a) Kimi Delta Attention chunked scan.
 *
 * This is the boundary SimpleTrain's KDA dispatch binds to.  The reference's
 * operator is the Python function
 *
 *     kda_chunked_scan(q, k, v, gate=None, decay=0.99, chunk_size=64,
 *                      use_triton=True) -> y                (kernels/kda_kernel.py:303-311)
 *
 * whose GPU work is the Triton launch in kda_chunked_scan_triton
 * (kernels/kda_kernel.py:195-238) and, in practice, the torch chunk loop
 * _kda_chunked_scan_torch (kernels/kda_kernel.py:244-297) plus autograd
 * through it for the backward pass.  The entry points below replace those:
 *
 *   kda_fwd_sm100  <- kda_chunked_scan_triton / _kda_chunked_scan_torch forward
 *   kda_bwd_sm100  <- autograd through _kda_chunked_scan_torch (:269-296)
 *
 * Conventions
 *   - All tensors are device pointers owned by the caller; nothing is
 *     allocated, freed or synchronised inside these calls.  Work is enqueued
 *     on `stream` (a cudaStream_t; NULL = legacy default stream).
 *   - q, k, v, g, y, dy, dq, dk, dv, dg are [B, H, T, D] views described by
 *     element strides (the KDA layer passes [B, T, H, D] memory viewed as
 *     [B, H, T, D], models/kimi_k3.py:99-102).  The innermost stride must be
 *     1, every other stride a multiple of 8 elements and every base pointer
 *     16-byte aligned (tensor-memory-accelerator copies need 16-byte rows).
 *   - States are fp32 [B, H, D, D] contiguous, row index = key channel.
 *   - decay is either a device fp32 array addressed as
 *     decay[b*decay_stride_b + h*decay_stride_h + d*decay_stride_d]
 *     (strides may be 0 to broadcast), or, when `decay` is NULL, the host
 *     scalar `decay_scalar` (the reference's float decay, :308).  The state
 *     is scaled per chunk of length L by decay**L along its key-channel rows
 *     (:295 with decay broadcast as [B, H, D, 1]).
 *   - Return value: KDA_OK or a kda_status code; nothing throws across the
 *     ABI.  Errors detected on the device (a bounded wait that expired) are
 *     OR-ed into *status when `status` is non-NULL and are never fatal to
 *     the CUDA context.
 *   - Thread-safe; reentrant per stream.  Two calls that overlap on the GPU
 *     must not share a workspace.
 */
#ifndef KDA_SM100_H
#define KDA_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_ABI_VERSION 2

typedef struct CUstream_st *kda_stream_t; /* identical to cudaStream_t */

enum kda_dtype { KDA_DTYPE_BF16 = 0, KDA_DTYPE_F16 = 1 };

enum kda_flags {
  /* Reference-exact state update U_c = K_c V_c^T (kernels/kda_kernel.py:294).
     Needs D == chunk; a ragged last chunk may not ask for the final state. */
  KDA_FLAG_LITERAL = 1u << 0,
  /* Per-token decay instead of the chunk-constant one (ABI version 2): the
     recurrence of the reference's docstring and Triton kernel
     (kernels/kda_kernel.py:8-11, :134-180)
         s_t = a s_{t-1} + k_t^T v_t,   o_t = q_t s_t,   y_t = g_t * o_t
     with one decay a per (batch, head): decay == NULL (decay_scalar) or
     decay_stride_d == 0, and 0.125 <= a <= 1 for bf16, 0.9 <= a <= 1 for
     fp16 (checked for decay_scalar; the kernels scale 16-bit q and k rows by
     powers a^-32 .. a^32).  state_out is s_T.  Not with KDA_FLAG_LITERAL;
     kda_bwd_sm100 takes ddecay == NULL. */
  KDA_FLAG_PER_STEP = 1u << 1,
};

enum kda_status {
  KDA_OK = 0,
  KDA_ERR_NULL_ARGUMENT = 1,   /* a required pointer is NULL */
  KDA_ERR_BAD_SHAPE = 2,       /* negative size, or literal mode with D != chunk */
  KDA_ERR_UNSUPPORTED = 3,     /* head dim / chunk / dtype / flag combination without a kernel */
  KDA_ERR_BAD_LAYOUT = 4,      /* stride or alignment rule violated */
  KDA_ERR_WORKSPACE = 5,       /* workspace missing or too small */
  KDA_ERR_CUDA = 6,            /* a CUDA runtime call or launch failed */
  KDA_ERR_DEVICE_TIMEOUT = 64, /* device-side: a bounded wait expired (status word bit) */
};

typedef struct kda_tensor {
  void *data; /* NULL only where documented optional */
  int64_t stride_b, stride_h, stride_t, stride_d; /* element strides of the [B,H,T,D] view */
} kda_tensor;

typedef struct kda_fwd_params {
  int32_t B, H, T, D; /* batch, heads, tokens, head dim (key dim == value dim) */
  int32_t chunk;      /* chunk length; 64 */
  int32_t dtype;      /* enum kda_dtype, for q, k, v, g, y */
  uint32_t flags;     /* enum kda_flags */
  kda_tensor q, k, v;
  kda_tensor g;       /* output gate; g.data == NULL means no gate (:288-289) */
  kda_tensor y;       /* output */
  const float *decay; /* NULL -> decay_scalar */
  int64_t decay_stride_b, decay_stride_h, decay_stride_d;
  double decay_scalar;
  const float *state_in; /* [B,H,D,D] initial state; NULL -> zeros (:264) */
  float *state_out;      /* [B,H,D,D] final state; NULL -> not written */
  void *workspace;       /* kda_fwd_workspace_bytes() bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t *status; /* optional device word for device-side errors */
} kda_fwd_params;

typedef struct kda_bwd_params {
  int32_t B, H, T, D, chunk, dtype;
  uint32_t flags;
  kda_tensor q, k, v, g, dy;     /* forward inputs and dL/dy; g.data may be NULL */
  kda_tensor dq, dk, dv, dg;     /* outputs; dg ignored when g.data == NULL */
  const float *decay;
  int64_t decay_stride_b, decay_stride_h, decay_stride_d;
  double decay_scalar;
  const float *state_in;   /* forward's initial state, NULL -> zeros */
  const float *dstate_out; /* dL/d(final state), NULL -> zero */
  float *dstate_in;        /* out: dL/d(initial state), NULL -> not written */
  float *ddecay;           /* out: [B,H,D] fp32 dL/d(decay[b,h,d]), NULL -> not computed */
  void *workspace;         /* kda_bwd_workspace_bytes() bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t *status;
} kda_bwd_params;

/* Workspace needed by one call on the CURRENT device (0 allowed).  flags as in
   the params.  It holds one fp32 D x D state slot per boundary between the
   call's work ranges (one range per resident CTA, so it is bounded by the
   device's SM count, not by B*H or T), so query it on the device that runs
   the call. */
size_t kda_fwd_workspace_bytes(int32_t B, int32_t H, int32_t T, int32_t D, int32_t chunk,
                               uint32_t flags);
size_t kda_bwd_workspace_bytes(int32_t B, int32_t H, int32_t T, int32_t D, int32_t chunk,
                               uint32_t flags);

/* Forward scan: y (and optionally the final state). */
int kda_fwd_sm100(const kda_fwd_params *p, kda_stream_t stream);

/* Backward scan: dq, dk, dv, dg, and optionally dL/d(initial state), dL/d(decay). */
int kda_bwd_sm100(const kda_bwd_params *p, kda_stream_t stream);

/* Human-readable text of a kda_status value (static storage). */
const char *kda_status_string(int32_t status);

/* KDA_ABI_VERSION of the loaded library. */
int32_t kda_abi_version(void);

/* Number of kernels this library has launched in the process so far
   (diagnostic; no counterpart in the reference). */
uint64_t kda_launch_count(void);

/* Per-kernel device times (diagnostic; no counterpart in the reference).
   kda_trace_start(n): from now on each of the next n KDA kernel launches of
   this library on the current device is bracketed by two CUDA events
   recorded on its launching stream.  Returns KDA_OK, KDA_ERR_BAD_SHAPE for
   n <= 0, or KDA_ERR_CUDA when the events cannot be created.
   kda_trace_stop(ms, kernel, cap): stops recording, waits for the recorded
   events and writes, in launch order, up to cap launch durations in
   milliseconds and kernel ids (kda_kernel_name names them; -1 marks a launch
   that failed).  Returns the number of launches recorded, or -KDA_ERR_CUDA.
   One tracer per process: a second start discards the first; launches on
   other devices and launches beyond n are not recorded.
   A launch made while its stream is being captured into a CUDA graph gets
   event-record nodes in the graph instead, recorded at every replay:
   kda_trace_read (same arguments and result as kda_trace_stop, but it keeps
   recording) then gives the times of the last replay.  Destroy such a graph
   before kda_trace_stop, which frees the events. */
int kda_trace_start(int32_t max_launches);
int32_t kda_trace_read(float *ms, int32_t *kernel, int32_t cap);
int32_t kda_trace_stop(float *ms, int32_t *kernel, int32_t cap);
const char *kda_kernel_name(int32_t kernel);

/* Size of the fixed device scratch array used by kda_fwd_sm100_noalloc. */
#define KDA_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/* Forward scan that allocates nothing and takes no workspace (no counterpart
   in the reference; an addition of this library).
   For callers that cannot allocate device memory for a workspace -- e.g. a
   host runtime that binds this ABI but only holds the tensors it was given,
   or a process whose device memory is reserved up front.  Inputs, outputs and
   results are exactly those of kda_fwd_sm100 (p->workspace and
   p->workspace_bytes are ignored); the scratch comes from a file-scope device
   array of KDA_NOALLOC_SCRATCH_BYTES that every GPU loading it holds until
   the process exits.
   - Checks its arguments as kda_fwd_sm100 does (same status codes), then
     returns KDA_ERR_WORKSPACE, before enqueuing anything, when the problem
     needs more than KDA_NOALLOC_SCRATCH_BYTES of scratch
     (kda_fwd_workspace_bytes() tells how much: 64 KiB per range boundary at
     D=128, 16 KiB at D=64, at most one boundary per resident CTA -- about
     10 MiB on a 148-SM GPU -- and, when a stream spans three or more ranges,
     one range aggregate of the same size per range -- about 19 MiB in all --
     plus a small header; only a KDA_SM100_RANGES override far above the CTA
     count reaches the limit).
   - The first call on a device looks up the array's device address; make that
     first call before any stream capture.  A failed lookup returns
     KDA_ERR_CUDA, leaves no CUDA error pending, and is retried by the next
     call.  The address is kept for the life of the process: it is invalid
     after cudaDeviceReset on that device.
   - Calls share the array and it keeps the last call's contents; each call
     clears what must start at zero on its own stream.  Calls that overlap on
     the GPU race on the array: serialise them (one stream, or events). */
int kda_fwd_sm100_noalloc(const kda_fwd_params *p, kda_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* KDA_SM100_H */
