// kda_fwd_sm100_noalloc: the forward scan with its scratch in a fixed,
// file-scope device array instead of a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory for a workspace --
// for instance a host runtime that binds this C ABI and only holds the tensors
// it was handed (its allocator belongs to someone else), or a serving process
// whose device memory is reserved up front and must not grow mid-run.  They
// pass inputs and outputs as usual; the scratch (the work-queue counter, the
// per-stream flags and the state handoff slots) comes from the array below.
//
// Cost and limits: every GPU that loads this module holds the array
// (kKdaScratchBytes) until the process exits.  Arguments are checked first,
// exactly as kda_fwd_sm100 checks them; then problems whose scratch would
// exceed the array are rejected with KDA_ERR_WORKSPACE, before anything is
// enqueued.  All calls share the array and it keeps the last call's contents:
// each call clears the part that must start at zero (the queue header) on its
// stream, and calls that overlap on the GPU (different streams, or different
// host threads) race on it and must be serialised by the caller.
//
// The array's device address is looked up once per device, on that device's
// first successful call, and kept; a failed lookup (e.g. during a stream
// capture) is not kept -- its error is cleared from the CUDA runtime and the
// next call tries again.  A kept address belongs to the device's current
// context: after cudaDeviceReset it is stale, and the library must not be used
// on that device again in this process.
#include <cuda_runtime.h>

#include <mutex>

#include "kda_internal.h"

namespace {

constexpr size_t kKdaScratchBytes = KDA_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_kda_scratch[kKdaScratchBytes];

std::mutex g_scratch_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of the array for the current device (host code may not use
// the symbol itself: on the host it names a stand-in object, not device memory).
int scratch_for_current_device(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KDA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_kda_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // leave no error behind for the caller; the next call retries
      return KDA_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return KDA_OK;
}

}  // namespace

extern "C" int kda_fwd_sm100_noalloc(const kda_fwd_params *p, kda_stream_t stream) {
  const int bad = kda::fwd_check_args(p);
  if (bad != KDA_OK) return bad;
  const size_t need = kda_fwd_workspace_bytes(p->B, p->H, p->T, p->D, p->chunk, p->flags);
  if (need > kKdaScratchBytes) return KDA_ERR_WORKSPACE;
  if (need == 0) return kda_fwd_sm100(p, stream);  // nothing needs scratch (an empty batch or sequence)
  void *scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != KDA_OK) return rc;
  kda_fwd_params q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kKdaScratchBytes;
  return kda_fwd_sm100(&q, stream);
}
