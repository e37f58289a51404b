// SimpleTrain's fused elementwise / row-reduction ops on sm_100a (C ABI in
// include/st_fused_ops.h), with the backward passes the Triton originals in
// kernels/fused_ops.py lack.
//
// All are HBM-bound: one pass over each operand with 16-byte vector accesses
// (eight 16-bit values), fp32 arithmetic, and grids sized to the SM count.
//   silu * mul      elementwise, grid-stride            (kernels/fused_ops.py:62-81)
//   RMSNorm + res   one warp per row, two sweeps of the row (the second hits
//                   L2); the weight gradient is summed per CTA in registers,
//                   then across CTAs in a fixed order  (kernels/fused_ops.py:129-145)
//   cross-entropy   one CTA per row: one pass over the vocabulary from HBM
//                   with a running maximum and sum of exponentials, an optional
//                   softmax sweep; the backward recomputes softmax from the saved
//                   log-sum-exp                        (kernels/fused_ops.py:209-263)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/st_fused_ops.h"
#include "kda_internal.h"
#include "tc_common.cuh"

namespace {

using kda::tc::pack2;
using kda::tc::unpack2;

constexpr int kBlock = 256;

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int status_of(cudaError_t e) { return e == cudaSuccess ? KDA_OK : KDA_ERR_CUDA; }

// eight 16-bit values <-> eight floats
template <bool BF>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  for (int i = 0; i < 4; ++i) {
    const float2 p = unpack2(w[i], BF);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}
template <bool BF>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack2(f[0], f[1], BF), pack2(f[2], f[3], BF), pack2(f[4], f[5], BF), pack2(f[6], f[7], BF));
}
template <bool BF>
__device__ __forceinline__ float load1(const void *p, int64_t i) {
  const uint16_t h = reinterpret_cast<const uint16_t *>(p)[i];
  return unpack2((uint32_t)h, BF).x;
}
template <bool BF>
__device__ __forceinline__ void store1(void *p, int64_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = (uint16_t)(pack2(v, 0.f, BF) & 0xffffu);
}

__device__ __forceinline__ float sigmoidf(float a) { return 1.f / (1.f + expf(-a)); }

// ------------------------------------------------------------------ silu*mul
template <bool BF, bool VEC>
__global__ void __launch_bounds__(kBlock) silu_mul_fwd_kernel(const void *a, const void *b, void *out, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * kBlock;
  if (VEC) {
    const int64_t nv = n / 8;
    const uint4 *a4 = reinterpret_cast<const uint4 *>(a), *b4 = reinterpret_cast<const uint4 *>(b);
    uint4 *o4 = reinterpret_cast<uint4 *>(out);
    for (int64_t i = blockIdx.x * (int64_t)kBlock + threadIdx.x; i < nv; i += stride) {
      float fa[8], fb[8], fo[8];
      unpack8<BF>(__ldg(a4 + i), fa);
      unpack8<BF>(__ldg(b4 + i), fb);
      for (int k = 0; k < 8; ++k) fo[k] = fa[k] * sigmoidf(fa[k]) * fb[k];
      o4[i] = pack8<BF>(fo);
    }
    for (int64_t i = nv * 8 + blockIdx.x * (int64_t)kBlock + threadIdx.x; i < n; i += stride) {
      const float x = load1<BF>(a, i);
      store1<BF>(out, i, x * sigmoidf(x) * load1<BF>(b, i));
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)kBlock + threadIdx.x; i < n; i += stride) {
      const float x = load1<BF>(a, i);
      store1<BF>(out, i, x * sigmoidf(x) * load1<BF>(b, i));
    }
  }
}

template <bool BF, bool VEC>
__global__ void __launch_bounds__(kBlock)
    silu_mul_bwd_kernel(const void *a, const void *b, const void *dout, void *da, void *db, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * kBlock;
  // d/da silu(a) = s (1 + a (1 - s)), s = sigmoid(a)
  auto one = [&](int64_t i) {
    const float x = load1<BF>(a, i), y = load1<BF>(b, i), g = load1<BF>(dout, i), s = sigmoidf(x);
    store1<BF>(da, i, g * y * s * (1.f + x * (1.f - s)));
    store1<BF>(db, i, g * x * s);
  };
  if (VEC) {
    const int64_t nv = n / 8;
    const uint4 *a4 = reinterpret_cast<const uint4 *>(a), *b4 = reinterpret_cast<const uint4 *>(b),
                *g4 = reinterpret_cast<const uint4 *>(dout);
    uint4 *da4 = reinterpret_cast<uint4 *>(da), *db4 = reinterpret_cast<uint4 *>(db);
    for (int64_t i = blockIdx.x * (int64_t)kBlock + threadIdx.x; i < nv; i += stride) {
      float fa[8], fb[8], fg[8], ra[8], rb[8];
      unpack8<BF>(__ldg(a4 + i), fa);
      unpack8<BF>(__ldg(b4 + i), fb);
      unpack8<BF>(__ldg(g4 + i), fg);
      for (int k = 0; k < 8; ++k) {
        const float s = sigmoidf(fa[k]);
        ra[k] = fg[k] * fb[k] * s * (1.f + fa[k] * (1.f - s));
        rb[k] = fg[k] * fa[k] * s;
      }
      da4[i] = pack8<BF>(ra);
      db4[i] = pack8<BF>(rb);
    }
    for (int64_t i = nv * 8 + blockIdx.x * (int64_t)kBlock + threadIdx.x; i < n; i += stride) one(i);
  } else {
    for (int64_t i = blockIdx.x * (int64_t)kBlock + threadIdx.x; i < n; i += stride) one(i);
  }
}

int elementwise_grid(int64_t n) {
  const int64_t want = (n / 8 + kBlock - 1) / kBlock;
  const int64_t cap = (int64_t)sm_count() * 8;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

// ------------------------------------------------------------ RMSNorm + res
__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// one warp per row; D % 8 == 0 (vector path) or any D (scalar path)
template <bool BF, bool VEC>
__global__ void __launch_bounds__(kBlock)
    rmsnorm_fwd_kernel(const void *x, const void *r, const void *w, void *out, float *rstd, int64_t N, int64_t D,
                       float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (kBlock / 32) + (threadIdx.x >> 5);
  if (row >= N) return;
  const int64_t base = row * D;
  float ss = 0.f;
  if (VEC) {
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x) + base / 8;
    for (int64_t i = lane; i < D / 8; i += 32) {
      float f[8];
      unpack8<BF>(__ldg(x4 + i), f);
      for (int k = 0; k < 8; ++k) ss = fmaf(f[k], f[k], ss);
    }
  } else {
    for (int64_t i = lane; i < D; i += 32) {
      const float v = load1<BF>(x, base + i);
      ss = fmaf(v, v, ss);
    }
  }
  const float rs = rsqrtf(warp_sum(ss) / (float)D + eps);
  if (lane == 0) rstd[row] = rs;
  if (VEC) {
    const uint4 *x4 = reinterpret_cast<const uint4 *>(x) + base / 8, *r4 = reinterpret_cast<const uint4 *>(r) + base / 8,
                *w4 = reinterpret_cast<const uint4 *>(w);
    uint4 *o4 = reinterpret_cast<uint4 *>(out) + base / 8;
    for (int64_t i = lane; i < D / 8; i += 32) {
      float fx[8], fr[8], fw[8], fo[8];
      unpack8<BF>(__ldg(x4 + i), fx);
      unpack8<BF>(__ldg(r4 + i), fr);
      unpack8<BF>(__ldg(w4 + i), fw);
      for (int k = 0; k < 8; ++k) fo[k] = fmaf(fx[k] * rs, fw[k], fr[k]);
      o4[i] = pack8<BF>(fo);
    }
  } else {
    for (int64_t i = lane; i < D; i += 32)
      store1<BF>(out, base + i, fmaf(load1<BF>(x, base + i) * rs, load1<BF>(w, i), load1<BF>(r, base + i)));
  }
}

// Persistent CTAs walk tiles of 8 rows grid-stride.  Per tile: each warp
// reduces one row's sum_j x_j w_j dy_j (kept in shared memory), then all 256
// threads sweep the tile's columns in 16-byte vectors, writing
//   dx_i = rstd w_i dy_i - rstd^3 / D * x_i * sum_j x_j w_j dy_j
// and adding dy_i x_i rstd into per-thread weight-gradient registers (thread
// t owns column vectors t, t + 256, ...).  Each CTA writes its partial at the
// end.  D % 8 == 0 and 16-byte aligned rows (else the scalar variant).
template <bool BF, int NV>
__global__ void __launch_bounds__(kBlock)
    rmsnorm_bwd_kernel(const void *x, const void *w, const float *rstd, const void *dy, void *dx, float *partials,
                       int64_t N, int64_t D) {
  constexpr int R = kBlock / 32;  // rows per tile
  __shared__ float sm_c[R], sm_rs[R];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t DV = D / 8;
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x), *g4 = reinterpret_cast<const uint4 *>(dy),
              *w4 = reinterpret_cast<const uint4 *>(w);
  uint4 *dx4 = reinterpret_cast<uint4 *>(dx);
  float acc[NV][8];
  for (int k = 0; k < NV; ++k)
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
  for (int64_t r0 = (int64_t)blockIdx.x * R; r0 < N; r0 += (int64_t)gridDim.x * R) {
    const int64_t row = r0 + warp;
    if (row < N) {
      float dot = 0.f;
      for (int64_t v = lane; v < DV; v += 32) {
        float fx[8], fg[8], fw[8];
        unpack8<BF>(__ldg(x4 + row * DV + v), fx);
        unpack8<BF>(__ldg(g4 + row * DV + v), fg);
        unpack8<BF>(__ldg(w4 + v), fw);
        for (int j = 0; j < 8; ++j) dot = fmaf(fx[j] * fw[j], fg[j], dot);
      }
      dot = warp_sum(dot);
      if (lane == 0) {
        const float rs = rstd[row];
        sm_rs[warp] = rs;
        sm_c[warp] = rs * rs * rs * dot / (float)D;
      }
    }
    __syncthreads();
    const int nr = (int)((N - r0) < R ? (N - r0) : R);
    for (int rr = 0; rr < nr; ++rr) {
      const int64_t rb = (r0 + rr) * DV;
      const float rs = sm_rs[rr], c = sm_c[rr];
      for (int k = 0; k < NV; ++k) {
        const int64_t v = threadIdx.x + (int64_t)kBlock * k;
        if (v < DV) {
          float fx[8], fg[8], fw[8], fo[8];
          unpack8<BF>(__ldg(x4 + rb + v), fx);  // L1 / L2: read by the dot pass just before
          unpack8<BF>(__ldg(g4 + rb + v), fg);
          unpack8<BF>(__ldg(w4 + v), fw);
          for (int j = 0; j < 8; ++j) {
            fo[j] = rs * fw[j] * fg[j] - c * fx[j];
            acc[k][j] = fmaf(fg[j] * fx[j], rs, acc[k][j]);
          }
          dx4[rb + v] = pack8<BF>(fo);
        }
      }
    }
    __syncthreads();
  }
  for (int k = 0; k < NV; ++k) {
    const int64_t v = threadIdx.x + (int64_t)kBlock * k;
    if (v < DV)
      for (int j = 0; j < 8; ++j) partials[(int64_t)blockIdx.x * D + 8 * v + j] = acc[k][j];
  }
}

// scalar variant (any D): warp per row, shared-memory weight-gradient sums
template <bool BF>
__global__ void __launch_bounds__(kBlock)
    rmsnorm_bwd_scalar_kernel(const void *x, const void *w, const float *rstd, const void *dy, void *dx,
                              float *partials, int64_t N, int64_t D) {
  extern __shared__ float dw_acc[];  // [D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t i = threadIdx.x; i < D; i += kBlock) dw_acc[i] = 0.f;
  __syncthreads();
  for (int64_t row = (int64_t)blockIdx.x * (kBlock / 32) + warp; row < N; row += (int64_t)gridDim.x * (kBlock / 32)) {
    const int64_t base = row * D;
    const float rs = rstd[row];
    float dot = 0.f;
    for (int64_t i = lane; i < D; i += 32)
      dot = fmaf(load1<BF>(x, base + i) * load1<BF>(w, i), load1<BF>(dy, base + i), dot);
    dot = warp_sum(dot);
    const float c = rs * rs * rs * dot / (float)D;
    for (int64_t i = lane; i < D; i += 32) {
      const float xv = load1<BF>(x, base + i), gv = load1<BF>(dy, base + i);
      store1<BF>(dx, base + i, rs * load1<BF>(w, i) * gv - c * xv);
      atomicAdd(&dw_acc[i], gv * xv * rs);
    }
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < D; i += kBlock) partials[(int64_t)blockIdx.x * D + i] = dw_acc[i];
}

__global__ void __launch_bounds__(kBlock) sum_rows_kernel(const float *partials, float *out, int rows, int64_t D) {
  for (int64_t i = blockIdx.x * (int64_t)kBlock + threadIdx.x; i < D; i += (int64_t)gridDim.x * kBlock) {
    float s = 0.f;
    for (int r = 0; r < rows; ++r) s += partials[(int64_t)r * D + i];  // fixed order: deterministic
    out[i] = s;
  }
}

int rmsnorm_bwd_grid(int64_t N) {
  const int64_t want = (N + kBlock / 32 - 1) / (kBlock / 32);
  const int64_t cap = (int64_t)sm_count() * 4;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

// ---------------------------------------------------------- cross-entropy
// 2^x by the hardware approximation (relative error ~2^-22); e^x = 2^(x log2 e)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Running (max m, sum s of exp(x - m)) pairs, merged: one exponential per
// element and one rescale when the maximum grows.  m = -inf means "no
// elements yet" (s = 0).
__device__ __forceinline__ void lse_merge(float &m, float &s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * ex2_approx((m - M) * kLog2e)) +
      (m2 == -INFINITY ? 0.f : s2 * ex2_approx((m2 - M) * kLog2e));
  m = M;
}

__device__ __forceinline__ void block_lse(float &m, float &s, float *sm_m, float *sm_s) {
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  if ((threadIdx.x & 31) == 0) {
    sm_m[threadIdx.x >> 5] = m;
    sm_s[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  m = sm_m[0];
  s = sm_s[0];
  for (int i = 1; i < kBlock / 32; ++i) lse_merge(m, s, sm_m[i], sm_s[i]);
}

// One CTA per row.  One pass over the row (HBM) keeps each thread's running
// maximum and sum of exponentials, rescaled once per 16-byte vector whose
// maximum exceeds the running one; the pairs are merged across the block.
template <bool BF, bool VEC>
__global__ void __launch_bounds__(kBlock)
    ce_fwd_kernel(const void *logits, const int64_t *labels, float *loss, float *lse_out, void *probs, int64_t V) {
  __shared__ float sm_m[kBlock / 32], sm_s[kBlock / 32];
  const int64_t row = blockIdx.x, base = row * V;
  const uint4 *l4 = reinterpret_cast<const uint4 *>(logits) + base / 8;
  float m = -INFINITY, s = 0.f;
  if (VEC) {
    for (int64_t i = threadIdx.x; i < V / 8; i += kBlock) {
      float f[8];
      unpack8<BF>(__ldg(l4 + i), f);
      float mv = f[0];
      for (int k = 1; k < 8; ++k) mv = fmaxf(mv, f[k]);
      if (mv > m) {
        s = (m == -INFINITY) ? 0.f : s * ex2_approx((m - mv) * kLog2e);
        m = mv;
      }
      if (m != -INFINITY) {
        const float mb = m * kLog2e;
        float t = 0.f;
        for (int k = 0; k < 8; ++k) t += ex2_approx(fmaf(f[k], kLog2e, -mb));
        s += t;
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += kBlock) lse_merge(m, s, load1<BF>(logits, base + i), 1.f);
  }
  block_lse(m, s, sm_m, sm_s);
  const float l = m + logf(s);
  if (threadIdx.x == 0) {
    lse_out[row] = l;
    const int64_t lab = labels[row];
    loss[row] = (lab >= 0 && lab < V) ? l - load1<BF>(logits, base + lab) : NAN;  // out-of-range label: NaN
  }
  if (probs == nullptr) return;
  if (VEC) {
    uint4 *p4 = reinterpret_cast<uint4 *>(probs) + base / 8;
    for (int64_t i = threadIdx.x; i < V / 8; i += kBlock) {
      float f[8];
      unpack8<BF>(__ldg(l4 + i), f);
      for (int k = 0; k < 8; ++k) f[k] = ex2_approx(fmaf(f[k], kLog2e, -l * kLog2e));
      p4[i] = pack8<BF>(f);
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += kBlock) store1<BF>(probs, base + i, expf(load1<BF>(logits, base + i) - l));
  }
}

template <bool BF, bool VEC>
__global__ void __launch_bounds__(kBlock)
    ce_bwd_kernel(const void *logits, const int64_t *labels, const float *lse, const float *dloss, void *dlogits,
                  int64_t V) {
  const int64_t row = blockIdx.x, base = row * V, lab = labels[row];
  const float l = lse[row], g = dloss[row];
  if (VEC) {
    const uint4 *l4 = reinterpret_cast<const uint4 *>(logits) + base / 8;
    uint4 *d4 = reinterpret_cast<uint4 *>(dlogits) + base / 8;
    for (int64_t i = threadIdx.x; i < V / 8; i += kBlock) {
      float f[8];
      unpack8<BF>(__ldg(l4 + i), f);
      for (int k = 0; k < 8; ++k) f[k] = (expf(f[k] - l) - (8 * i + k == lab ? 1.f : 0.f)) * g;
      d4[i] = pack8<BF>(f);
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += kBlock)
      store1<BF>(dlogits, base + i, (expf(load1<BF>(logits, base + i) - l) - (i == lab ? 1.f : 0.f)) * g);
  }
}

bool dtype_ok(int32_t d) { return d == KDA_DTYPE_BF16 || d == KDA_DTYPE_F16; }

#define ST_DISPATCH(BFV, VECV, ...)          \
  do {                                       \
    if (BFV) {                               \
      if (VECV) {                            \
        constexpr bool BF = true, VEC = true; \
        __VA_ARGS__;                         \
      } else {                               \
        constexpr bool BF = true, VEC = false; \
        __VA_ARGS__;                         \
      }                                      \
    } else {                                 \
      if (VECV) {                            \
        constexpr bool BF = false, VEC = true; \
        __VA_ARGS__;                         \
      } else {                               \
        constexpr bool BF = false, VEC = false; \
        __VA_ARGS__;                         \
      }                                      \
    }                                        \
  } while (0)

}  // namespace

extern "C" {

int st_silu_mul_fwd(const void *a, const void *b, void *out, int64_t n, int32_t dtype, kda_stream_t stream) {
  if (n < 0) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  if (n == 0) return KDA_OK;
  if (!a || !b || !out) return KDA_ERR_NULL_ARGUMENT;
  const bool vec = aligned16(a) && aligned16(b) && aligned16(out);
  const int grid = elementwise_grid(n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ST_DISPATCH(dtype == KDA_DTYPE_BF16, vec, (silu_mul_fwd_kernel<BF, VEC><<<grid, kBlock, 0, st>>>(a, b, out, n)));
  kda::count_launches(1);
  return status_of(cudaGetLastError());
}

int st_silu_mul_bwd(const void *a, const void *b, const void *dout, void *da, void *db, int64_t n, int32_t dtype,
                    kda_stream_t stream) {
  if (n < 0) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  if (n == 0) return KDA_OK;
  if (!a || !b || !dout || !da || !db) return KDA_ERR_NULL_ARGUMENT;
  const bool vec = aligned16(a) && aligned16(b) && aligned16(dout) && aligned16(da) && aligned16(db);
  const int grid = elementwise_grid(n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ST_DISPATCH(dtype == KDA_DTYPE_BF16, vec,
              (silu_mul_bwd_kernel<BF, VEC><<<grid, kBlock, 0, st>>>(a, b, dout, da, db, n)));
  kda::count_launches(1);
  return status_of(cudaGetLastError());
}

int st_rmsnorm_residual_fwd(const void *x, const void *residual, const void *weight, void *out, float *rstd,
                            int64_t N, int64_t D, float eps, int32_t dtype, kda_stream_t stream) {
  if (N < 0 || D <= 0) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  if (N == 0) return KDA_OK;
  if (!x || !residual || !weight || !out || !rstd) return KDA_ERR_NULL_ARGUMENT;
  const bool vec = D % 8 == 0 && aligned16(x) && aligned16(residual) && aligned16(weight) && aligned16(out);
  const int grid = (int)((N + kBlock / 32 - 1) / (kBlock / 32));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ST_DISPATCH(dtype == KDA_DTYPE_BF16, vec,
              (rmsnorm_fwd_kernel<BF, VEC><<<grid, kBlock, 0, st>>>(x, residual, weight, out, rstd, N, D, eps)));
  kda::count_launches(1);
  return status_of(cudaGetLastError());
}

size_t st_rmsnorm_residual_bwd_scratch(int64_t N, int64_t D) {
  if (N <= 0 || D <= 0) return 0;
  return (size_t)rmsnorm_bwd_grid(N) * (size_t)D * sizeof(float);
}

int st_rmsnorm_residual_bwd(const void *x, const void *weight, const float *rstd, const void *dy, void *dx,
                            float *dweight, float *partials, int64_t N, int64_t D, int32_t dtype,
                            kda_stream_t stream) {
  if (N < 0 || D <= 0) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (N == 0) return status_of(cudaMemsetAsync(dweight, 0, (size_t)D * sizeof(float), st));
  if (!x || !weight || !rstd || !dy || !dx || !dweight || !partials) return KDA_ERR_NULL_ARGUMENT;
  const int grid = rmsnorm_bwd_grid(N);
  const bool bf = dtype == KDA_DTYPE_BF16;
  const bool vec = D % 8 == 0 && aligned16(x) && aligned16(weight) && aligned16(dy) && aligned16(dx);
  const int nvec = (int)((D / 8 + kBlock - 1) / kBlock);
  if (vec && nvec <= 8) {
#define ST_RMS_BWD(NC)                                                                                        \
  if (nvec <= NC) {                                                                                         \
    if (bf) rmsnorm_bwd_kernel<true, NC><<<grid, kBlock, 0, st>>>(x, weight, rstd, dy, dx, partials, N, D); \
    else rmsnorm_bwd_kernel<false, NC><<<grid, kBlock, 0, st>>>(x, weight, rstd, dy, dx, partials, N, D);   \
  } else
    ST_RMS_BWD(1) ST_RMS_BWD(2) ST_RMS_BWD(4) ST_RMS_BWD(8) {}
#undef ST_RMS_BWD
  } else {
    const size_t smem = (size_t)D * sizeof(float);
    if (smem > 200 * 1024) return KDA_ERR_UNSUPPORTED;
    cudaError_t e0;
    if (bf) {
      e0 = cudaFuncSetAttribute(rmsnorm_bwd_scalar_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e0 == cudaSuccess)
        rmsnorm_bwd_scalar_kernel<true><<<grid, kBlock, smem, st>>>(x, weight, rstd, dy, dx, partials, N, D);
    } else {
      e0 = cudaFuncSetAttribute(rmsnorm_bwd_scalar_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e0 == cudaSuccess)
        rmsnorm_bwd_scalar_kernel<false><<<grid, kBlock, smem, st>>>(x, weight, rstd, dy, dx, partials, N, D);
    }
    if (e0 != cudaSuccess) return status_of(e0);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return status_of(e);
  const int g2 = (int)((D + kBlock - 1) / kBlock);
  sum_rows_kernel<<<g2 < 1024 ? g2 : 1024, kBlock, 0, st>>>(partials, dweight, grid, D);
  kda::count_launches(2);
  return status_of(cudaGetLastError());
}

int st_cross_entropy_fwd(const void *logits, const int64_t *labels, float *loss, float *lse, void *probs, int64_t N,
                         int64_t V, int32_t dtype, kda_stream_t stream) {
  if (N < 0 || V <= 0 || N > 0x7fffffff) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  if (N == 0) return KDA_OK;
  if (!logits || !labels || !loss || !lse) return KDA_ERR_NULL_ARGUMENT;
  const bool vec = V % 8 == 0 && aligned16(logits) && (probs == nullptr || aligned16(probs));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ST_DISPATCH(dtype == KDA_DTYPE_BF16, vec,
              (ce_fwd_kernel<BF, VEC><<<(unsigned)N, kBlock, 0, st>>>(logits, labels, loss, lse, probs, V)));
  kda::count_launches(1);
  return status_of(cudaGetLastError());
}

int st_cross_entropy_bwd(const void *logits, const int64_t *labels, const float *lse, const float *dloss,
                         void *dlogits, int64_t N, int64_t V, int32_t dtype, kda_stream_t stream) {
  if (N < 0 || V <= 0 || N > 0x7fffffff) return KDA_ERR_BAD_SHAPE;
  if (!dtype_ok(dtype)) return KDA_ERR_UNSUPPORTED;
  if (N == 0) return KDA_OK;
  if (!logits || !labels || !lse || !dloss || !dlogits) return KDA_ERR_NULL_ARGUMENT;
  const bool vec = V % 8 == 0 && aligned16(logits) && aligned16(dlogits);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ST_DISPATCH(dtype == KDA_DTYPE_BF16, vec,
              (ce_bwd_kernel<BF, VEC><<<(unsigned)N, kBlock, 0, st>>>(logits, labels, lse, dloss, dlogits, V)));
  kda::count_launches(1);
  return status_of(cudaGetLastError());
}

}  // extern "C"
