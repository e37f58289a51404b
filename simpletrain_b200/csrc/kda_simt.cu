// Straightforward fp32 CUDA-core KDA kernels (forward, backward).
//
// One CTA walks all chunks of one (batch, head) -- the forward additionally
// splits the value dimension into 32-wide tiles -- with the state in shared
// memory.  These kernels carry the exact arithmetic of the chunk loop in
// kernels/kda_kernel.py:269-296 (fp32 everywhere), and the two-direction
// backward with the closed-form decay gradient.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kda_internal.h"

namespace kda {
namespace {

constexpr int kC = 64;        // chunk length
constexpr int kThreads = 256;
constexpr int kDV = 32;       // value tile of the forward kernel
constexpr int kPad = kC + 1;  // padded row of the [C, C] score tiles

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

template <typename T>
__device__ __forceinline__ const T *elem(const View &v, int b, int h, int t, int d) {
  return reinterpret_cast<const T *>(v.data) + b * v.sb + h * v.sh + (int64_t)t * v.st + d * v.sd;
}
template <typename T>
__device__ __forceinline__ T *elem_w(const View &v, int b, int h, int t, int d) {
  return reinterpret_cast<T *>(v.data) + b * v.sb + h * v.sh + (int64_t)t * v.st + d * v.sd;
}

// Load rows [t0, t0+L) x cols [0, ncol) of a view into shared fp32 [kC][ld], zero rows >= L.
template <typename T>
__device__ void load_tile(float *dst, int ld, const View &v, int b, int h, int t0, int L, int c0, int ncol) {
  for (int i = threadIdx.x; i < kC * ncol; i += blockDim.x) {
    const int r = i / ncol, c = i % ncol;
    dst[r * ld + c] = (r < L) ? to_f(*elem<T>(v, b, h, t0 + r, c0 + c)) : 0.f;
  }
}

// ---------------------------------------------------------------------------
// forward: grid (B*H, D/kDV)
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) fwd_simt_kernel(FwdArgs a) {
  extern __shared__ float sm[];
  float *sQ = sm;               // [kC][D]
  float *sK = sQ + kC * D;      // [kC][D]
  float *sV = sK + kC * D;      // [kC][D]  (all value columns: literal mode needs them)
  float *sG = sV + kC * D;      // [kC][kDV]
  float *sP = sG + kC * kDV;    // [kC][kPad]
  float *sS = sP + kC * kPad;   // [D][kDV]
  float *sA = sS + D * kDV;     // [D] alpha of the current chunk

  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int e0 = blockIdx.y * kDV;
  const int tid = threadIdx.x;
  const size_t sbase = ((size_t)b * a.H + h) * D * D;

  for (int i = tid; i < D * kDV; i += kThreads) {
    const int d = i / kDV, e = i % kDV;
    sS[i] = a.s_in ? a.s_in[sbase + (size_t)d * D + e0 + e] : 0.f;
  }
  for (int t0 = 0; t0 < a.T; t0 += kC) {
    const int L = min(kC, a.T - t0);
    __syncthreads();
    load_tile<T>(sQ, D, a.q, b, h, t0, L, 0, D);
    load_tile<T>(sK, D, a.k, b, h, t0, L, 0, D);
    load_tile<T>(sV, D, a.v, b, h, t0, L, 0, D);
    if (a.g.data) load_tile<T>(sG, kDV, a.g, b, h, t0, L, e0, kDV);
    for (int d = tid; d < D; d += kThreads) sA[d] = chunk_alpha(a.decay, b, h, d, L, kC);
    __syncthreads();
    // masked scores tril(Q K^T)                               (:279-280)
    for (int i = tid; i < kC * kC; i += kThreads) {
      const int r = i / kC, c = i % kC;
      float s = 0.f;
      if (c <= r)
        for (int d = 0; d < D; ++d) s = fmaf(sQ[r * D + d], sK[c * D + d], s);
      sP[r * kPad + c] = s;
    }
    __syncthreads();
    // o = P V + Q S ; y = o * g                                (:281-290)
    for (int i = tid; i < kC * kDV; i += kThreads) {
      const int r = i / kDV, e = i % kDV;
      if (r >= L) continue;
      float o = 0.f;
      for (int j = 0; j <= r; ++j) o = fmaf(sP[r * kPad + j], sV[j * D + e0 + e], o);
      for (int d = 0; d < D; ++d) o = fmaf(sQ[r * D + d], sS[d * kDV + e], o);
      if (a.g.data) o *= sG[r * kDV + e];
      *elem_w<T>(a.y, b, h, t0 + r, e0 + e) = from_f<T>(o);
    }
    __syncthreads();
    // S <- alpha S + U                                          (:292-295)
    if (a.literal && L != kC) continue;  // last ragged chunk: state not defined, not used
    for (int i = tid; i < D * kDV; i += kThreads) {
      const int d = i / kDV, e = i % kDV;
      float u = 0.f;
      if (!a.literal) {
        for (int j = 0; j < L; ++j) u = fmaf(sK[j * D + d], sV[j * D + e0 + e], u);
      } else {  // (K V^T)[p][q], p = d, q = e0 + e (token indices; D == kC)
        for (int x = 0; x < D; ++x) u = fmaf(sK[d * D + x], sV[(e0 + e) * D + x], u);
      }
      sS[i] = fmaf(sA[d], sS[i], u);
    }
  }
  __syncthreads();
  if (a.s_out)
    for (int i = tid; i < D * kDV; i += kThreads) {
      const int d = i / kDV, e = i % kDV;
      a.s_out[sbase + (size_t)d * D + e0 + e] = sS[i];
    }
}

// ---------------------------------------------------------------------------
// backward, shared-memory plan for both directions (one CTA per (b, h))
//   Q, K, V, dY in their 16-bit input type (exact), dO = dY*g, S/dS, P, dP fp32
// ---------------------------------------------------------------------------
template <typename T, int D>
struct BwdSmem {
  static constexpr int kTile = kC * D;
  static constexpr size_t bytes = sizeof(T) * 4 * kTile +
                                  sizeof(float) * (kTile + D * D + 2 * kC * kPad + 2 * D) +
                                  sizeof(double) * D;
};

template <typename T>
__device__ void load_tile_raw(T *dst, const View &v, int b, int h, int t0, int L, int D) {
  for (int i = threadIdx.x; i < kC * D; i += blockDim.x) {
    const int r = i / D, c = i % D;
    dst[i] = (r < L) ? *elem<T>(v, b, h, t0 + r, c) : from_f<T>(0.f);
  }
}

template <typename T, int D>
__device__ void bwd_load_chunk(const BwdArgs &a, int b, int h, int t0, int L, T *sQ, T *sK,
                               T *sV, T *sY, float *sO) {
  load_tile_raw<T>(sQ, a.q, b, h, t0, L, D);
  load_tile_raw<T>(sK, a.k, b, h, t0, L, D);
  load_tile_raw<T>(sV, a.v, b, h, t0, L, D);
  load_tile_raw<T>(sY, a.dy, b, h, t0, L, D);
  for (int i = threadIdx.x; i < kC * D; i += kThreads) {
    const int r = i / D, c = i % D;
    float o = 0.f;
    if (r < L) {
      o = to_f(*elem<T>(a.dy, b, h, t0 + r, c));
      if (a.g.data) o *= to_f(*elem<T>(a.g, b, h, t0 + r, c));
    }
    sO[i] = o;
  }
}

// scores P = tril(Q K^T) and dP = tril(dO V^T)
template <typename T, int D>
__device__ void bwd_scores(const T *sQ, const T *sK, const T *sV, const float *sO, float *sP,
                           float *sdP) {
  for (int i = threadIdx.x; i < kC * kC; i += kThreads) {
    const int r = i / kC, c = i % kC;
    float s = 0.f, ds = 0.f;
    if (c <= r)
      for (int d = 0; d < D; ++d) {
        s = fmaf(to_f(sQ[r * D + d]), to_f(sK[c * D + d]), s);
        ds = fmaf(sO[r * D + d], to_f(sV[c * D + d]), ds);
      }
    sP[r * kPad + c] = s;
    sdP[r * kPad + c] = ds;
  }
}

#define KDA_BWD_SMEM_CARVE                                                              \
  extern __shared__ __align__(16) unsigned char smraw[];                                \
  T *sQ = reinterpret_cast<T *>(smraw), *sK = sQ + kC * D, *sV = sK + kC * D,           \
    *sY = sV + kC * D;                                                                  \
  float *sO = reinterpret_cast<float *>(sY + kC * D), *sS = sO + kC * D,                \
        *sP = sS + D * D, *sdP = sP + kC * kPad, *sA = sdP + kC * kPad;                 \
  double *sAcc = reinterpret_cast<double *>(sA + 2 * D);

// Forward-direction pass: dq, dg and the sink part of the decay gradient.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) bwd_fwddir_simt_kernel(BwdArgs a) {
  KDA_BWD_SMEM_CARVE
  double *sSink = sAcc;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, tid = threadIdx.x;
  const size_t sbase = ((size_t)b * a.H + h) * D * D;
  for (int i = tid; i < D * D; i += kThreads) sS[i] = a.s_in ? a.s_in[sbase + i] : 0.f;
  for (int i = tid; i < D; i += kThreads) sSink[i] = 0.0;
  const int c = tid % D;        // the column this thread owns in the row loops
  const int rstep = kThreads / D;
  for (int t0 = 0; t0 < a.T; t0 += kC) {
    const int L = min(kC, a.T - t0);
    __syncthreads();
    bwd_load_chunk<T, D>(a, b, h, t0, L, sQ, sK, sV, sY, sO);
    for (int d = tid; d < D; d += kThreads) sA[d] = chunk_alpha(a.decay, b, h, d, L, kC);
    __syncthreads();
    bwd_scores<T, D>(sQ, sK, sV, sO, sP, sdP);
    __syncthreads();
    double sink = 0.0;
    for (int r = tid / D; r < L; r += rstep) {
      // O[r][c] = P V + Q S ; dg = dy * O
      if (a.g.data) {
        float o = 0.f;
        for (int j = 0; j <= r; ++j) o = fmaf(sP[r * kPad + j], to_f(sV[j * D + c]), o);
        for (int d = 0; d < D; ++d) o = fmaf(to_f(sQ[r * D + d]), sS[d * D + c], o);
        *elem_w<T>(a.dg, b, h, t0 + r, c) = from_f<T>(to_f(sY[r * D + c]) * o);
      }
      // dq = dP K + dO S^T
      float qi = 0.f, qx = 0.f;
      for (int e = 0; e < D; ++e) qx = fmaf(sO[r * D + e], sS[c * D + e], qx);
      for (int j = 0; j <= r; ++j) qi = fmaf(sdP[r * kPad + j], to_f(sK[j * D + c]), qi);
      *elem_w<T>(a.dq, b, h, t0 + r, c) = from_f<T>(qi + qx);
      sink += (double)(to_f(sQ[r * D + c]) * qx);
    }
    if (a.ddecay) atomicAdd(&sSink[c], sink * (double)t0);
    __syncthreads();
    if (a.literal && L != kC) continue;
    for (int i = tid; i < D * D; i += kThreads) {
      const int d = i / D, e = i % D;
      float u = 0.f;
      if (!a.literal) {
        for (int j = 0; j < L; ++j) u = fmaf(to_f(sK[j * D + d]), to_f(sV[j * D + e]), u);
      } else {
        for (int x = 0; x < D; ++x) u = fmaf(to_f(sK[d * D + x]), to_f(sV[e * D + x]), u);
      }
      sS[i] = fmaf(sA[d], sS[i], u);
    }
  }
  __syncthreads();
  if (a.ddecay)
    for (int i = tid; i < D; i += kThreads) a.sink[((size_t)b * a.H + h) * D + i] = sSink[i];
}

// Reverse pass: dk, dv, d(initial state) and the final decay gradient.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) bwd_revdir_simt_kernel(BwdArgs a) {
  KDA_BWD_SMEM_CARVE
  double *sSrc = sAcc;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, tid = threadIdx.x;
  const size_t sbase = ((size_t)b * a.H + h) * D * D;
  float *sdS = sS;
  for (int i = tid; i < D * D; i += kThreads) sdS[i] = a.ds_out ? a.ds_out[sbase + i] : 0.f;
  for (int i = tid; i < D; i += kThreads) {
    double t3 = 0.0;
    if (a.ddecay && a.ds_out)
      for (int j = 0; j < D; ++j)
        t3 += (double)a.ds_out[sbase + (size_t)i * D + j] * (double)a.s_out[sbase + (size_t)i * D + j];
    sSrc[i] = -t3 * (double)a.T;  // accumulates (source - T<dS_T, S_T>)
  }
  const int c = tid % D;
  const int rstep = kThreads / D;
  const int nchunks = (a.T + kC - 1) / kC;
  for (int ci = nchunks - 1; ci >= 0; --ci) {
    const int t0 = ci * kC, L = min(kC, a.T - t0), t1 = t0 + L;
    __syncthreads();
    bwd_load_chunk<T, D>(a, b, h, t0, L, sQ, sK, sV, sY, sO);
    for (int d = tid; d < D; d += kThreads) sA[d] = chunk_alpha(a.decay, b, h, d, L, kC);
    __syncthreads();
    bwd_scores<T, D>(sQ, sK, sV, sO, sP, sdP);
    __syncthreads();
    const bool upd = !(a.literal && L != kC);  // a ragged literal tail has no state update
    double src = 0.0;
    for (int r = tid / D; r < L; r += rstep) {
      float ki = 0.f, vi = 0.f, kx = 0.f, vx = 0.f;
      for (int j = r; j < L; ++j) {  // dK = dP^T Q, dV = P^T dO  (P, dP lower-triangular)
        ki = fmaf(sdP[j * kPad + r], to_f(sQ[j * D + c]), ki);
        vi = fmaf(sP[j * kPad + r], sO[j * D + c], vi);
      }
      if (upd) {
        if (!a.literal) {
          for (int e = 0; e < D; ++e) kx = fmaf(to_f(sV[r * D + e]), sdS[c * D + e], kx);  // V dS^T
          for (int d = 0; d < D; ++d) vx = fmaf(to_f(sK[r * D + d]), sdS[d * D + c], vx);  // K dS
          src += (double)(to_f(sK[r * D + c]) * kx);
        } else {
          for (int q = 0; q < D; ++q) kx = fmaf(sdS[r * D + q], to_f(sV[q * D + c]), kx);  // dS V
          for (int p = 0; p < D; ++p) vx = fmaf(sdS[p * D + r], to_f(sK[p * D + c]), vx);  // dS^T K
          if (a.ddecay) atomicAdd(&sSrc[r], (double)(to_f(sK[r * D + c]) * kx) * (double)t1);
        }
      }
      *elem_w<T>(a.dk, b, h, t0 + r, c) = from_f<T>(ki + kx);
      *elem_w<T>(a.dv, b, h, t0 + r, c) = from_f<T>(vi + vx);
    }
    if (a.ddecay && !a.literal) atomicAdd(&sSrc[c], src * (double)t1);
    __syncthreads();
    // dS <- alpha dS + Q^T dO
    for (int i = tid; i < D * D; i += kThreads) {
      const int d = i / D, e = i % D;
      float u = 0.f;
      for (int j = 0; j < L; ++j) u = fmaf(to_f(sQ[j * D + d]), sO[j * D + e], u);
      sdS[i] = fmaf(sA[d], sdS[i], u);
    }
  }
  __syncthreads();
  if (a.ds_in)
    for (int i = tid; i < D * D; i += kThreads) a.ds_in[sbase + i] = sdS[i];
  if (a.ddecay)
    for (int i = tid; i < D; i += kThreads) {
      const double dlog = a.sink[((size_t)b * a.H + h) * D + i] - sSrc[i];
      const double av = (double)decay_value(a.decay, b, h, i);
      a.ddecay[((size_t)b * a.H + h) * D + i] = (av != 0.0) ? (float)(dlog / av) : 0.f;
    }
}

template <typename T, int D>
cudaError_t fwd_launch(const FwdArgs &a, cudaStream_t st) {
  const size_t smem = sizeof(float) * (3 * kC * D + kC * kDV + kC * kPad + D * kDV + D);
  auto kern = fwd_simt_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(a.B * a.H, D / kDV);
  kern<<<grid, kThreads, smem, st>>>(a);
  count_launches(1);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t bwd_launch(const BwdArgs &a, cudaStream_t st) {
  const size_t smem = BwdSmem<T, D>::bytes;
  auto k1 = bwd_fwddir_simt_kernel<T, D>;
  auto k2 = bwd_revdir_simt_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k1<<<a.B * a.H, kThreads, smem, st>>>(a);
  count_launches(1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k2<<<a.B * a.H, kThreads, smem, st>>>(a);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_simt(const FwdArgs &a, int dtype, cudaStream_t st) {
  if (a.D == 64) return dtype == KDA_DTYPE_BF16 ? fwd_launch<__nv_bfloat16, 64>(a, st) : fwd_launch<__half, 64>(a, st);
  return dtype == KDA_DTYPE_BF16 ? fwd_launch<__nv_bfloat16, 128>(a, st) : fwd_launch<__half, 128>(a, st);
}

cudaError_t launch_bwd_simt(const BwdArgs &a, int dtype, cudaStream_t st) {
  if (a.D == 64) return dtype == KDA_DTYPE_BF16 ? bwd_launch<__nv_bfloat16, 64>(a, st) : bwd_launch<__half, 64>(a, st);
  return dtype == KDA_DTYPE_BF16 ? bwd_launch<__nv_bfloat16, 128>(a, st) : bwd_launch<__half, 128>(a, st);
}

}  // namespace kda
