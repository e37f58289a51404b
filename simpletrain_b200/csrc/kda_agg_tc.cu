// Range aggregates for long streams (sm_100a, tcgen05 + TMEM + TMA).
//
// When (batch, head) streams are longer than a work range, the carry of a
// stream passes through several ranges.  The carry recurrences are linear with
// a diagonal (per key channel) decay, so the exit carry of a range's publishing
// piece (a middle range, or the piece that starts -- reverse: ends -- a
// stream) is
//
//   S_out = A S_in + S_loc,         A = decay^(64 n)   (n full chunks)
//   T_out = A T_in + 64 n A S_in + T_loc               (decay tangent)
//   dS_out = A dS_in + dS_loc                          (reverse pass; a piece
//                      that ends its stream holds the ragged last chunk)
//
// where the _loc terms are the same recurrences run from zero over the
// piece's chunks.
// This kernel computes carry_loc for every range (one CTA per range, all in
// parallel); each piece of the main kernels then folds its own entry carry
// from the stream's boundary carry and the aggregates of the ranges before it
// (entry_fold_kernel), so no range waits for another for its carry
// (kernels/kda_kernel.py:292-295 is the recurrence).
//
//   MODE 0  S_loc from K, V            (forward)
//   MODE 1  S_loc, T_loc from K, V     (backward, forward direction)
//   MODE 2  dS_loc from Q, dO          (backward, reverse direction)
//
// Warp 0 loads the two tiles of each chunk into a ring, warp 1 issues one
// UMMA per chunk (K^T V, literal K V^T, or Q^T dO) into one of two TMEM
// accumulators, warps 2-9 fold it into the fp32 carry in registers.  In
// per-step mode (PS) the fold applies a scalar factor, S <- a^64 S +
// a^(64-kRef) K~^T V with the k rows scaled first by warp 10 like in the main
// kernels (kda_tc_epi.cuh, kRef), or dS <- a^64 dS + a^kRef Q^T dO^ with the
// row-scaled dO^ the forward-direction pass wrote.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "kda_internal.h"
#include "kda_tc_epi.cuh"
#include "tmap.h"

namespace kda {
namespace {
using namespace tc;

template <int D, int NS>
struct AggLayout {
  static constexpr int KB = D / 64;
  static constexpr int BOX = KB * kTile;
  static constexpr int ST_A = 0, ST_B = BOX, STAGE = 2 * BOX;
  static constexpr int BAR = NS * STAGE;
  static constexpr int NBAR = 3 * NS + 8;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int SMEM = ABORT + 8 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * D <= 128 ? 128 : 256;  // two accumulators of D columns
};

// a row-scaler warp: per-step mode, k tiles (mode 0)
template <bool PS, int MODE>
constexpr bool agg_scales() { return PS && MODE == 0; }

template <typename T, int D, bool LIT, bool PS, int MODE, int NS>
__global__ void __launch_bounds__(kThreads + (agg_scales<PS, MODE>() ? 32 : 0), 1)
    agg_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const AggArgs a,
                  const Queue qu) {
  using L = AggLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool REV = MODE == 2;
  // this CTA's range: the aggregate of the piece through which it publishes a carry
  // (reverse: a piece that ends at its stream's end starts with the ragged last chunk,
  // whose own decay factor multiplies a zero carry here and enters the consumer's A)
  pdl_launch_dependents();  // entry_fold_kernel may start; it waits for this grid before reading
  const Span sp = span_of(qu, REV ? qu.nranges - 1 - (int)blockIdx.x : (int)blockIdx.x, REV);
  int stream, c_begin, c_end;
  if (!published_piece(qu, sp, REV, stream, c_begin, c_end)) return;
  const int n = c_end - c_begin;
  const int b = stream / a.H, h = stream - b * a.H;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  enum { ACC_FULL = 2 * NS, ACC_FREE = ACC_FULL + 2, FIN = ACC_FREE + 2, SCALED = FIN + 1 };
  const int FULL = 0, EMPTY = NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 1);
    }
    mbar_init(bar(ACC_FULL + 0), 1);
    mbar_init(bar(ACC_FULL + 1), 1);
    mbar_init(bar(ACC_FREE + 0), kEpi);
    mbar_init(bar(ACC_FREE + 1), kEpi);
    mbar_init(bar(FIN), 1);
    for (int s = 0; s < NS; ++s) mbar_init(bar(SCALED + s), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(sb + L::TMEM_SLOT, L::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::TMEM_SLOT);
  auto chunk_of = [&](int k) { return REV ? c_end - 1 - k : c_begin + k; };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tb);
      int k = 0;
      for (; k < n; ++k) {
        const int s = k % NS, use = k / NS, c = chunk_of(k);
        if (!mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag)) break;
        const uint32_t st = sb + s * L::STAGE;
        mbar_arrive_expect_tx(bar(FULL + s), (uint32_t)(2 * L::BOX));
        for (int kb = 0; kb < L::KB; ++kb) {
          tma_load_4d(st + L::ST_A + kb * kTile, &ta, bar(FULL + s), 64 * kb, 64 * c, h, b);
          tma_load_4d(st + L::ST_B + kb * kTile, &tb, bar(FULL + s), 64 * kb, 64 * c, h, b);
        }
      }
      for (int d = k - 1; d >= 0 && d >= k - NS; --d) mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // forward modes: K^T V (literal: K V^T); reverse: Q^T dO
      const uint32_t id = (LIT && !REV) ? idesc_f16(64, 64, BF, false, false) : idesc_f16(D, D, BF, true, true);
      for (int k = 0; k < n; ++k) {
        const int s = k % NS, use = k / NS, buf = k & 1;
        const uint32_t st = sb + s * L::STAGE;
        if (!(mbar_wait(bar((agg_scales<PS, MODE>() ? SCALED : FULL) + s), use & 1, a.status, abort_flag) &&
              mbar_wait(bar(ACC_FREE + buf), ((k >> 1) & 1) ^ 1, a.status, abort_flag)))
          break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks) {
          if (LIT && !REV)
            mma_f16(tmem + buf * D, sdesc_k(st + L::ST_A + ks * 32), sdesc_k(st + L::ST_B + ks * 32), id, ks > 0);
          else
            mma_f16(tmem + buf * D, sdesc_mn(st + L::ST_A + ks * 2048, kTile), sdesc_mn(st + L::ST_B + ks * 2048, kTile),
                    id, ks > 0);
        }
        mma_commit(bar(ACC_FULL + buf));
        mma_commit(bar(EMPTY + s));
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp < kThreads / 32) {
    const Epi e;
    Carry<D> S, Tn;
    S.init_rows(e);
    S.zero();
    Tn.row[0] = S.row[0];
    Tn.row[Carry<D>::NR - 1] = S.row[Carry<D>::NR - 1];
    Tn.zero();
    float al[Carry<D>::NR];
    for (int r = 0; r < Carry<D>::NR; ++r) al[r] = chunk_alpha(a.decay, b, h, S.row[r], 64, 64);
    float aw = 1.f;  // per-step factor of each chunk's product
    if constexpr (PS) aw = pow_log2(log2f(decay_value(a.decay, b, h, 0)), (float)(REV ? kRef : 64 - kRef));
    bool ok = true;
    for (int k = 0; k < n && ok; ++k) {
      const int buf = k & 1;
      if (!(ok = mbar_wait(bar(ACC_FULL + buf), (k >> 1) & 1, a.status, abort_flag))) break;
      tc_fence_after();
      if (D == 128) {
        for (int sl = 0; sl < Carry<D>::NV / 16; ++sl) {  // column slices of 16
          uint32_t u[16];
          tmem_ld_32x32b_x16(tmem + e.lane_off + buf * D + Carry<D>::W * e.cg + 16 * sl, u);
          for (int i = 0; i < 16; ++i) {
            float &sv = S.x[0][16 * sl + i];
            if (MODE == 1) Tn.x[0][16 * sl + i] = al[0] * fmaf(64.f, sv, Tn.x[0][16 * sl + i]);  // T <- a (T + L S)
            sv = fmaf(al[0], sv, aw * __uint_as_float(u[i]));
          }
        }
        tc_fence_before();
        mbar_arrive(bar(ACC_FREE + buf));
      } else {
        Carry<D> U;
        U.row[0] = S.row[0];
        U.row[Carry<D>::NR - 1] = S.row[Carry<D>::NR - 1];
        U.tmem_load(e, tmem, buf * D);
        tc_fence_before();
        mbar_arrive(bar(ACC_FREE + buf));
        for (int r = 0; r < Carry<D>::NR; ++r)
          for (int i = 0; i < Carry<D>::NV; ++i) {
            if (MODE == 1) Tn.x[r][i] = al[r] * fmaf(64.f, S.x[r][i], Tn.x[r][i]);  // T <- a (T + L S_prev)
            S.x[r][i] = fmaf(al[r], S.x[r][i], aw * U.x[r][i]);
          }
      }
    }
    if (ok) {
      float4 *dst = a.agg + (size_t)sp.r * a.agg_f4 * kEpi;
      S.store_slot(e, dst);
      if (MODE == 1) Tn.store_slot(e, dst + (Carry<D>::FLOATS / 4) * kEpi);
    }
  } else if constexpr (agg_scales<PS, MODE>()) {
    // row scaler: K~ rows a^(kRef-1-j) of tile A
    const float l2a = log2f(decay_value(a.decay, b, h, 0));
    const uint2 f0 = k_row_factor<BF>(l2a, lane), f1 = k_row_factor<BF>(l2a, lane + 32);
    for (int k = 0; k < n; ++k) {
      const int s = k % NS, use = k / NS;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag))) break;
      scale_tile_row<L::KB, BF>(sb + s * L::STAGE + L::ST_A, lane, f0);
      scale_tile_row<L::KB, BF>(sb + s * L::STAGE + L::ST_A, lane + 32, f1);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(SCALED + s));
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <typename T, int D, bool LIT, bool PS, int MODE>
cudaError_t agg_launch(const AggArgs &a, const View &va, const View &vb, const Queue &q, cudaStream_t st) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NS = 4;
  CUtensorMap ma, mb;
  if (!make_tmap_bhtd(&ma, va, a.B, a.H, a.T, D, BF) || !make_tmap_bhtd(&mb, vb, a.B, a.H, a.T, D, BF))
    return cudaErrorInvalidValue;
  using L = AggLayout<D, NS>;
  auto kern = agg_tc_kernel<T, D, LIT, PS, MODE, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return e;
  const int tr = trace_before(st);
  kern<<<q.nranges, kThreads + (agg_scales<PS, MODE>() ? 32 : 0), L::SMEM, st>>>(ma, mb, a, q);
  trace_after(tr, kTraceAgg, st);
  count_launches(1);
  return cudaGetLastError();
}

// Entry carries of long streams, after the aggregates.  One group of CTAs per
// stream that spans several ranges walks the ranges it spans once, in stream
// order (reverse: from the stream's end), folding the boundary carry x (initial
// state; reverse: final-state gradient; `boundary`, or zero) through the
// aggregate of each range's publishing piece,
//   x <- A_j x + x_loc_j    (with the tangent: t <- A_j t + 64 n_j A_j x + t_loc_j),
// A_j the product of piece j's chunk decays, and stores the carry entering the
// next range into that range boundary's slot, where the main kernel reads it
// without waiting.  Slots and aggregates follow the epilogue thread layout of
// the main kernels (a thread's carry registers in order); a CTA is that layout's
// 256 threads without the main kernels' producer warps, and grid (streams,
// parts) splits every thread's carry into parts of NP float4, NP chosen so the
// grid fits one wave: the aggregates of several links are loaded ahead of the
// multiply-adds that use them.  The fold order is fixed, so the result does not
// depend on timing.
constexpr int kMaxFoldLinks = 1024;  // links whose chunk counts are staged in shared memory

template <int D, bool REV, bool TAN, int NP>
__global__ void __launch_bounds__(kEpi) entry_fold_kernel(AggArgs a, Queue qu, const float *boundary) {
  pdl_launch_dependents();  // the main kernel may start; its epilogue waits for this grid
  const int stream = (int)blockIdx.x;
  const long long first = (long long)stream * qu.nchunks;
  const int j_lo = range_of(qu, first), j_hi = range_of(qu, first + qu.nchunks - 1);
  if (j_lo == j_hi) return;  // the stream lies in one range: no carry crosses a boundary
  constexpr int NV = Carry<D>::NV, N4 = Carry<D>::FLOATS / 4;
  static_assert(N4 % NP == 0 && NV % (4 * NP) == 0, "a part lies in one carry row");
  constexpr int U = (TAN ? 4 : 8) / NP > 0 ? (TAN ? 4 : 8) / NP : 1;  // links per batch of loads
  const Epi e(64 + (int)threadIdx.x);
  const int i0 = (int)blockIdx.y * NP;
  const int row = Carry<D>::row_of(e, (4 * i0) / NV);
  float4 x[NP], t[NP];
  for (int k = 0; k < NP; ++k) {
    x[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    t[k] = x[k];
    if (boundary) {
      const int c = (4 * (i0 + k)) % NV;
      const float *src = boundary + (size_t)stream * D * D + (size_t)row * D;
      const float2 lo = __ldg(reinterpret_cast<const float2 *>(src + Carry<D>::col_of(e, c)));
      const float2 hi = __ldg(reinterpret_cast<const float2 *>(src + Carry<D>::col_of(e, c + 2)));
      x[k] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
  }
  const int b = stream / a.H, h = stream - b * a.H;
  const int Ltail = a.T - (qu.nchunks - 1) * 64;
  const float af = chunk_alpha(a.decay, b, h, row, 64, 64), at = chunk_alpha(a.decay, b, h, row, Ltail, 64);

  // links in fold order: the range, and its piece's chunk count (negative: the
  // piece holds the stream's ragged last chunk), staged once by all threads --
  // a range's boundaries take 64-bit divisions
  const int nlinks = j_hi - j_lo;
  auto link_range = [&](int l) { return REV ? j_hi - l : j_lo + l; };
  auto link_chunks = [&](int l) {
    int s, cb, ce;
    published_piece(qu, span_of(qu, link_range(l), false), REV, s, cb, ce);
    return (REV && ce == qu.nchunks) ? -(ce - cb) : ce - cb;
  };
  __shared__ int link_n[kMaxFoldLinks];
  const bool staged = nlinks <= kMaxFoldLinks;
  if (staged) {
    for (int l = e.et; l < nlinks; l += kEpi) link_n[l] = link_chunks(l);
    __syncthreads();
  }
  pdl_wait();  // the aggregates: agg_tc_kernel, launched just before this grid

  int n_prev = 0;
  bool tail_prev = false;
  float A = 1.f;
  for (int base = 0; base < nlinks; base += U) {
    float4 g[U][NP], gt[U][TAN ? NP : 1];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (base + u < nlinks) {
        const float4 *ag = agg_ptr(qu, link_range(base + u));
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          g[u][k] = __ldcg(ag + (i0 + k) * kEpi + e.et);
          if constexpr (TAN) gt[u][k] = __ldcg(ag + (N4 + i0 + k) * kEpi + e.et);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int l = base + u;
      if (l >= nlinks) break;
      const int cn = staged ? link_n[l] : link_chunks(l);
      const int n = cn < 0 ? -cn : cn;
      const bool tail = cn < 0;
      if (n != n_prev || tail != tail_prev) {
        A = tail ? powf(af, (float)(n - 1)) * at : powf(af, (float)n);
        n_prev = n;
        tail_prev = tail;
      }
      // the carry entering the next range in fold order: its boundary slot
      // (forward: range j + 1's entry, slot j + 1; reverse: range j - 1's, slot j)
      const int j = link_range(l);
      float4 *slot = slot_ptr(qu, REV ? j : j + 1);
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        if constexpr (TAN) {
          const float An = 64.f * (float)n * A;
          t[k] = make_float4(fmaf(A, t[k].x, fmaf(An, x[k].x, gt[u][k].x)),
                             fmaf(A, t[k].y, fmaf(An, x[k].y, gt[u][k].y)),
                             fmaf(A, t[k].z, fmaf(An, x[k].z, gt[u][k].z)),
                             fmaf(A, t[k].w, fmaf(An, x[k].w, gt[u][k].w)));
        }
        x[k] = make_float4(fmaf(A, x[k].x, g[u][k].x), fmaf(A, x[k].y, g[u][k].y), fmaf(A, x[k].z, g[u][k].z),
                           fmaf(A, x[k].w, g[u][k].w));
        __stcg(slot + (i0 + k) * kEpi + e.et, x[k]);
        if constexpr (TAN) __stcg(slot + (N4 + i0 + k) * kEpi + e.et, t[k]);
      }
    }
  }
}

template <int D, bool REV, bool TAN>
cudaError_t fold_launch(const AggArgs &a, const Queue &q, const float *boundary, cudaStream_t st) {
  // float4 per thread per CTA: as few as fit one wave of two 256-thread CTAs per SM
  // (a part lies in one carry row: at most 4 float4 at D=128, 2 at D=64)
  constexpr int N4 = Carry<D>::FLOATS / 4, NP_MAX = Carry<D>::NV / 4 < 4 ? Carry<D>::NV / 4 : 4;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int np = 1;
  while (np < NP_MAX && (long long)q.nstreams * (N4 / np) > 2LL * sms) np *= 2;
  const int tr = trace_before(st);
  const dim3 grid(q.nstreams, N4 / np);
  cudaError_t e = cudaSuccess;
  if (np == 1) e = launch_kernel(entry_fold_kernel<D, REV, TAN, 1>, grid, dim3(kEpi), 0, st, true, a, q, boundary);
  else if (np == 2) e = launch_kernel(entry_fold_kernel<D, REV, TAN, 2>, grid, dim3(kEpi), 0, st, true, a, q, boundary);
  else if constexpr (NP_MAX >= 4)
    e = launch_kernel(entry_fold_kernel<D, REV, TAN, 4>, grid, dim3(kEpi), 0, st, true, a, q, boundary);
  trace_after(tr, kTraceFold, st);
  count_launches(1);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int MODE>
cudaError_t agg_dispatch(const AggArgs &a, const View &va, const View &vb, const Queue &q, int dtype,
                         cudaStream_t st) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if constexpr (MODE != 1) {
    if (a.per_step) {
      if (a.D == 64)
        return bf ? agg_launch<__nv_bfloat16, 64, false, true, MODE>(a, va, vb, q, st)
                  : agg_launch<__half, 64, false, true, MODE>(a, va, vb, q, st);
      return bf ? agg_launch<__nv_bfloat16, 128, false, true, MODE>(a, va, vb, q, st)
                : agg_launch<__half, 128, false, true, MODE>(a, va, vb, q, st);
    }
  }
  if (a.D == 64) {
    if (a.literal)
      return bf ? agg_launch<__nv_bfloat16, 64, true, false, MODE>(a, va, vb, q, st)
                : agg_launch<__half, 64, true, false, MODE>(a, va, vb, q, st);
    return bf ? agg_launch<__nv_bfloat16, 64, false, false, MODE>(a, va, vb, q, st)
              : agg_launch<__half, 64, false, false, MODE>(a, va, vb, q, st);
  }
  return bf ? agg_launch<__nv_bfloat16, 128, false, false, MODE>(a, va, vb, q, st)
            : agg_launch<__half, 128, false, false, MODE>(a, va, vb, q, st);
}

}  // namespace

cudaError_t launch_agg_tc(int mode, const AggArgs &a, const View &va, const View &vb, const tc::Queue &q, int dtype,
                          const float *boundary, cudaStream_t st) {
  cudaError_t e = mode == 0 ? agg_dispatch<0>(a, va, vb, q, dtype, st)
                  : mode == 1 ? agg_dispatch<1>(a, va, vb, q, dtype, st)
                              : agg_dispatch<2>(a, va, vb, q, dtype, st);
  if (e != cudaSuccess) return e;
  if (a.D == 64)
    return mode == 0 ? fold_launch<64, false, false>(a, q, boundary, st)
           : mode == 1 ? fold_launch<64, false, true>(a, q, boundary, st)
                       : fold_launch<64, true, false>(a, q, boundary, st);
  return mode == 0 ? fold_launch<128, false, false>(a, q, boundary, st)
         : mode == 1 ? fold_launch<128, false, true>(a, q, boundary, st)
                     : fold_launch<128, true, false>(a, q, boundary, st);
}

}  // namespace kda
