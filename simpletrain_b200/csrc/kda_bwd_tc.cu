// KDA chunked-scan backward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Two persistent kernels over (batch*head stream, segment) units
// (kda_tc_epi.cuh), each walking chunks of 64 tokens with a fp32 D x D carry.
// Gradients of the chunk loop in kernels/kda_kernel.py:269-296 (autograd
// there), with dO = dy * g, P = tril(Q K^T), dP = tril(dO V^T), W = Q^T dO:
//
// forward direction (carry S_{c-1}: recomputed, never stored; it lives in
// tensor memory and the K^T V product accumulates into it):
//   O = P V + Q S              -> dg = dy * O
//   dq = dO S^T + dP K
//   S <- decay^L S + K^T V     (literal: K V^T)
//   decay gradient, forward mode: the tangent T = dS/dlog(decay) (row-wise,
//   fp32 registers) obeys T <- decay^L (T + L S), and
//   dL/dlog decay[i] = sum_c <T_{c-1}[i,:], W_c[i,:]> + <dS_T[i,:], T_T[i,:]>.
// reverse direction (carry dS_c = dL/dS_c, fp32 registers):
//   dk = V dS^T + dP^T Q       (literal: dS V + dP^T Q)
//   dv = K dS + P^T dO         (literal: dS^T K + P^T dO)
//   dS <- decay^L dS + W
//
// Per-step decay (PS, one decay a per stream): k rows are scaled in the
// stage by two extra warps, K~ = diag(a^(kRef-1-j)) K, the forward-direction
// pass writes dO^ = diag(a^(i+1-kRef)) g dy for both passes, and with them
// (m = kRef, L the chunk length)
//   O  = diag(a^(i+1-m)) [tril(Q K~^T) V + Q (a^m S)]    -> dg = dy * O
//   dq = tril(dO^ V^T) K~ + dO^ (a^m S)^T                S <- a^L S + a^(L-m) K~^T V
//   dk = diag(a^(m-1-j)) [tril(dO^ V^T)^T Q + V (a^(L-m) dS)^T]
//   dv = tril(Q K~^T)^T dO^ + K~ (a^(L-m) dS)            dS <- a^L dS + a^m Q^T dO^
// i.e. the same products, scalar factors on the carries and a row factor on
// O and dk.  The decay is not differentiated in this mode.
//
// Warp 0: unit tickets + TMA loads (q, k, v, g, dy) into a two-stage ring;
// warp 1: tensor memory and the single MMA-issuing thread; warps 2-9:
// epilogue (PS: warps 10-11 scale k).  Outputs leave through TMA
// stores.  Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "kda_internal.h"
#include "kda_tc_epi.cuh"
#include "tmap.h"

KDA_TRACE_DEFINE

namespace kda {
namespace {
using namespace tc;


// forward-direction pass: stage = q, k, v, g, dy
// threads of a backward CTA: + two row-scaler warps in per-step mode
template <bool PS>
constexpr int bwd_threads() { return kThreads + (PS ? 64 : 0); }

template <int D, int NS>
struct BwdLayout {
  static constexpr int KB = D / 64;
  static constexpr int BOX = KB * kTile;  // one [64 tokens x D] tile
  static constexpr int ST_Q = 0, ST_K = BOX, ST_V = 2 * BOX, ST_G = 3 * BOX, ST_DY = 4 * BOX;
  static constexpr int STAGE = 5 * BOX;
  static constexpr int P = NS * STAGE;
  static constexpr int DP = P + kTile;
  static constexpr int DO = DP + kTile;
  static constexpr int PANEL = D * 128;  // [D rows x 64 columns] of the carried state operand
  static constexpr int SB = DO + BOX;
  static constexpr int BAR = SB + KB * PANEL;
  static constexpr int NBAR = 4 * NS + 20;
  static constexpr int RING = BAR + NBAR * 8;
  static constexpr int RED = RING + 16;   // float [D] row sums
  static constexpr int TMEM_SLOT = RED + 4 * D;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int SMEM = ABORT + 8 + 1024;
  static constexpr uint32_t A_QK = 0, A_DP = 64, A_X = 128, A_Y = 128 + D, A_Z = 128 + 2 * D;
  static constexpr uint32_t TMEM_COLS = 512;
};

// reverse pass: stage = q, k, v, dO (written by the forward-direction pass);
// dk and dv leave through two staging tiles and TMA stores
template <int D, int NS>
struct RevLayout {
  static constexpr int KB = D / 64;
  static constexpr int BOX = KB * kTile;
  static constexpr int ST_Q = 0, ST_K = BOX, ST_V = 2 * BOX, ST_DO = 3 * BOX;
  static constexpr int STAGE = 4 * BOX;
  static constexpr int P = NS * STAGE;
  static constexpr int DP = P + kTile;
  static constexpr int PANEL = D * 128;
  static constexpr int SB = DP + kTile;
  static constexpr int DK = SB + KB * PANEL;
  static constexpr int DV = DK + BOX;
  static constexpr int BAR = DV + BOX;
  static constexpr int NBAR = 4 * NS + 20;
  static constexpr int RING = BAR + NBAR * 8;
  static constexpr int TMEM_SLOT = RING + 16;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int SMEM = ABORT + 8 + 1024;
  static constexpr uint32_t A_QK = 0, A_DP = 64, A_X = 128, A_Y = 128 + D, A_Z = 128 + 2 * D;
  static constexpr uint32_t TMEM_COLS = 512;
};

// Piece-loop preamble shared by the MMA and epilogue roles.
#define KDA_TAKE_UNIT(REVERSE)                                                           \
  if (!mbar_wait(bar(UNIT_FULL0 + (i & 1)), (i >> 1) & 1, a.status, abort_flag)) break; \
  const int t = ring[2 * (i & 1)], p = ring[2 * (i & 1) + 1];                            \
  mbar_arrive(bar(UNIT_FREE0 + (i & 1)));                                                \
  if (t >= qu.nranges) break;                                                            \
  const Piece u = piece_of(qu, span_of(qu, t, REVERSE), p, REVERSE);

// Producer: tickets and TMA loads of the stage tiles for every chunk of every
// piece.  Stage slot j (BOX bytes each) is filled from maps[j]; a null map
// leaves its slot untouched (no gate).  KFULL >= 0 (per-step mode): slot 1,
// the k tile, is loaded first and completes barrier KFULL + stage instead.
template <int D, int NS, int NT>
__device__ void bwd_producer(const BwdArgs &a, const Queue &qu, bool reverse, uint32_t sb, int stage_bytes,
                             volatile int *ring, volatile int *abort_flag, const CUtensorMap *const (&maps)[NT],
                             uint32_t bar_base, int FULL, int EMPTY, int UNIT_FULL0, int UNIT_FREE0,
                             int KFULL = -1) {
  constexpr int KB = D / 64, BOX = KB * kTile;
  auto bar = [&](int i) { return bar_base + 8u * i; };
  int ntiles = 0;
  for (int j = 0; j < NT; ++j)
    if (maps[j]) {
      prefetch_tmap(maps[j]);
      ++ntiles;
    }
  const uint32_t tx = (uint32_t)((ntiles - (KFULL >= 0 ? 1 : 0)) * BOX);
  int gc = 0, i = 0;
  bool ok = true;
  while (ok) {
    const int t = atomicAdd(qu.ticket, 1);
    const Span sp = t < qu.nranges ? span_of(qu, t, reverse) : Span{};
    const int m = t < qu.nranges ? sp.npieces() : 1;
    for (int p = 0; p < m && ok; ++p, ++i) {
      if (!(ok = mbar_wait(bar(UNIT_FREE0 + (i & 1)), ((i >> 1) & 1) ^ 1, a.status, abort_flag))) break;
      ring[2 * (i & 1)] = t;
      ring[2 * (i & 1) + 1] = p;
      mbar_arrive(bar(UNIT_FULL0 + (i & 1)));
      if (t >= qu.nranges) { ok = false; break; }
      const Piece u = piece_of(qu, sp, p, reverse);
      const int b = u.stream / a.H, h = u.stream - b * a.H;
      const int n = u.c_end - u.c_begin;
      for (int k = 0; k < n; ++k, ++gc) {
        const int c = reverse ? u.c_end - 1 - k : u.c_begin + k;
        const int s = gc % NS, use = gc / NS;
        if (!(ok = mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag))) break;
        const uint32_t st = sb + s * stage_bytes;
        if (KFULL >= 0) {
          mbar_arrive_expect_tx(bar(KFULL + s), (uint32_t)BOX);
          for (int kb = 0; kb < KB; ++kb)
            tma_load_4d(st + BOX + kb * kTile, maps[1], bar(KFULL + s), 64 * kb, 64 * c, h, b);
        }
        mbar_arrive_expect_tx(bar(FULL + s), tx);
        for (int j = 0; j < NT; ++j)
          if (maps[j] && !(KFULL >= 0 && j == 1))
            for (int kb = 0; kb < KB; ++kb)
              tma_load_4d(st + j * BOX + kb * kTile, maps[j], bar(FULL + s), 64 * kb, 64 * c, h, b);
      }
    }
  }
  for (int d = gc - 1; d >= 0 && d >= gc - NS; --d) {
    mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
    if (KFULL >= 0) mbar_wait(bar(KFULL + d % NS), (d / NS) & 1, a.status, abort_flag);
  }
}

// ===========================================================================
// forward-direction pass: dq, dg, decay gradient
// ===========================================================================
template <typename T, int D, bool LIT, bool PS, int NS>
__global__ void __launch_bounds__(bwd_threads<PS>(), 1)
    bwd_fwddir_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                         const __grid_constant__ CUtensorMap tdy, const __grid_constant__ CUtensorMap tdq,
                         const __grid_constant__ CUtensorMap tdg, const __grid_constant__ CUtensorMap tdo,
                         const BwdArgs a, const Queue qu) {
  using L = BwdLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  // tensor memory: A_QK scores and A_DP dP, then together (A_DQ) dq; A_X O; A_Y W; A_Z the carried state
  constexpr uint32_t A_DQ = L::A_QK;
  enum {
    QK_FULL = 2 * NS, DO_FULL, W_FULL, S_READY, KV_FULL, P_FULL, DP_FULL, DPM_FULL, O_FULL, DQ_FULL, OUT_FREE,
    UNIT_FULL0, UNIT_FULL1, UNIT_FREE0, UNIT_FREE1, FIN, SCALED, KFULL = SCALED + NS
  };
  const int FULL = 0, EMPTY = NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  volatile int *ring = reinterpret_cast<volatile int *>(smem + L::RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool gate = a.g.data != nullptr;
  const bool want_dd = a.ddecay != nullptr;

  if (threadIdx.x == 0) {
    KDA_TRACE_CTA(0, kda_globaltimer());
    KDA_TRACE_CTA(7, kda_smid());
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 2);
    }
    mbar_init(bar(QK_FULL), 1);
    mbar_init(bar(DO_FULL), 1);
    mbar_init(bar(W_FULL), 1);
    mbar_init(bar(S_READY), 1);  // also: W read, tensor memory holds decay^L S_{c-1}
    mbar_init(bar(KV_FULL), 1);
    mbar_init(bar(P_FULL), 1);
    mbar_init(bar(DP_FULL), 1);
    mbar_init(bar(DPM_FULL), 1);  // also: the scores and dP were read
    mbar_init(bar(O_FULL), 1);
    mbar_init(bar(DQ_FULL), 1);
    mbar_init(bar(OUT_FREE), kEpi);  // O and dq were read
    mbar_init(bar(UNIT_FULL0), 1);
    mbar_init(bar(UNIT_FULL1), 1);
    mbar_init(bar(UNIT_FREE0), 1 + kEpi + (PS ? 2 : 0));
    mbar_init(bar(UNIT_FREE1), 1 + kEpi + (PS ? 2 : 0));
    mbar_init(bar(FIN), 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(SCALED + s), 2);
      mbar_init(bar(KFULL + s), 1);  // per-step: the k tile alone, loaded first
    }
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

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap *const maps[5] = {&tq, &tk, &tv, gate ? &tg : nullptr, &tdy};
      bwd_producer<D, NS, 5>(a, qu, false, sb, L::STAGE, ring, abort_flag, maps, sb + L::BAR, FULL, EMPTY, UNIT_FULL0,
                             UNIT_FREE0, PS ? (int)KFULL : -1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);  // Q K^T
      const uint32_t id_w = idesc_f16(D, D, BF, true, true);       // Q^T dO
      const uint32_t id_qs = idesc_f16(64, D, BF, false, true);    // Q S      (B = S, MN-major)
      const uint32_t id_kv = LIT ? idesc_f16(64, 64, BF, false, false) : idesc_f16(D, D, BF, true, true);
      const uint32_t id_pv = idesc_f16(64, D, BF, false, true);    // P V
      const uint32_t id_dp = idesc_f16(64, 64, BF, false, false);  // dO V^T
      const uint32_t id_ds = idesc_f16(64, D, BF, false, false);   // dO S^T   (B = S rows, K-major)
      const uint32_t id_dq = idesc_f16(64, D, BF, false, true);    // dP K     (B = K, MN-major)
      int gc = 0;
      for (int i = 0;; ++i) {
        KDA_TAKE_UNIT(false)
        bool ok = true;
        for (int c = u.c_begin; c < u.c_end; ++c, ++gc) {
          const int s = gc % NS, use = gc / NS, ph = gc & 1;
          const uint32_t st = sb + s * L::STAGE;
          // the last chunk's O and dq were read: A_QK, A_DP, A_X free
          if (!(ok = mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag) &&
                     (!PS || mbar_wait(bar(SCALED + s), use & 1, a.status, abort_flag)) &&
                     mbar_wait(bar(OUT_FREE), ph ^ 1, a.status, abort_flag)))
            break;
          KDA_TRACE_EVENT(13, gc);
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_QK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
          }
          mma_commit(bar(QK_FULL));
          // W = Q^T dO and dP = dO V^T once dO is staged
          if (!(ok = mbar_wait(bar(DO_FULL), ph, a.status, abort_flag))) break;
          KDA_TRACE_EVENT(14, gc);
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_DP, sdesc_k(sb + L::DO + off), sdesc_k(st + L::ST_V + off), id_dp, ks > 0);
          }
          mma_commit(bar(DP_FULL));
          if (want_dd)  // W feeds only the decay gradient
            for (int ks = 0; ks < 4; ++ks)
              mma_f16(tmem + L::A_Y, sdesc_mn(st + L::ST_Q + ks * 2048, kTile),
                      sdesc_mn(sb + L::DO + ks * 2048, kTile), id_w, ks > 0);
          mma_commit(bar(W_FULL));
          // intra-chunk parts while the epilogue steps the state: O = P V, dq = dP K
          if (!(ok = mbar_wait(bar(P_FULL), ph, a.status, abort_flag))) break;
          KDA_TRACE_EVENT(15, gc);
          tc_fence_after();
          for (int ks = 0; ks < 4; ++ks)
            mma_f16(tmem + L::A_X, sdesc_k(sb + L::P + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_pv,
                    ks > 0);
          if (!(ok = mbar_wait(bar(DPM_FULL), ph, a.status, abort_flag))) break;
          tc_fence_after();
          for (int ks = 0; ks < 4; ++ks)
            mma_f16(tmem + A_DQ, sdesc_k(sb + L::DP + ks * 32), sdesc_mn(st + L::ST_K + ks * 2048, kTile), id_dq,
                    ks > 0);
          // inter-chunk parts: O += Q S_{c-1}, dq += dO S_{c-1}^T, S += K^T V
          if (!(ok = mbar_wait(bar(S_READY), ph, a.status, abort_flag))) break;
          KDA_TRACE_EVENT(17, gc);
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_X, sdesc_k(st + L::ST_Q + off), sdesc_mn(sb + L::SB + ks * 2048, L::PANEL), id_qs, 1);
          }
          mma_commit(bar(O_FULL));
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
            mma_f16(tmem + A_DQ, sdesc_k(sb + L::DO + off), sdesc_k(sb + L::SB + poff), id_ds, 1);
          }
          mma_commit(bar(DQ_FULL));
          for (int ks = 0; ks < 4; ++ks) {
            if (LIT)
              mma_f16(tmem + L::A_Z, sdesc_k(st + L::ST_K + ks * 32), sdesc_k(st + L::ST_V + ks * 32), id_kv, 1);
            else
              mma_f16(tmem + L::A_Z, sdesc_mn(st + L::ST_K + ks * 2048, kTile),
                      sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_kv, 1);
          }
          mma_commit(bar(KV_FULL));
          mma_commit(bar(EMPTY + s));
        }
        if (!ok) break;
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp < kThreads / 32) {
    const Epi e;
    pdl_wait();  // long streams: the entry carries come from entry_fold_kernel, launched just before
    Carry<D> Td;  // decay tangent (fp32 registers)
    Td.init_rows(e);
    float dl[Carry<D>::NR];  // this thread's share of dL/dlog decay for its rows
    float *red = reinterpret_cast<float *>(smem + L::RED);
#ifdef KDA_TRACE
    // trace build: per-CTA totals of the epilogue's waits and steps (cycles)
    long long tw_full = 0, tw_qk = 0, tw_dp = 0, tw_s = 0, tw_o = 0, tw_dq = 0;
    long long ts_do = 0, ts_mask = 0, ts_rd = 0, ts_state = 0, ts_dg = 0, ts_dq = 0;
    long long ts_sl = 0, ts_wst = 0, ts_sync = 0;
#endif
    int gc = 0;
    for (int i = 0;; ++i) {
      KDA_TAKE_UNIT(false)
      const int b = u.stream / a.H, h = u.stream - b * a.H;
      const size_t sbase = (size_t)u.stream * D * D;
      // this thread's chunk decays: loaded before the boundary wait below (their round
      // trip overlaps it), raised to the chunk lengths after it
      float af[Carry<D>::NR], at[Carry<D>::NR];
      const int Ltail = a.T - (qu.nchunks - 1) * 64;
      for (int r = 0; r < Carry<D>::NR; ++r) af[r] = decay_value(a.decay, b, h, Td.row[r]);
      // entry state and tangent: the initial ones, or the ones at the range boundary
      // (long streams: folded there before this kernel started; no wait)
      const bool fold = u.folds(qu);
      if (!fold && !chain_wait(e, qu, u.wait_slot, a.status, abort_flag)) break;
      for (int r = 0; r < Carry<D>::NR; ++r) {
        const float dv = af[r];
        af[r] = chunk_alpha_of(a.decay, dv, 64, 64);
        at[r] = chunk_alpha_of(a.decay, dv, Ltail, 64);
      }
      if (e.et == 0 && i < 2) {
        KDA_TRACE_CTA(3 + 2 * i, kda_globaltimer());
        if (i == 0) KDA_TRACE_CTA(1, t);
      }
      const float4 *prev = u.wait_slot >= 0 ? slot_ptr(qu, u.wait_slot) : nullptr;
      constexpr int CF4 = Carry<D>::FLOATS / 4;  // float4 per thread of one carry
      // the previous range's decay-gradient share is added at the end of the piece
      for (int r = 0; r < Carry<D>::NR; ++r) dl[r] = 0.f;
      // D=128 (chunk-constant decay): the entry state goes to tensor memory here, its
      // loads issued together with the tangent's, so the piece's first state step reads
      // it from tensor memory like every later one instead of from global memory in
      // four dependent column slices (tensor memory's state column block is free: the
      // previous piece's last K^T V was read at its end, the next is issued after this
      // piece's first state step)
      bool entry_in_tmem = false;
      if constexpr (D == 128 && !PS) {
        if (prev || a.s_in) {
          float4 v[CF4];
          if (prev) {
            for (int i4 = 0; i4 < CF4; ++i4) v[i4] = __ldcg(prev + i4 * kEpi + e.et);
          } else {
            const float4 *s4 = reinterpret_cast<const float4 *>(a.s_in + sbase + (size_t)Td.row[0] * D +
                                                                 Carry<D>::W * e.cg);
            for (int i4 = 0; i4 < CF4; ++i4) v[i4] = __ldg(s4 + i4);
          }
          if (prev) Td.load_slot(e, prev + CF4 * kEpi);
          else Td.zero();
          for (int half = 0; half < 2; ++half) {
            uint32_t u32[32];
            for (int q4 = 0; q4 < 8; ++q4) {
              const float4 x = v[8 * half + q4];
              u32[4 * q4] = __float_as_uint(x.x); u32[4 * q4 + 1] = __float_as_uint(x.y);
              u32[4 * q4 + 2] = __float_as_uint(x.z); u32[4 * q4 + 3] = __float_as_uint(x.w);
            }
            tmem_st_32x32b_x32_nowait(tmem + e.lane_off + L::A_Z + Carry<D>::W * e.cg + 32 * half, u32);
          }
          tmem_wait_st();
          entry_in_tmem = true;
        } else {
          Td.zero();
        }
      } else {
        if (prev && !PS) Td.load_slot(e, prev + CF4 * kEpi);  // per-step mode carries no tangent
        else Td.zero();
      }
      if (e.et == 0) KDA_TRACE_EVENT(16, gc);  // piece preamble done
      // per-step: carry factors a^kRef (operand of the first chunk), a^(64-kRef)
      // (tensor-memory carry -> state), the O row factors a^(row+1-kRef) for
      // rows r0 and r0 + 8, and the factor of this thread's dO row
      float am = 1.f, au_f = 1.f, rq[2] = {1.f, 1.f}, rdo = 1.f;
      if constexpr (PS) {
        const float l2a = log2f(decay_value(a.decay, b, h, 0));
        am = pow_log2(l2a, (float)kRef);
        au_f = pow_log2(l2a, (float)(64 - kRef));
        for (int ee = 0; ee < 2; ++ee) rq[ee] = pow_log2(l2a, (float)(e.r0 + 8 * ee + 1 - kRef));
        rdo = pow_log2(l2a, (float)(make_do_row(e.et) + 1 - kRef));
      }
      bool ok = true;
      for (int c = u.c_begin; c < u.c_end; ++c, ++gc) {
        const int s = gc % NS, use = gc / NS, ph = gc & 1;
        const uint32_t st = sb + s * L::STAGE;
        const int t0 = 64 * c, Lc = min(64, a.T - t0);
        if (!(ok = KDA_TIMED(tw_full, mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)))) break;
        KDA_CLK(kc0);
        if (e.et == 0) KDA_TRACE_EVENT(0, gc);
        // (0) dO (the DO tile's last readers were the previous chunk's MMAs)
        if (e.et == 0) KDA_TRACE_EVENT(27, gc);
        make_do<D, BF, PS>(e, st + L::ST_G, st + L::ST_DY, sb + L::DO, gate, rdo);
        if (e.et == 0) KDA_TRACE_EVENT(28, gc);
        fence_async_smem();
        if (e.et == 0) KDA_TRACE_EVENT(29, gc);
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          KDA_TRACE_EVENT(30, gc);
          mbar_arrive(bar(DO_FULL));
          // dO also goes to the workspace, where the reverse pass reads it
          for (int kb = 0; kb < L::KB; ++kb) tma_store_4d(&tdo, sb + L::DO + kb * kTile, 64 * kb, t0, h, b);
          tma_store_commit();
          KDA_TRACE_EVENT(1, gc);
        }
        KDA_ADD(ts_do, kc0);
        KDA_CLK(kc1);
        // (a) P, (b) dP
        if (!(ok = KDA_TIMED(tw_qk, mbar_wait(bar(QK_FULL), ph, a.status, abort_flag)))) break;
        if (e.et == 0) KDA_TRACE_EVENT(5, gc);
        tc_fence_after();
        masked_tile<BF>(e, tmem + e.lane_off + L::A_QK, sb + L::P);
        if (e.et == 0) KDA_TRACE_EVENT(31, gc);
        if (!(ok = KDA_TIMED(tw_dp, mbar_wait(bar(DP_FULL), ph, a.status, abort_flag)))) break;
        if (e.et == 0) KDA_TRACE_EVENT(6, gc);
        tc_fence_after();
        masked_tile<BF>(e, tmem + e.lane_off + L::A_DP, sb + L::DP);
        fence_async_smem();
        if (e.et == 0) {
          // this chunk's dO store has read the DO tile (rewritten next chunk), and the last
          // chunk's dg / dq stores have read its stage: hand that stage back
          KDA_CLK(kr);
          tma_store_wait_read<0>();
          KDA_ADD(ts_rd, kr);
          if (gc > 0) mbar_arrive(bar(EMPTY + (gc - 1) % NS));
        }
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          mbar_arrive(bar(P_FULL));
          mbar_arrive(bar(DPM_FULL));
          KDA_TRACE_EVENT(7, gc);
        }
        KDA_ADD(ts_mask, kc1);
        KDA_CLK(kc2);
        // (s) state step: S_{c-1} -> operand, decay^L S_{c-1} -> tensor memory,
        //     decay term <T_{c-1}, W_c>, tangent update; column slices of 32
        if (c > u.c_begin && !(ok = KDA_TIMED(tw_s, mbar_wait(bar(KV_FULL), (gc - 1) & 1, a.status, abort_flag)))) break;
        if (!(ok = KDA_TIMED(tw_s, mbar_wait(bar(W_FULL), ph, a.status, abort_flag)))) break;
        if (e.et == 0) KDA_TRACE_EVENT(2, gc);
        tc_fence_after();
        {
          float alr[Carry<D>::NR];
          for (int r = 0; r < Carry<D>::NR; ++r) alr[r] = (Lc == 64) ? af[r] : at[r];
          const float Lf = (float)Lc;
          // factors of the loaded carry for the operand and for tensor memory; per-step:
          // both a^kRef S_{c-1}.  Past the first chunk tensor memory holds
          // Z = a^(kRef-64) S_{c-1}, brought back to S_{c-1} by a^(64-kRef) first: the
          // single factor a^64 would flush to zero in fp32 for a < 2^(-126/64) ~ 0.26
          float sop = 1.f, stm = alr[0], pre = 1.f;
          if constexpr (PS) {
            sop = stm = am;
            if (c != u.c_begin) pre = au_f;
          }
          if (D == 128) {
            const int row = Td.row[0];
            constexpr int W = Carry<D>::W;
            // column slices of SW, one tensor-memory round trip each: 32 without the
            // decay gradient, 16 when W and the tangent come along (register budget)
            auto slices = [&](auto swc) {
              constexpr int SW = decltype(swc)::value;
              for (int sl = 0; sl < W / SW; ++sl) {
                const int col0 = W * e.cg + SW * sl;
                const uint32_t pb = sb + L::SB + (uint32_t)((col0 >> 6) * L::PANEL);
                const uint32_t tz = tmem + e.lane_off + L::A_Z + col0, tw = tmem + e.lane_off + L::A_Y + col0;
                uint32_t u32[SW], w32[SW];
                if (c == u.c_begin && !entry_in_tmem) {
                  if (prev) {
                    for (int q4 = 0; q4 < SW / 4; ++q4) {
                      const float4 v = __ldcg(prev + ((SW / 4) * sl + q4) * kEpi + e.et);
                      u32[4 * q4] = __float_as_uint(v.x); u32[4 * q4 + 1] = __float_as_uint(v.y);
                      u32[4 * q4 + 2] = __float_as_uint(v.z); u32[4 * q4 + 3] = __float_as_uint(v.w);
                    }
                  } else if (a.s_in) {
                    const float4 *s4 = reinterpret_cast<const float4 *>(a.s_in + sbase + (size_t)row * D + col0);
                    for (int q4 = 0; q4 < SW / 4; ++q4) {
                      const float4 v = __ldg(s4 + q4);
                      u32[4 * q4] = __float_as_uint(v.x); u32[4 * q4 + 1] = __float_as_uint(v.y);
                      u32[4 * q4 + 2] = __float_as_uint(v.z); u32[4 * q4 + 3] = __float_as_uint(v.w);
                    }
                  } else {
                    for (int k = 0; k < SW; ++k) u32[k] = 0u;
                  }
                  if (want_dd) {
                    if constexpr (SW == 16) tmem_ld_32x32b_x16(tw, w32);
                    else tmem_ld_32x32b_x32(tw, w32);
                  }
                } else if constexpr (SW == 16) {
                  if (want_dd) tmem_ld2_32x32b_x16(tz, u32, tw, w32);
                  else tmem_ld_32x32b_x16(tz, u32);
                } else {
                  if (want_dd) {
                    tmem_ld_32x32b_x32_nowait(tz, u32);
                    tmem_ld_32x32b_x32_nowait(tw, w32);
                    tmem_wait_ld_bind(u32, w32);
                  } else {
                    tmem_ld_32x32b_x32(tz, u32);
                  }
                }
                if constexpr (PS)
                  for (int k = 0; k < SW; ++k) u32[k] = __float_as_uint(pre * __uint_as_float(u32[k]));
                if (want_dd) {
                  float acc = 0.f;
                  for (int k = 0; k < SW; ++k) acc = fmaf(Td.x[0][SW * sl + k], __uint_as_float(w32[k]), acc);
                  dl[0] += acc;
                }
                for (int j = 0; j < SW / 8; ++j)
                  st_shared_v4(pb + swz(row, (col0 & 63) + 8 * j),
                               pack2(sop * __uint_as_float(u32[8 * j]), sop * __uint_as_float(u32[8 * j + 1]), BF),
                               pack2(sop * __uint_as_float(u32[8 * j + 2]), sop * __uint_as_float(u32[8 * j + 3]), BF),
                               pack2(sop * __uint_as_float(u32[8 * j + 4]), sop * __uint_as_float(u32[8 * j + 5]), BF),
                               pack2(sop * __uint_as_float(u32[8 * j + 6]), sop * __uint_as_float(u32[8 * j + 7]), BF));
                for (int k = 0; k < SW; ++k) {
                  const float sv = __uint_as_float(u32[k]);
                  if (!PS && want_dd) Td.x[0][SW * sl + k] = alr[0] * fmaf(Lf, sv, Td.x[0][SW * sl + k]);
                  u32[k] = __float_as_uint(stm * sv);
                }
                if constexpr (SW == 16) tmem_st_32x32b_x16_nowait(tz, u32);
                else tmem_st_32x32b_x32_nowait(tz, u32);
              }
            };
            KDA_CLK(ks0);
            if (want_dd) slices(std::integral_constant<int, 16>{});
            else slices(std::integral_constant<int, 32>{});
            KDA_ADD(ts_sl, ks0);
            KDA_CLK(ks1);
            tmem_wait_st();
            KDA_ADD(ts_wst, ks1);
          } else {
            Carry<D> Sp;
            Sp.row[0] = Td.row[0];
            Sp.row[Carry<D>::NR - 1] = Td.row[Carry<D>::NR - 1];
            if (c == u.c_begin) {
              if (prev) Sp.load_slot(e, prev);
              else Sp.load_rm(e, a.s_in ? a.s_in + sbase : nullptr);
            } else {
              Sp.tmem_load(e, tmem, L::A_Z);
              if constexpr (PS)
                for (int r = 0; r < Carry<D>::NR; ++r)
                  for (int k = 0; k < Carry<D>::NV; ++k) Sp.x[r][k] *= pre;
            }
            if (want_dd) {
              Carry<D> W;
              W.tmem_load(e, tmem, L::A_Y);
              for (int r = 0; r < Carry<D>::NR; ++r)
                for (int k = 0; k < Carry<D>::NV; ++k) dl[r] = fmaf(Td.x[r][k], W.x[r][k], dl[r]);
            }
            Sp.template write_operand<BF>(e, sb + L::SB, sop);
            for (int r = 0; r < Carry<D>::NR; ++r)
              for (int k = 0; k < Carry<D>::NV; ++k) {
                if (!PS && want_dd) Td.x[r][k] = alr[r] * fmaf(Lf, Sp.x[r][k], Td.x[r][k]);
                Sp.x[r][k] *= PS ? stm : alr[r];
              }
            Sp.tmem_store(e, tmem, L::A_Z);
          }
        }
        if (e.et == 0) KDA_TRACE_EVENT(3, gc);
        KDA_CLK(ks2);
        fence_async_smem();
        tc_fence_before();
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          mbar_arrive(bar(S_READY));
          KDA_TRACE_EVENT(4, gc);
        }
        KDA_ADD(ts_sync, ks2);
        KDA_ADD(ts_state, kc2);
        KDA_CLK(kc3);
        // (c) dg = dy * O over the dy tile, then a TMA store
        if (!(ok = KDA_TIMED(tw_o, mbar_wait(bar(O_FULL), ph, a.status, abort_flag)))) break;
        if (e.et == 0) KDA_TRACE_EVENT(8, gc);
        tc_fence_after();
        if (gate) {
          frag_to_tile<D, BF>(e, tmem + e.lane_off + L::A_X, st + L::ST_DY, st + L::ST_DY, true, rq);
          fence_async_smem();
          named_bar_sync(1, kEpi);
          if (e.et == 0) {
            for (int kb = 0; kb < L::KB; ++kb) tma_store_4d(&tdg, st + L::ST_DY + kb * kTile, 64 * kb, t0, h, b);
            tma_store_commit();
          }
        }
        if (e.et == 0) KDA_TRACE_EVENT(9, gc);
        KDA_ADD(ts_dg, kc3);
        KDA_CLK(kc4);
        // (d) dq over the stage's gate tile (read only by the dO step), then a TMA store
        if (!(ok = KDA_TIMED(tw_dq, mbar_wait(bar(DQ_FULL), ph, a.status, abort_flag)))) break;
        tc_fence_after();
        frag_to_tile<D, BF>(e, tmem + e.lane_off + A_DQ, st + L::ST_G, 0, false);
        tc_fence_before();
        mbar_arrive(bar(OUT_FREE));
        fence_async_smem();
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          for (int kb = 0; kb < L::KB; ++kb) tma_store_4d(&tdq, st + L::ST_G + kb * kTile, 64 * kb, t0, h, b);
          tma_store_commit();
          KDA_TRACE_EVENT(10, gc);
        }
        if (e.et == 0) KDA_TRACE_EVENT(12, gc);
        KDA_ADD(ts_dq, kc4);
      }
      if (!ok) break;
      if (e.et == 0 && i < 2) KDA_TRACE_CTA(4 + 2 * i, kda_globaltimer());
      // piece end: the last K^T V has landed in tensor memory
      if (!mbar_wait(bar(KV_FULL), (gc - 1) & 1, a.status, abort_flag)) break;
      tc_fence_after();
      if (want_dd && prev && u.pub_slot < 0) {
        // the piece that ends a stream begun in earlier ranges adds their shares of
        // the decay gradient (each range publishes only its own, at level 2): all
        // flags are waited for at once, then the shares are summed in stream order,
        // so the sum is the same whichever range finished first
        const int j0 = range_of(qu, (long long)u.stream * qu.nchunks);
        if (!shares_wait(e, qu, j0 + 1, u.range + 1, a.status, abort_flag)) break;
#pragma unroll 4
        for (int j = j0; j < u.range; ++j) {
          const float4 v = __ldcg(slot_ptr(qu, j + 1) + 2 * CF4 * kEpi + e.et);
          dl[0] += v.x;
          if (Carry<D>::NR > 1) dl[Carry<D>::NR - 1] += v.y;
        }
      }
      if (u.pub_slot >= 0) {
        float4 *slot = slot_ptr(qu, u.pub_slot);
        if (!fold) {
          Carry<D> S;
          S.row[0] = Td.row[0];
          S.row[Carry<D>::NR - 1] = Td.row[Carry<D>::NR - 1];
          S.tmem_load(e, tmem, L::A_Z);
          if constexpr (PS)  // tensor memory holds a^(kRef-64) S after a full chunk
            for (int r = 0; r < Carry<D>::NR; ++r)
              for (int k = 0; k < Carry<D>::NV; ++k) S.x[r][k] *= au_f;
          S.store_slot(e, slot);
          Td.store_slot(e, slot + CF4 * kEpi);
        }
        __stcg(slot + 2 * CF4 * kEpi + e.et, make_float4(dl[0], dl[Carry<D>::NR - 1], 0.f, 0.f));
        tc_fence_before();
        chain_publish(e, qu, u.pub_slot, 2);
        if (e.et == 0) KDA_TRACE_EVENT(11, gc);  // exit carry published
      } else if (want_dd) {
        // <dS_T, T_T> row-wise, then the two column halves of every row meet in smem
        if (a.ds_out) {
          Carry<D> dST;
          dST.row[0] = Td.row[0];
          dST.row[Carry<D>::NR - 1] = Td.row[Carry<D>::NR - 1];
          dST.load_rm(e, a.ds_out + sbase);
          for (int r = 0; r < Carry<D>::NR; ++r)
            for (int k = 0; k < Carry<D>::NV; ++k) dl[r] = fmaf(dST.x[r][k], Td.x[r][k], dl[r]);
        }
        named_bar_sync(1, kEpi);
        if (e.et < D) red[e.et] = 0.f;
        named_bar_sync(1, kEpi);
        for (int r = 0; r < Carry<D>::NR; ++r) atomicAdd(&red[Td.row[r]], dl[r]);
        named_bar_sync(1, kEpi);
        if (e.et < D) {
          const float av = decay_value(a.decay, b, h, e.et);
          a.ddecay[(size_t)u.stream * D + e.et] = (av != 0.f) ? red[e.et] / av : 0.f;
        }
        tc_fence_before();
      }
    }
    if (e.et == 0) {  // trace build: per-CTA totals (cycles) of waits and steps
      KDA_TRACE_CTA(8, tw_s);
      KDA_TRACE_CTA(9, ts_do);
      KDA_TRACE_CTA(10, ts_mask);
      KDA_TRACE_CTA(11, ts_sl);
      KDA_TRACE_CTA(12, ts_state);
      KDA_TRACE_CTA(13, ts_wst);
      KDA_TRACE_CTA(14, ts_sync);
      KDA_TRACE_CTA(15, gc);
    }
  } else if constexpr (PS) {
    scaler_role<D, BF, NS>(qu, false, a.H, a.decay, sb, L::STAGE, L::ST_K, warp - kThreads / 32, ring, abort_flag,
                           a.status, sb + L::BAR, KFULL, SCALED, UNIT_FULL0, UNIT_FREE0);
  }
  if (threadIdx.x == 64) {
    tma_store_wait_all();  // dg / dq stores of the last chunk
    KDA_TRACE_CTA(2, kda_globaltimer());
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ===========================================================================
// reverse pass: dk, dv, d(initial state)
// ===========================================================================
template <typename T, int D, bool LIT, bool PS, int NS>
__global__ void __launch_bounds__(bwd_threads<PS>(), 1)
    bwd_revdir_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tdk, const __grid_constant__ CUtensorMap tdv,
                         const BwdArgs a, const Queue qu) {
  using L = RevLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  // D=128, chunk-constant decay: dk and dv are accumulated transposed (M = 128 over the
  // head dimension, N = 64 tokens: full-height tcgen05 tiles instead of M=64 ones) and
  // written back through transposing stores; literal and per-step keep the M=64 form.
  constexpr bool TR = !LIT && !PS && D == 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  // tensor memory: A_QK scores, A_DP dP, A_X dk, A_Y dv, A_Z W = Q^T dO
  enum {
    QK_FULL = 2 * NS, QK_FREE, DP_FULL, DP_FREE, W_FULL, W_FREE, DS_READY, DKV_FREE, INTER_FULL, P_FULL, DPM_FULL,
    DKV_FULL, UNIT_FULL0, UNIT_FULL1, UNIT_FREE0, UNIT_FREE1, FIN, SCALED, KFULL = SCALED + NS
  };
  const int FULL = 0, EMPTY = NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  volatile int *ring = reinterpret_cast<volatile int *>(smem + L::RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 1);  // MMA commit (the epilogue reads nothing from the stage)
    }
    mbar_init(bar(QK_FULL), 1);
    mbar_init(bar(QK_FREE), kEpi);
    mbar_init(bar(DP_FULL), 1);
    mbar_init(bar(DP_FREE), kEpi);
    mbar_init(bar(W_FULL), 1);
    mbar_init(bar(W_FREE), kEpi);
    mbar_init(bar(DS_READY), 1);
    mbar_init(bar(DKV_FREE), kEpi);
    mbar_init(bar(INTER_FULL), 1);
    mbar_init(bar(P_FULL), 1);
    mbar_init(bar(DPM_FULL), 1);
    mbar_init(bar(DKV_FULL), 1);
    mbar_init(bar(UNIT_FULL0), 1);
    mbar_init(bar(UNIT_FULL1), 1);
    mbar_init(bar(UNIT_FREE0), 1 + kEpi + (PS ? 2 : 0));
    mbar_init(bar(UNIT_FREE1), 1 + kEpi + (PS ? 2 : 0));
    mbar_init(bar(FIN), 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(SCALED + s), 2);
      mbar_init(bar(KFULL + s), 1);  // per-step: the k tile alone, loaded first
    }
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

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap *const maps[4] = {&tq, &tk, &tv, &tdo};
      bwd_producer<D, NS, 4>(a, qu, true, sb, L::STAGE, ring, abort_flag, maps, sb + L::BAR, FULL, EMPTY, UNIT_FULL0,
                             UNIT_FREE0, PS ? (int)KFULL : -1);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);
      const uint32_t id_dp = idesc_f16(64, 64, BF, false, false);
      const uint32_t id_w = idesc_f16(D, D, BF, true, true);  // Q^T dO
      const uint32_t id_dki = LIT ? idesc_f16(64, 64, BF, false, true) : idesc_f16(64, D, BF, false, false);
      const uint32_t id_dvi = LIT ? idesc_f16(64, 64, BF, true, true) : idesc_f16(64, D, BF, false, true);
      const uint32_t id_t = idesc_f16(64, D, BF, true, true);  // dP^T Q and P^T dO
      // transposed dk / dv (TR): M = D over the head dimension, N = 64 tokens
      const uint32_t id_dkt = idesc_f16(D, 64, BF, false, false);  // dS V^T
      const uint32_t id_dvt = idesc_f16(D, 64, BF, true, false);   // dS^T K^T
      const uint32_t id_tt = idesc_f16(D, 64, BF, true, true);     // Q^T dP and dO^T P
      int gc = 0;
      for (int i = 0;; ++i) {
        KDA_TAKE_UNIT(true)
        bool ok = true;
        for (int k = 0; k < u.c_end - u.c_begin; ++k, ++gc) {
          const int s = gc % NS, use = gc / NS, ph = gc & 1;
          const uint32_t st = sb + s * L::STAGE;
          if (!(ok = mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag) &&
                     (!PS || mbar_wait(bar(SCALED + s), use & 1, a.status, abort_flag)) &&
                     mbar_wait(bar(QK_FREE), ph ^ 1, a.status, abort_flag)))
            break;
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_QK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
          }
          mma_commit(bar(QK_FULL));
          if (!(ok = mbar_wait(bar(DP_FREE), ph ^ 1, a.status, abort_flag) &&
                     mbar_wait(bar(W_FREE), ph ^ 1, a.status, abort_flag)))
            break;
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_DP, sdesc_k(st + L::ST_DO + off), sdesc_k(st + L::ST_V + off), id_dp, ks > 0);
          }
          mma_commit(bar(DP_FULL));
          for (int ks = 0; ks < 4; ++ks)
            mma_f16(tmem + L::A_Z, sdesc_mn(st + L::ST_Q + ks * 2048, kTile),
                    sdesc_mn(st + L::ST_DO + ks * 2048, kTile), id_w, ks > 0);
          mma_commit(bar(W_FULL));
          if (!(ok = mbar_wait(bar(DS_READY), ph, a.status, abort_flag) &&
                     mbar_wait(bar(DKV_FREE), ph ^ 1, a.status, abort_flag)))
            break;
          tc_fence_after();
          if (LIT) {
            for (int ks = 0; ks < 4; ++ks) {
              mma_f16(tmem + L::A_X, sdesc_k(sb + L::SB + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_dki,
                      ks > 0);
              mma_f16(tmem + L::A_Y, sdesc_mn(sb + L::SB + ks * 2048, L::PANEL),
                      sdesc_mn(st + L::ST_K + ks * 2048, kTile), id_dvi, ks > 0);
            }
          } else if (TR) {
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
              const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
              mma_f16(tmem + L::A_X, sdesc_k(sb + L::SB + poff), sdesc_k(st + L::ST_V + off), id_dkt, ks > 0);
              mma_f16(tmem + L::A_Y, sdesc_mn(sb + L::SB + ks * 2048, L::PANEL), sdesc_k(st + L::ST_K + off), id_dvt,
                      ks > 0);
            }
          } else {
            for (int ks = 0; ks < D / 16; ++ks) {
              const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
              const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
              mma_f16(tmem + L::A_X, sdesc_k(st + L::ST_V + off), sdesc_k(sb + L::SB + poff), id_dki, ks > 0);
              mma_f16(tmem + L::A_Y, sdesc_k(st + L::ST_K + off), sdesc_mn(sb + L::SB + ks * 2048, L::PANEL), id_dvi,
                      ks > 0);
            }
          }
          mma_commit(bar(INTER_FULL));
          if (!(ok = mbar_wait(bar(P_FULL), ph, a.status, abort_flag) &&
                     mbar_wait(bar(DPM_FULL), ph, a.status, abort_flag)))
            break;
          tc_fence_after();
          for (int ks = 0; ks < 4; ++ks) {
            if (TR) {
              mma_f16(tmem + L::A_X, sdesc_mn(st + L::ST_Q + ks * 2048, kTile), sdesc_mn(sb + L::DP + ks * 2048, kTile),
                      id_tt, 1);
              mma_f16(tmem + L::A_Y, sdesc_mn(st + L::ST_DO + ks * 2048, kTile), sdesc_mn(sb + L::P + ks * 2048, kTile),
                      id_tt, 1);
            } else {
              mma_f16(tmem + L::A_X, sdesc_mn(sb + L::DP + ks * 2048, kTile), sdesc_mn(st + L::ST_Q + ks * 2048, kTile),
                      id_t, 1);
              mma_f16(tmem + L::A_Y, sdesc_mn(sb + L::P + ks * 2048, kTile), sdesc_mn(st + L::ST_DO + ks * 2048, kTile),
                      id_t, 1);
            }
          }
          mma_commit(bar(DKV_FULL));
          mma_commit(bar(EMPTY + s));
        }
        if (!ok) break;
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp < kThreads / 32) {
    const Epi e;
    pdl_wait();  // long streams: the entry carries come from entry_fold_kernel, launched just before
    Carry<D> dS;
    dS.init_rows(e);
    int gc = 0;
    for (int i = 0;; ++i) {
      KDA_TAKE_UNIT(true)
      const int b = u.stream / a.H, h = u.stream - b * a.H;
      const size_t sbase = (size_t)u.stream * D * D;
      // this thread's chunk decays: loaded before the boundary wait below (their round
      // trip overlaps it), raised to the chunk lengths after it
      float af[Carry<D>::NR], at[Carry<D>::NR];
      const int Ltail = a.T - (qu.nchunks - 1) * 64;
      for (int r = 0; r < Carry<D>::NR; ++r) af[r] = decay_value(a.decay, b, h, dS.row[r]);
      // dS at the piece's end: the final-state gradient, or the one at the range boundary
      // (long streams: folded there before this kernel started; no wait)
      const bool fold = u.folds(qu);
      if (!fold && !chain_wait(e, qu, u.wait_slot, a.status, abort_flag)) break;
      for (int r = 0; r < Carry<D>::NR; ++r) {
        const float dv = af[r];
        af[r] = chunk_alpha_of(a.decay, dv, 64, 64);
        at[r] = chunk_alpha_of(a.decay, dv, Ltail, 64);
      }
      if (u.wait_slot < 0) dS.load_rm(e, a.ds_out ? a.ds_out + sbase : nullptr);
      else dS.load_slot(e, slot_ptr(qu, u.wait_slot));
      // per-step: W factor a^kRef, operand factor a^(L-kRef) for the chunk that
      // reads it (full, or the stream's tail chunk first), dk row factors a^(kRef-1-row)
      float am = 1.f, ad_f = 1.f, ad_0 = 1.f, rk[2] = {1.f, 1.f};
      if constexpr (PS) {
        const float l2a = log2f(decay_value(a.decay, b, h, 0));
        const int L0 = min(64, a.T - 64 * (u.c_end - 1));
        am = pow_log2(l2a, (float)kRef);
        ad_f = pow_log2(l2a, (float)(64 - kRef));
        ad_0 = pow_log2(l2a, (float)(L0 - kRef));
        for (int ee = 0; ee < 2; ++ee) rk[ee] = pow_log2(l2a, (float)(kRef - 1 - e.r0 - 8 * ee));
      }
      dS.template write_operand<BF>(e, sb + L::SB, ad_0);
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(DS_READY));
      bool ok = true;
      for (int k = 0; k < u.c_end - u.c_begin; ++k, ++gc) {
        const int c = u.c_end - 1 - k;
        const int ph = gc & 1;
        const int t0 = 64 * c, Lc = min(64, a.T - t0);
        // (a) P, (b) dP
        if (!(ok = mbar_wait(bar(QK_FULL), ph, a.status, abort_flag))) break;
        if (e.et == 0) KDA_TRACE_EVENT(18, gc);
        tc_fence_after();
        masked_tile<BF>(e, tmem + e.lane_off + L::A_QK, sb + L::P);
        mbar_arrive(bar(QK_FREE));
        if (!(ok = mbar_wait(bar(DP_FULL), ph, a.status, abort_flag))) break;
        if (e.et == 0) KDA_TRACE_EVENT(19, gc);
        tc_fence_after();
        masked_tile<BF>(e, tmem + e.lane_off + L::A_DP, sb + L::DP);
        mbar_arrive(bar(DP_FREE));
        fence_async_smem();
        if (e.et == 0) tma_store_wait_read<0>();  // the last chunk's dk / dv stores have read their tiles
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          mbar_arrive(bar(P_FULL));
          mbar_arrive(bar(DPM_FULL));
          KDA_TRACE_EVENT(20, gc);
        }
        // (c) dS <- decay^L dS + Q^T dO once the inter MMAs have read dS_c
        if (!(ok = mbar_wait(bar(INTER_FULL), ph, a.status, abort_flag) &&
                   mbar_wait(bar(W_FULL), ph, a.status, abort_flag)))
          break;
        if (e.et == 0) KDA_TRACE_EVENT(21, gc);
        tc_fence_after();
        {
          float al[Carry<D>::NR];
          for (int r = 0; r < Carry<D>::NR; ++r) al[r] = (Lc == 64) ? af[r] : at[r];
          if (D == 128) {
            for (int sl = 0; sl < Carry<D>::NV / 32; ++sl) {
              uint32_t w32[32];
              tmem_ld_32x32b_x32(tmem + e.lane_off + L::A_Z + Carry<D>::W * e.cg + 32 * sl, w32);
              for (int kk = 0; kk < 32; ++kk)
                dS.x[0][32 * sl + kk] = fmaf(al[0], dS.x[0][32 * sl + kk], am * __uint_as_float(w32[kk]));
            }
          } else {
            Carry<D> W;
            W.tmem_load(e, tmem, L::A_Z);
            for (int r = 0; r < Carry<D>::NR; ++r)
              for (int kk = 0; kk < Carry<D>::NV; ++kk) dS.x[r][kk] = fmaf(al[r], dS.x[r][kk], am * W.x[r][kk]);
          }
        }
        tc_fence_before();
        mbar_arrive(bar(W_FREE));
        if (e.et == 0) KDA_TRACE_EVENT(22, gc);
        if (k + 1 < u.c_end - u.c_begin) {
          dS.template write_operand<BF>(e, sb + L::SB, ad_f);
          fence_async_smem();
          named_bar_sync(1, kEpi);
          if (e.et == 0) mbar_arrive(bar(DS_READY));
        }
        if (e.et == 0) KDA_TRACE_EVENT(23, gc);
        // (e) dk, dv -> staging tiles -> TMA stores
        if (!(ok = mbar_wait(bar(DKV_FULL), ph, a.status, abort_flag))) break;
        if (e.et == 0) KDA_TRACE_EVENT(24, gc);
        tc_fence_after();
        if constexpr (TR) {
          tile_from_transposed<BF>(e, tmem, L::A_X, sb + L::DK);
          if (e.et == 0) KDA_TRACE_EVENT(25, gc);
          tile_from_transposed<BF>(e, tmem, L::A_Y, sb + L::DV);
        } else {
          frag_to_tile<D, BF>(e, tmem + e.lane_off + L::A_X, sb + L::DK, 0, false, rk);
          if (e.et == 0) KDA_TRACE_EVENT(25, gc);
          frag_to_tile<D, BF>(e, tmem + e.lane_off + L::A_Y, sb + L::DV, 0, false);
        }
        tc_fence_before();
        mbar_arrive(bar(DKV_FREE));
        fence_async_smem();
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          for (int kb = 0; kb < L::KB; ++kb) {
            tma_store_4d(&tdk, sb + L::DK + kb * kTile, 64 * kb, t0, h, b);
            tma_store_4d(&tdv, sb + L::DV + kb * kTile, 64 * kb, t0, h, b);
          }
          tma_store_commit();
          KDA_TRACE_EVENT(26, gc);
        }
      }
      if (!ok) break;
      if (u.pub_slot >= 0) {
        if (!fold) {
          dS.store_slot(e, slot_ptr(qu, u.pub_slot));
          chain_publish(e, qu, u.pub_slot);
        }
      } else if (a.ds_in) {
        dS.store_rm(e, a.ds_in + sbase);
      }
    }
    if (e.et == 0) tma_store_wait_all();
  } else if constexpr (PS) {
    scaler_role<D, BF, NS>(qu, true, a.H, a.decay, sb, L::STAGE, L::ST_K, warp - kThreads / 32, ring, abort_flag,
                           a.status, sb + L::BAR, KFULL, SCALED, UNIT_FULL0, UNIT_FREE0);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <typename T, int D, bool LIT, bool PS, int NS>
cudaError_t bwd_tc_launch(const BwdArgs &a, const Queue &q1, const Queue &q2, int grid1, int grid2,
                          cudaStream_t st) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mg, mdy, mdq, mdg, mdo, mdk, mdv;
  const View gview = a.g.data ? a.g : a.q;
  const View dgview = a.dg.data ? a.dg : a.dq;
  auto map = [&](CUtensorMap *m, const View &v) { return make_tmap_bhtd(m, v, a.B, a.H, a.T, a.D, BF); };
  const bool ok = map(&mq, a.q) && map(&mk, a.k) && map(&mv, a.v) && map(&mg, gview) && map(&mdy, a.dy) &&
                  map(&mdq, a.dq) && map(&mdg, dgview) && map(&mdo, a.dO) && map(&mdk, a.dk) && map(&mdv, a.dv);
  if (!ok) return cudaErrorInvalidValue;
  using L1 = BwdLayout<D, NS>;
  using L2 = RevLayout<D, NS>;
  auto k1 = bwd_fwddir_tc_kernel<T, D, LIT, PS, NS>;
  auto k2 = bwd_revdir_tc_kernel<T, D, LIT, PS, NS>;
  cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, L1::SMEM);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, L2::SMEM);
  if (e != cudaSuccess) return e;
  const int dtype = BF ? KDA_DTYPE_BF16 : KDA_DTYPE_F16;
  if (q1.agg) {  // long streams: state (and tangent) aggregates from k, v
    const AggArgs g{a.B, a.H, a.T, a.D, a.literal, a.per_step, a.decay, q1.agg, q1.agg_f4, a.status};
    if ((e = launch_agg_tc(PS ? 0 : 1, g, a.k, a.v, q1, dtype, a.s_in, st)) != cudaSuccess) return e;
  }
  int tr = trace_before(st);
  e = launch_kernel(k1, dim3(grid1), dim3(bwd_threads<PS>()), L1::SMEM, st, q1.agg != nullptr, mq, mk, mv, mg, mdy,
                    mdq, mdg, mdo, a, q1);
  trace_after(tr, kTraceBwdFwdDir, st);
  count_launches(1);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (q2.agg) {  // long streams: dS aggregates from q and the dO the first pass wrote
    const AggArgs g{a.B, a.H, a.T, a.D, a.literal, a.per_step, a.decay, q2.agg, q2.agg_f4, a.status};
    if ((e = launch_agg_tc(2, g, a.q, a.dO, q2, dtype, a.ds_out, st)) != cudaSuccess) return e;
  }
  tr = trace_before(st);
  e = launch_kernel(k2, dim3(grid2), dim3(bwd_threads<PS>()), L2::SMEM, st, q2.agg != nullptr, mq, mk, mv, mdo, mdk,
                    mdv, a, q2);
  trace_after(tr, kTraceBwdRevDir, st);
  count_launches(1);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_tc(const BwdArgs &a, const tc::Queue &q1, const tc::Queue &q2, int grid1, int grid2,
                          int dtype, cudaStream_t st) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if (a.per_step) {
    if (a.D == 64)
      return bf ? bwd_tc_launch<__nv_bfloat16, 64, false, true, 2>(a, q1, q2, grid1, grid2, st)
                : bwd_tc_launch<__half, 64, false, true, 2>(a, q1, q2, grid1, grid2, st);
    return bf ? bwd_tc_launch<__nv_bfloat16, 128, false, true, 2>(a, q1, q2, grid1, grid2, st)
              : bwd_tc_launch<__half, 128, false, true, 2>(a, q1, q2, grid1, grid2, st);
  }
  if (a.D == 64) {
    if (a.literal)
      return bf ? bwd_tc_launch<__nv_bfloat16, 64, true, false, 2>(a, q1, q2, grid1, grid2, st)
                : bwd_tc_launch<__half, 64, true, false, 2>(a, q1, q2, grid1, grid2, st);
    return bf ? bwd_tc_launch<__nv_bfloat16, 64, false, false, 2>(a, q1, q2, grid1, grid2, st)
              : bwd_tc_launch<__half, 64, false, false, 2>(a, q1, q2, grid1, grid2, st);
  }
  return bf ? bwd_tc_launch<__nv_bfloat16, 128, false, false, 2>(a, q1, q2, grid1, grid2, st)
            : bwd_tc_launch<__half, 128, false, false, 2>(a, q1, q2, grid1, grid2, st);
}

}  // namespace kda

#ifdef KDA_TRACE
extern "C" int kda_trace_copy_bwd(unsigned long long *host) {
  return (int)cudaMemcpyFromSymbol(host, g_kda_trace, sizeof(g_kda_trace));
}
extern "C" int kda_trace_copy_bwd_cta(unsigned long long *host) {
  return (int)cudaMemcpyFromSymbol(host, g_kda_trace_cta, sizeof(g_kda_trace_cta));
}
#endif
