// KDA chunked-scan forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent CTAs take (batch*head stream, segment) units from a work queue
// (kda_tc_epi.cuh) and walk the segment's chunks of 64 tokens, keeping the
// fp32 D x D state in the epilogue warps' registers.  Per chunk c
// (kernels/kda_kernel.py:273-295):
//
//   A_c  = Q_c K_c^T                   UMMA M=64 N=64 K=D  -> TMEM
//   O_c  = Q_c S_{c-1}                 UMMA M=64 N=D  K=D  -> TMEM
//   U_c  = K_c^T V_c (literal K_c V_c^T)  UMMA M=D N=D K=64 -> TMEM
//   P_c  = tril(A_c)                   epilogue -> 16-bit smem operand
//   O_c += P_c V_c                     UMMA M=64 N=D  K=64
//   S_c  = decay^L S_{c-1} + U_c       epilogue registers -> 16-bit smem operand
//   y_c  = g_c * O_c                   epilogue -> global (16-byte stores)
//
// Warp 0 takes range tickets (kda_tc_epi.cuh) and issues TMA loads of q, k, v
// into an NS-stage ring; warp 1 owns tensor memory and one thread issues the
// MMAs; warps 2-9 run the epilogue (two per TMEM sub-partition); lane 1 of
// warp 0 loads g into an NY-deep ring of tiles that the epilogue overwrites in
// place with y = g * O and stores with TMA.  A piece starts from the initial state
// or from the state published at its range boundary, and publishes its own
// when it ends mid-stream.
//
// Per-step decay (PS): two more warps scale each stage's k rows in place
// after the TMA load, K~ = diag(a^(kRef-1-j)) K (kda_tc_epi.cuh); the MMAs
// wait for them, the products are unchanged, and the epilogue applies the
// factors: y = g * a^(i+1-kRef) O, operand a^kRef S, S <- a^L S + a^(L-kRef) K~^T V.
//
// Pipelining: O is double-buffered in tensor memory and the epilogue runs
// "state update of c -> store y_c -> mask P_{c+1}", so the MMAs of chunk c+1
// (Q K^T, Q S_c, K^T V) execute while y_c is gated and stored.  The gate tile
// of chunk c is requested NY-1 chunks ahead, which hides the load latency of
// a saturated memory system without tying up a q/k/v stage.
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

// q/k/v stages and gate-in / y-out tiles per head dimension.  D=64: four stages
// (three chunks of loads in flight; a chunk takes ~1.2 us there, less than the
// loads' latency under load): 100m-shape forward 51.6 -> 49.0 us.  D=128: a third
// stage fits only with two gate tiles, and that measured slower (1b shape 85 -> 95 us).
#ifndef KDA_FWD_NS64
#define KDA_FWD_NS64 4
#endif
#ifndef KDA_FWD_NS128
#define KDA_FWD_NS128 2
#endif
#ifndef KDA_FWD_NY128
#define KDA_FWD_NY128 4
#endif
template <int D>
constexpr int fwd_ns() { return D == 64 ? KDA_FWD_NS64 : KDA_FWD_NS128; }
template <int D>
constexpr int fwd_ny() { return D == 64 ? 4 : KDA_FWD_NY128; }
constexpr int kFwdThreads = kThreads;

template <int D, int NS, int NY>
struct FwdLayout {
  static constexpr int KB = D / 64;
  static constexpr int BOX = KB * kTile;
  static constexpr int ST_Q = 0, ST_K = BOX, ST_V = 2 * BOX, STAGE = 3 * BOX;
  static constexpr int P = NS * STAGE;
  static constexpr int SB = P + kTile;  // S_{c-1}: KB panels of [D rows x 64]
  static constexpr int Y = SB + KB * D * 128;  // NY tiles (BOX each): g in, y out
  static constexpr int BAR = Y + NY * BOX;
  static constexpr int NBAR = 4 * NS + 2 * NY + 16;
  static constexpr int RING = BAR + NBAR * 8;  // two (ticket, piece) entries
  static constexpr int TMEM_SLOT = RING + 16;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int SMEM = ABORT + 8 + 1024;
  static constexpr uint32_t A_QK = 0, A_O0 = 64, A_O1 = 64 + D, A_KV = 64 + 2 * D;
  static constexpr uint32_t TMEM_COLS = (64 + 3 * D) <= 256 ? 256 : 512;
};

// threads of a forward CTA: + two row-scaler warps in per-step mode
template <bool PS>
constexpr int fwd_threads() { return kFwdThreads + (PS ? 64 : 0); }

template <typename T, int D, bool LIT, bool PS, int NS, int NY>
__global__ void __launch_bounds__(fwd_threads<PS>(), 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                  const __grid_constant__ CUtensorMap ty, const FwdArgs a, const Queue qu) {
  using L = FwdLayout<D, NS, NY>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr int KB = L::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  enum {
    QK_FULL = 2 * NS + 2 * NY, QK_FREE, S_READY, O_FREE0, O_FREE1, KV_FREE, KV_FULL, P_FULL, O_FULL, UNIT_FULL0,
    UNIT_FULL1, UNIT_FREE0, UNIT_FREE1, FIN, SCALED, KFULL = SCALED + NS
  };
  const int FULL = 0, EMPTY = NS, GFULL = 2 * NS, GEMPTY = 2 * NS + NY;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  volatile int *ring = reinterpret_cast<volatile int *>(smem + L::RING);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool gate = a.g.data != nullptr;

  if (threadIdx.x == 0) {
    KDA_TRACE_CTA(0, kda_globaltimer());
    KDA_TRACE_CTA(7, kda_smid());
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 1);  // MMA commit
    }
    for (int j = 0; j < NY; ++j) {
      mbar_init(bar(GFULL + j), 1);
      mbar_init(bar(GEMPTY + j), 1);  // the y store from the tile has read it
    }
    mbar_init(bar(QK_FULL + 0), 1);
    mbar_init(bar(QK_FULL + 1), kEpi);
    mbar_init(bar(QK_FULL + 2), 1);
    mbar_init(bar(QK_FULL + 3), kEpi);
    mbar_init(bar(QK_FULL + 4), kEpi);
    mbar_init(bar(QK_FULL + 5), kEpi);
    mbar_init(bar(QK_FULL + 6), 1);
    mbar_init(bar(QK_FULL + 7), 1);
    mbar_init(bar(QK_FULL + 8), 1);
    mbar_init(bar(QK_FULL + 9), 1);
    mbar_init(bar(QK_FULL + 10), 1);
    mbar_init(bar(QK_FULL + 11), 2 + kEpi + (PS ? 2 : 0));  // unit ring slots: MMA, gate loader, epilogue, scalers
    mbar_init(bar(QK_FULL + 12), 2 + kEpi + (PS ? 2 : 0));
    mbar_init(bar(QK_FULL + 13), 1);
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
    // ----------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&ty);
      const uint32_t tx = (uint32_t)((PS ? 2 : 3) * L::BOX);
      int gc = 0, i = 0;
      bool ok = true;
      while (ok) {
        const int t = atomicAdd(qu.ticket, 1);
        const Span sp = t < qu.nranges ? span_of(qu, t, false) : Span{};
        const int m = t < qu.nranges ? sp.npieces() : 1;
        for (int p = 0; p < m && ok; ++p, ++i) {
          if (!(ok = mbar_wait(bar(UNIT_FREE0 + (i & 1)), ((i >> 1) & 1) ^ 1, a.status, abort_flag))) break;
          ring[2 * (i & 1)] = t;
          ring[2 * (i & 1) + 1] = p;
          mbar_arrive(bar(UNIT_FULL0 + (i & 1)));
          if (t >= qu.nranges) { ok = false; break; }
          const Piece u = piece_of(qu, sp, p, false);
          const int b = u.stream / a.H, h = u.stream - b * a.H;
          for (int c = u.c_begin; c < u.c_end; ++c, ++gc) {
            const int s = gc % NS, use = gc / NS;
            if (!(ok = mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag))) break;
            KDA_TRACE_EVENT(0, gc);
            const uint32_t st = sb + s * L::STAGE;
            if (PS) {  // k first, on its own barrier: its row scaling overlaps the q and v loads
              mbar_arrive_expect_tx(bar(KFULL + s), (uint32_t)L::BOX);
              for (int kb = 0; kb < KB; ++kb)
                tma_load_4d(st + L::ST_K + kb * kTile, &tk, bar(KFULL + s), 64 * kb, 64 * c, h, b);
            }
            mbar_arrive_expect_tx(bar(FULL + s), tx);
            for (int kb = 0; kb < KB; ++kb) {
              tma_load_4d(st + L::ST_Q + kb * kTile, &tq, bar(FULL + s), 64 * kb, 64 * c, h, b);
              if (!PS) tma_load_4d(st + L::ST_K + kb * kTile, &tk, bar(FULL + s), 64 * kb, 64 * c, h, b);
              tma_load_4d(st + L::ST_V + kb * kTile, &tv, bar(FULL + s), 64 * kb, 64 * c, h, b);
            }
            KDA_TRACE_EVENT(1, gc);
          }
        }
      }
      for (int d = gc - 1; d >= 0 && d >= gc - NS; --d) {
        mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
        if (PS) mbar_wait(bar(KFULL + d % NS), (d / NS) & 1, a.status, abort_flag);
      }
    } else if (lane == 1) {
      // ------------------------------------------------------- gate loader
      if (gate) prefetch_tmap(&tg);
      int gc = 0;
      for (int i = 0;; ++i) {
        if (!mbar_wait(bar(UNIT_FULL0 + (i & 1)), (i >> 1) & 1, a.status, abort_flag)) break;
        const int t = ring[2 * (i & 1)], p = ring[2 * (i & 1) + 1];
        mbar_arrive(bar(UNIT_FREE0 + (i & 1)));
        if (t >= qu.nranges) break;
        const Piece u = piece_of(qu, span_of(qu, t, false), p, false);
        if (!gate) continue;
        const int b = u.stream / a.H, h = u.stream - b * a.H;
        bool ok = true;
        for (int c = u.c_begin; c < u.c_end; ++c, ++gc) {
          const int j = gc % NY, use = gc / NY;
          if (!(ok = mbar_wait(bar(GEMPTY + j), (use & 1) ^ 1, a.status, abort_flag))) break;
          const uint32_t yt = sb + L::Y + j * L::BOX;
          mbar_arrive_expect_tx(bar(GFULL + j), (uint32_t)L::BOX);
          for (int kb = 0; kb < KB; ++kb) tma_load_4d(yt + kb * kTile, &tg, bar(GFULL + j), 64 * kb, 64 * c, h, b);
        }
        if (!ok) break;
      }
      for (int d = gc - 1; d >= 0 && d >= gc - NY; --d)
        mbar_wait(bar(GFULL + d % NY), (d / NY) & 1, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);
      const uint32_t id_qs = idesc_f16(64, D, BF, false, true);
      const uint32_t id_kv = LIT ? idesc_f16(64, 64, BF, false, false) : idesc_f16(D, D, BF, true, true);
      const uint32_t id_pv = idesc_f16(64, D, BF, false, true);
      int gc = 0;
      for (int i = 0;; ++i) {
        if (!mbar_wait(bar(UNIT_FULL0 + (i & 1)), (i >> 1) & 1, a.status, abort_flag)) break;
        const int t = ring[2 * (i & 1)], p = ring[2 * (i & 1) + 1];
        mbar_arrive(bar(UNIT_FREE0 + (i & 1)));
        if (t >= qu.nranges) break;
        const Piece u = piece_of(qu, span_of(qu, t, false), p, false);
        bool ok = true;
        for (int c = u.c_begin; c < u.c_end && ok; ++c, ++gc) {
          const int s = gc % NS, use = gc / NS, ph = gc & 1;
          const uint32_t st = sb + s * L::STAGE;
          ok = mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag) &&
               (!PS || mbar_wait(bar(SCALED + s), use & 1, a.status, abort_flag));
          KDA_TRACE_EVENT(2, gc);
          ok = ok && mbar_wait(bar(QK_FREE), ph ^ 1, a.status, abort_flag);
          if (!ok) break;
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + L::A_QK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
          }
          mma_commit(bar(QK_FULL));
          const int ob = gc & 1;
          const uint32_t acc_o = ob ? L::A_O1 : L::A_O0;
          ok = mbar_wait(bar(S_READY), ph, a.status, abort_flag);
          KDA_TRACE_EVENT(3, gc);
          ok = ok && mbar_wait(bar(O_FREE0 + ob), ((gc >> 1) & 1) ^ 1, a.status, abort_flag);
          KDA_TRACE_EVENT(4, gc);
          if (!ok) break;
          tc_fence_after();
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            mma_f16(tmem + acc_o, sdesc_k(st + L::ST_Q + off), sdesc_mn(sb + L::SB + ks * 2048, D * 128), id_qs,
                    ks > 0);
          }
          if (!(ok = mbar_wait(bar(KV_FREE), ph ^ 1, a.status, abort_flag))) break;
          KDA_TRACE_EVENT(5, gc);
          tc_fence_after();
          for (int ks = 0; ks < 4; ++ks) {
            if (LIT)
              mma_f16(tmem + L::A_KV, sdesc_k(st + L::ST_K + ks * 32), sdesc_k(st + L::ST_V + ks * 32), id_kv,
                      ks > 0);
            else
              mma_f16(tmem + L::A_KV, sdesc_mn(st + L::ST_K + ks * 2048, kTile),
                      sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_kv, ks > 0);
          }
          mma_commit(bar(KV_FULL));
          if (!(ok = mbar_wait(bar(P_FULL), ph, a.status, abort_flag))) break;
          KDA_TRACE_EVENT(6, gc);
          tc_fence_after();
          for (int ks = 0; ks < 4; ++ks)
            mma_f16(tmem + acc_o, sdesc_k(sb + L::P + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_pv,
                    1);
          mma_commit(bar(O_FULL));
          mma_commit(bar(EMPTY + s));
        }
        if (!ok) break;
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp < kFwdThreads / 32) {
    // ----------------------------------------------------------- epilogue
    const Epi e;
    pdl_wait();  // long streams: the entry carries come from entry_fold_kernel, launched just before
    Carry<D> S;
    S.init_rows(e);
    int gc = 0;
    for (int i = 0;; ++i) {
      if (!mbar_wait(bar(UNIT_FULL0 + (i & 1)), (i >> 1) & 1, a.status, abort_flag)) break;
      const int t = ring[2 * (i & 1)], p = ring[2 * (i & 1) + 1];
      mbar_arrive(bar(UNIT_FREE0 + (i & 1)));
      if (t >= qu.nranges) break;
      const Piece u = piece_of(qu, span_of(qu, t, false), p, false);
      const int b = u.stream / a.H, h = u.stream - b * a.H;
      const size_t sbase = (size_t)u.stream * D * D;
      // this thread's chunk decays: loaded before the boundary wait below (their round
      // trip overlaps it), raised to the chunk lengths after it
      float af[Carry<D>::NR], at[Carry<D>::NR];
      const int Ltail = a.T - (qu.nchunks - 1) * 64;
      for (int r = 0; r < Carry<D>::NR; ++r) af[r] = decay_value(a.decay, b, h, S.row[r]);
      // piece-start state: the initial state, or the one at the range boundary
      // (long streams: folded there before this kernel started; no wait)
      const bool fold = u.folds(qu);
      if (e.et == 0) KDA_TRACE_EVENT(15, gc);
      if (!fold && !chain_wait(e, qu, u.wait_slot, a.status, abort_flag)) break;
      if (e.et == 0) KDA_TRACE_EVENT(16, gc);
      for (int r = 0; r < Carry<D>::NR; ++r) {
        const float dv = af[r];
        af[r] = chunk_alpha_of(a.decay, dv, 64, 64);
        at[r] = chunk_alpha_of(a.decay, dv, Ltail, 64);
      }
      if (e.et == 0 && i == 0) {
        KDA_TRACE_CTA(4, kda_globaltimer());
        KDA_TRACE_CTA(6, t);
      }
      if (u.wait_slot < 0) S.load_rm(e, a.s_in ? a.s_in + sbase : nullptr);
      else S.load_slot(e, slot_ptr(qu, u.wait_slot));
      // per-step: operand a^kRef S, U factor a^(L-kRef) (full / tail chunk),
      // y row factors a^(row+1-kRef) for rows r0 and r0 + 8
      float am = 1.f, au_f = 1.f, au_t = 1.f, rq[2] = {1.f, 1.f};
      if constexpr (PS) {
        const float l2a = log2f(decay_value(a.decay, b, h, 0));
        am = pow_log2(l2a, (float)kRef);
        au_f = pow_log2(l2a, (float)(64 - kRef));
        au_t = pow_log2(l2a, (float)(Ltail - kRef));
        for (int ee = 0; ee < 2; ++ee) rq[ee] = pow_log2(l2a, (float)(e.r0 + 8 * ee + 1 - kRef));
      }
      if (e.et == 0 && i == 0) KDA_TRACE_CTA(5, kda_globaltimer());
      S.template write_operand<BF>(e, sb + L::SB, am);
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) {
        mbar_arrive(bar(S_READY));
        if (i == 0) KDA_TRACE_CTA(1, kda_globaltimer());
      }
      // masked scores -> P for chunk gc (its Q K^T was issued ahead)
      auto make_p = [&](int g) -> bool {
        if (e.et == 0) KDA_TRACE_EVENT(12, g);
        if (!mbar_wait(bar(QK_FULL), g & 1, a.status, abort_flag)) return false;
        if (e.et == 0) KDA_TRACE_EVENT(13, g);
        tc_fence_after();
        masked_tile<BF>(e, tmem + e.lane_off + L::A_QK, sb + L::P);
        mbar_arrive(bar(QK_FREE));
        fence_async_smem();
        named_bar_sync(1, kEpi);
        if (e.et == 0) {
          mbar_arrive(bar(P_FULL));
          KDA_TRACE_EVENT(14, g);
        }
        return true;
      };
      bool ok = make_p(gc);
      for (int c = u.c_begin; c < u.c_end && ok; ++c, ++gc) {
        const int ph = gc & 1, ob = gc & 1;
        const int t0 = 64 * c, Lc = min(64, a.T - t0);
        const bool last = c + 1 == u.c_end;
        // (b) S_c = decay^L S_{c-1} + U_c  (U_c's MMA follows Q S_{c-1}, so the operand is free)
        if (!(ok = mbar_wait(bar(KV_FULL), ph, a.status, abort_flag))) break;
        if (e.et == 0) KDA_TRACE_EVENT(8, gc);
        tc_fence_after();
        {
          const bool upd = !(LIT && Lc != 64);
          const float au = PS ? ((Lc == 64) ? au_f : au_t) : 1.f;
          if (D == 128) {
            const float al = (Lc == 64) ? af[0] : at[0];
            for (int sl = 0; sl < Carry<D>::NV / 32; ++sl) {
              uint32_t uu[32];
              tmem_ld_32x32b_x32(tmem + e.lane_off + L::A_KV + Carry<D>::W * e.cg + 32 * sl, uu);
              if (upd)
                for (int k = 0; k < 32; ++k)
                  S.x[0][32 * sl + k] = fmaf(al, S.x[0][32 * sl + k], au * __uint_as_float(uu[k]));
            }
          } else {
            Carry<D> U;
            U.tmem_load(e, tmem, L::A_KV);
            if (upd)
              for (int r = 0; r < Carry<D>::NR; ++r) {
                const float al = (Lc == 64) ? af[r] : at[r];
                for (int k = 0; k < Carry<D>::NV; ++k) S.x[r][k] = fmaf(al, S.x[r][k], au * U.x[r][k]);
              }
          }
          tc_fence_before();
          mbar_arrive(bar(KV_FREE));
          if (e.et == 0) KDA_TRACE_EVENT(17, gc);
        }
        if (!last) {
          S.template write_operand<BF>(e, sb + L::SB, am);
          if (e.et == 0) KDA_TRACE_EVENT(18, gc);
          fence_async_smem();
          if (e.et == 0) KDA_TRACE_EVENT(19, gc);
          named_bar_sync(1, kEpi);
          if (e.et == 0) {
            mbar_arrive(bar(S_READY));
            KDA_TRACE_EVENT(9, gc);
          }
        } else if (u.pub_slot >= 0) {
          if (!fold) {
            // hand the state across the range boundary before storing the last y
            S.store_slot(e, slot_ptr(qu, u.pub_slot));
            chain_publish(e, qu, u.pub_slot);
          }
        } else if (a.s_out) {
          S.store_rm(e, a.s_out + sbase);
        }
        // (c) y_c = g_c * O_c  -> staging tile -> TMA store
        if (e.et == 0) KDA_TRACE_EVENT(7, gc);
        const int j = gc % NY;
        const uint32_t yt = sb + L::Y + j * L::BOX;
        if (gate && !(ok = mbar_wait(bar(GFULL + j), (gc / NY) & 1, a.status, abort_flag))) break;
        if (!(ok = mbar_wait(bar(O_FULL), ph, a.status, abort_flag))) break;
        if (e.et == 0) KDA_TRACE_EVENT(10, gc);
        tc_fence_after();
        {
          constexpr int W = D / kQ;
          Frag<W> fo;
          ld_frag(tmem + e.lane_off + (ob ? L::A_O1 : L::A_O0) + W * e.cg, fo);
          tc_fence_before();
          mbar_arrive(bar(O_FREE0 + ob));
          if (e.et == 0) KDA_TRACE_EVENT(20, gc);
          if (!gate) {
            // no gate tile was loaded: wait until the store that last used tile j has read it
            if (e.et == 0) tma_store_wait_read<NY - 1>();
            named_bar_sync(1, kEpi);
          }
          if (e.et == 0) KDA_TRACE_EVENT(21, gc);
          uint32_t gv[W / 4];  // all gate loads first: the shared-memory accesses are ordered asm
          if (gate)
            for (int jj = 0; jj < W / 8; ++jj)
              for (int ee = 0; ee < 2; ++ee)
                gv[2 * jj + ee] = ld_shared_u32(box_addr(yt, e.r0 + 8 * ee, W * e.cg + 8 * jj + e.cq));
          for (int jj = 0; jj < W / 8; ++jj)
            for (int ee = 0; ee < 2; ++ee) {
              float o0 = fo.v(ee, jj, 0), o1 = fo.v(ee, jj, 1);
              if constexpr (PS) {
                o0 *= rq[ee];
                o1 *= rq[ee];
              }
              if (gate) {
                const float2 g2 = unpack2(gv[2 * jj + ee], BF);
                o0 *= g2.x;
                o1 *= g2.y;
              }
              // y over g, element by element
              st_shared_u32(box_addr(yt, e.r0 + 8 * ee, W * e.cg + 8 * jj + e.cq), pack2(o0, o1, BF));
            }
          if (e.et == 0) KDA_TRACE_EVENT(22, gc);
          fence_async_smem();
          if (e.et == 0) KDA_TRACE_EVENT(23, gc);
          named_bar_sync(1, kEpi);
          if (e.et == 0) KDA_TRACE_EVENT(24, gc);
          if (e.et == 0) {
            for (int kb = 0; kb < KB; ++kb) tma_store_4d(&ty, yt + kb * kTile, 64 * kb, t0, h, b);
            tma_store_commit();
            if (gate && gc > 0) {
              // the previous chunk's store has read its tile: hand it back to the gate loader
              tma_store_wait_read<1>();
              mbar_arrive(bar(GEMPTY + (gc - 1) % NY));
            }
            KDA_TRACE_EVENT(11, gc);
          }
        }
        // (a) P for the next chunk of the piece
        if (!last) ok = make_p(gc + 1);
      }
      if (!ok) break;
    }
    if (e.et == 0) {
      tma_store_wait_all();
      KDA_TRACE_CTA(2, kda_globaltimer());
      KDA_TRACE_CTA(3, gc);
    }
  } else if constexpr (PS) {
    // ------------------------------------------------------- row scalers
    scaler_role<D, BF, NS>(qu, false, a.H, a.decay, sb, L::STAGE, L::ST_K, warp - kFwdThreads / 32, ring,
                           abort_flag, a.status, sb + L::BAR, KFULL, SCALED, UNIT_FULL0, UNIT_FREE0);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

template <typename T, int D, bool LIT, bool PS, int NS = fwd_ns<D>(), int NY = fwd_ny<D>()>
cudaError_t fwd_tc_launch(const FwdArgs &a, const Queue &q, int grid, cudaStream_t st) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mg, my;
  const View gview = a.g.data ? a.g : a.q;
  if (!make_tmap_bhtd(&mq, a.q, a.B, a.H, a.T, a.D, BF) || !make_tmap_bhtd(&mk, a.k, a.B, a.H, a.T, a.D, BF) ||
      !make_tmap_bhtd(&mv, a.v, a.B, a.H, a.T, a.D, BF) || !make_tmap_bhtd(&mg, gview, a.B, a.H, a.T, a.D, BF) ||
      !make_tmap_bhtd(&my, a.y, a.B, a.H, a.T, a.D, BF))
    return cudaErrorInvalidValue;
  using L = FwdLayout<D, NS, NY>;
  auto kern = fwd_tc_kernel<T, D, LIT, PS, NS, NY>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return e;
  if (q.agg) {  // long streams: the state aggregates and the range-boundary states first
    const AggArgs g{a.B, a.H, a.T, a.D, a.literal, a.per_step, a.decay, q.agg, q.agg_f4, a.status};
    e = launch_agg_tc(0, g, a.k, a.v, q, BF ? KDA_DTYPE_BF16 : KDA_DTYPE_F16, a.s_in, st);
    if (e != cudaSuccess) return e;
  }
  const int tr = trace_before(st);
  e = launch_kernel(kern, dim3(grid), dim3(fwd_threads<PS>()), L::SMEM, st, q.agg != nullptr, mq, mk, mv, mg, my, a,
                    q);
  trace_after(tr, kTraceFwd, st);
  count_launches(1);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename T, int D, bool LIT, bool PS, int NS = fwd_ns<D>(), int NY = fwd_ny<D>()>
int fwd_ctas_per_sm() {
  auto kern = fwd_tc_kernel<T, D, LIT, PS, NS, NY>;
  int n = 0;
  // the dynamic shared memory must be allowed before the occupancy query counts it
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<D, NS, NY>::SMEM) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, fwd_threads<PS>(), FwdLayout<D, NS, NY>::SMEM) !=
          cudaSuccess)
    return 1;
  // tensor memory is not in the occupancy model: a CTA holds TMEM_COLS of the SM's 512 columns
  const int tmem_cap = 512 / (int)FwdLayout<D, NS, NY>::TMEM_COLS;
  n = n < tmem_cap ? n : tmem_cap;
  return n > 0 ? n : 1;
}

}  // namespace

// Stage and gate-tile counts of the per-step kernels.
constexpr int kPsNS = 2, kPsNY = 4;

int fwd_tc_occupancy(int D, int dtype, bool literal, bool per_step) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if (per_step) {
    if (D == 64)
      return bf ? fwd_ctas_per_sm<__nv_bfloat16, 64, false, true>() : fwd_ctas_per_sm<__half, 64, false, true>();
    return bf ? fwd_ctas_per_sm<__nv_bfloat16, 128, false, true, kPsNS, kPsNY>()
              : fwd_ctas_per_sm<__half, 128, false, true, kPsNS, kPsNY>();
  }
  if (D == 64) {
    if (literal) return bf ? fwd_ctas_per_sm<__nv_bfloat16, 64, true, false>() : fwd_ctas_per_sm<__half, 64, true, false>();
    return bf ? fwd_ctas_per_sm<__nv_bfloat16, 64, false, false>() : fwd_ctas_per_sm<__half, 64, false, false>();
  }
  return bf ? fwd_ctas_per_sm<__nv_bfloat16, 128, false, false>() : fwd_ctas_per_sm<__half, 128, false, false>();
}

cudaError_t launch_fwd_tc(const FwdArgs &a, const tc::Queue &q, int grid, int dtype, cudaStream_t st) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if (a.per_step) {
    if (a.D == 64)
      return bf ? fwd_tc_launch<__nv_bfloat16, 64, false, true>(a, q, grid, st)
                : fwd_tc_launch<__half, 64, false, true>(a, q, grid, st);
    return bf ? fwd_tc_launch<__nv_bfloat16, 128, false, true, kPsNS, kPsNY>(a, q, grid, st)
              : fwd_tc_launch<__half, 128, false, true, kPsNS, kPsNY>(a, q, grid, st);
  }
  if (a.D == 64) {
    if (a.literal)
      return bf ? fwd_tc_launch<__nv_bfloat16, 64, true, false>(a, q, grid, st)
                : fwd_tc_launch<__half, 64, true, false>(a, q, grid, st);
    return bf ? fwd_tc_launch<__nv_bfloat16, 64, false, false>(a, q, grid, st)
              : fwd_tc_launch<__half, 64, false, false>(a, q, grid, st);
  }
  return bf ? fwd_tc_launch<__nv_bfloat16, 128, false, false>(a, q, grid, st)
            : fwd_tc_launch<__half, 128, false, false>(a, q, grid, st);
}

}  // namespace kda

#ifdef KDA_TRACE
extern "C" int kda_trace_copy_fwd(unsigned long long *host) {
  return (int)cudaMemcpyFromSymbol(host, g_kda_trace, sizeof(g_kda_trace));
}
extern "C" int kda_trace_copy_fwd_cta(unsigned long long *host) {
  return (int)cudaMemcpyFromSymbol(host, g_kda_trace_cta, sizeof(g_kda_trace_cta));
}
#endif
