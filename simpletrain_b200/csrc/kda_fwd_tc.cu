// KDA chunked-scan forward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA owns one (batch, head, 64-wide value tile) and walks all chunks of
// 64 tokens in order, keeping the fp32 state slice S[:, dv0:dv0+64] in the
// epilogue warps' registers.  Per chunk c (kernels/kda_kernel.py:273-295):
//
//   A_c  = Q_c K_c^T                    UMMA M=64  N=64 K=D   -> TMEM
//   O_c  = Q_c S_{c-1}                  UMMA M=64  N=64 K=D   -> TMEM
//   U_c  = K_c^T V_c  (literal: K_c V_c^T)  UMMA M=D N=64 K=64 -> TMEM
//   P_c  = tril(A_c) (bf16, smem)       epilogue
//   O_c += P_c V_c                      UMMA M=64  N=64 K=64  -> TMEM
//   S_c  = decay^L * S_{c-1} + U_c      epilogue (fp32 registers) -> bf16 smem operand
//   y_c  = g_c * O_c                    epilogue -> smem -> TMA store
//
// Warp roles: warp 0 issues TMA loads (q, k, v, g tiles) into an NS-stage ring;
// warp 1 allocates tensor memory and one thread issues every MMA; warps 2-5
// (one per TMEM sub-partition) run the epilogue.  Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "kda_internal.h"
#include "tc_common.cuh"
#include "tmap.h"

namespace kda {
namespace {
using namespace tc;

constexpr int kTile = 64 * 64 * 2;  // one [64 x 64] 16-bit box, 8 KB
constexpr int kThreadsTc = 192;
constexpr uint32_t kAccQK = 0, kAccO = 64, kAccKV = 128, kTmemCols = 256;

template <int D, int NS>
struct FwdLayout {
  static constexpr int KB = D / 64;
  static constexpr int ST_Q = 0;
  static constexpr int ST_K = KB * kTile;
  static constexpr int ST_V = 2 * KB * kTile;
  static constexpr int ST_G = ST_V + kTile;
  static constexpr int STAGE = ST_G + kTile;
  static constexpr int P = NS * STAGE;
  static constexpr int S = P + kTile;  // state operand: D rows (key channel) x 64 value columns
  static constexpr int Y = S + D * 128;
  static constexpr int BAR = Y + kTile;
  // barriers: full[NS], empty[NS], qk_full, qk_empty, kv_full, kv_empty,
  //           o_full, o_empty, p_full, s_full, fin
  static constexpr int NBAR = 2 * NS + 9;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int BYTES = ABORT + 8;
  static constexpr int SMEM = BYTES + 1024;
};

template <typename T, int D, bool LIT, int NS>
__global__ void __launch_bounds__(kThreadsTc, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                  const __grid_constant__ CUtensorMap ty, const FwdArgs a) {
  using L = FwdLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  const int FULL = 0, EMPTY = NS, QK_FULL = 2 * NS, QK_EMPTY = 2 * NS + 1, KV_FULL = 2 * NS + 2,
            KV_EMPTY = 2 * NS + 3, O_FULL = 2 * NS + 4, O_EMPTY = 2 * NS + 5, P_FULL = 2 * NS + 6,
            S_FULL = 2 * NS + 7, FIN = 2 * NS + 8;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int dv0 = blockIdx.y * 64;
  const int nchunks = (a.T + 63) / 64;
  const bool gate = a.g.data != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 2);  // MMA commit + epilogue (done with the gate tile)
    }
    mbar_init(bar(QK_FULL), 1);
    mbar_init(bar(QK_EMPTY), 128);
    mbar_init(bar(KV_FULL), 1);
    mbar_init(bar(KV_EMPTY), 128);
    mbar_init(bar(O_FULL), 1);
    mbar_init(bar(O_EMPTY), 128);
    mbar_init(bar(P_FULL), 1);
    mbar_init(bar(S_FULL), 1);
    mbar_init(bar(FIN), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    if (gate) prefetch_tmap(&tg);
    prefetch_tmap(&ty);
  }
  if (warp == 1) {
    tmem_alloc(sb + L::TMEM_SLOT, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::TMEM_SLOT);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t tx = (uint32_t)((2 * L::KB + 1 + (gate ? 1 : 0)) * kTile);
      int c = 0;
      for (; c < nchunks; ++c) {
        const int s = c % NS, use = c / NS;
        if (!mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag)) break;
        const uint32_t st = sb + s * L::STAGE;
        mbar_arrive_expect_tx(bar(FULL + s), tx);
        const int t0 = c * 64;
        for (int kb = 0; kb < L::KB; ++kb) {
          tma_load_4d(st + L::ST_Q + kb * kTile, &tq, bar(FULL + s), 64 * kb, t0, h, b);
          tma_load_4d(st + L::ST_K + kb * kTile, &tk, bar(FULL + s), 64 * kb, t0, h, b);
        }
        tma_load_4d(st + L::ST_V, &tv, bar(FULL + s), dv0, t0, h, b);
        if (gate) tma_load_4d(st + L::ST_G, &tg, bar(FULL + s), dv0, t0, h, b);
      }
      // drain: every issued load has landed before the CTA can exit
      for (int d = c - 1; d >= 0 && d >= c - NS; --d)
        mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);
      const uint32_t id_qs = idesc_f16(64, 64, BF, false, true);
      const uint32_t id_kv = LIT ? idesc_f16(64, 64, BF, false, false) : idesc_f16(D, 64, BF, true, true);
      const uint32_t id_pv = idesc_f16(64, 64, BF, false, true);
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % NS, use = c / NS;
        const uint32_t st = sb + s * L::STAGE;
        if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(QK_EMPTY), (c & 1) ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + kAccQK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
        }
        mma_commit(bar(QK_FULL));
        if (!mbar_wait(bar(S_FULL), c & 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(O_EMPTY), (c & 1) ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + kAccO, sdesc_k(st + L::ST_Q + off), sdesc_mn(sb + L::S + ks * 2048, kTile), id_qs,
                  ks > 0);
        }
        if (!mbar_wait(bar(KV_EMPTY), (c & 1) ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks) {
          if (LIT)
            mma_f16(tmem + kAccKV, sdesc_k(st + L::ST_K + ks * 32), sdesc_k(st + L::ST_V + ks * 32), id_kv, ks > 0);
          else
            mma_f16(tmem + kAccKV, sdesc_mn(st + L::ST_K + ks * 2048, kTile),
                    sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_kv, ks > 0);
        }
        mma_commit(bar(KV_FULL));
        if (!mbar_wait(bar(P_FULL), c & 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks)
          mma_f16(tmem + kAccO, sdesc_k(sb + L::P + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_pv, 1);
        mma_commit(bar(O_FULL));
        mma_commit(bar(EMPTY + s));
      }
      // every MMA has completed before tensor memory is released
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;          // 0..127
    const int sp = warp & 3;                  // TMEM sub-partition of this warp
    const uint32_t lane_off = (uint32_t)(32 * sp) << 16;
    const int r0 = 16 * sp + (lane >> 2);     // M=64 fragment rows r0, r0 + 8
    const int cq = 2 * (lane & 3);            // M=64 fragment column offset
    const size_t sbase = ((size_t)b * a.H + h) * D * D;
    // state rows owned by this thread
    constexpr int NR = (D == 128) ? 1 : 2;    // rows
    constexpr int NV = (D == 128) ? 64 : 16;  // values per row
    int rows[NR];
    if (D == 128) rows[0] = 32 * sp + lane;
    else { rows[0] = r0; rows[NR - 1] = r0 + 8; }
    auto col_of = [&](int i) {  // value index -> column within the 64-wide tile
      return (D == 128) ? i : (8 * (i >> 1) + cq + (i & 1));
    };
    float S[NR][NV];
    float af[NR], at[NR];
    const int Ltail = a.T - (nchunks - 1) * 64;
    for (int r = 0; r < NR; ++r) {
      af[r] = chunk_alpha(a.decay, b, h, rows[r], 64, 64);
      at[r] = chunk_alpha(a.decay, b, h, rows[r], Ltail, 64);
      for (int i = 0; i < NV; ++i)
        S[r][i] = a.s_in ? a.s_in[sbase + (size_t)rows[r] * D + dv0 + col_of(i)] : 0.f;
    }
    auto write_state = [&]() {
      if (D == 128) {
        const int r = rows[0];
        for (int j = 0; j < 8; ++j)
          st_shared_v4(sb + L::S + swz(r, 8 * j), pack2(S[0][8 * j], S[0][8 * j + 1], BF),
                       pack2(S[0][8 * j + 2], S[0][8 * j + 3], BF), pack2(S[0][8 * j + 4], S[0][8 * j + 5], BF),
                       pack2(S[0][8 * j + 6], S[0][8 * j + 7], BF));
      } else {
        for (int r = 0; r < NR; ++r)
          for (int j = 0; j < 8; ++j)
            st_shared_u32(sb + L::S + swz(rows[r], 8 * j + cq), pack2(S[r][2 * j], S[r][2 * j + 1], BF));
      }
      fence_async_smem();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive(bar(S_FULL));
    };
    write_state();

    for (int c = 0; c < nchunks; ++c) {
      const int s = c % NS, use = c / NS;
      const uint32_t st = sb + s * L::STAGE;
      const int Lc = min(64, a.T - c * 64);
      uint32_t r[32];
      // (a) scores -> masked P
      if (!mbar_wait(bar(QK_FULL), c & 1, a.status, abort_flag)) break;
      tc_fence_after();
      tmem_ld_16x256b_x8(tmem + lane_off + kAccQK, r);
      tc_fence_before();
      mbar_arrive(bar(QK_EMPTY));
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * j + cq;
        const float v00 = col <= r0 ? __uint_as_float(r[4 * j]) : 0.f;
        const float v01 = col + 1 <= r0 ? __uint_as_float(r[4 * j + 1]) : 0.f;
        const float v10 = col <= r0 + 8 ? __uint_as_float(r[4 * j + 2]) : 0.f;
        const float v11 = col + 1 <= r0 + 8 ? __uint_as_float(r[4 * j + 3]) : 0.f;
        st_shared_u32(sb + L::P + swz(r0, col), pack2(v00, v01, BF));
        st_shared_u32(sb + L::P + swz(r0 + 8, col), pack2(v10, v11, BF));
      }
      fence_async_smem();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive(bar(P_FULL));

      // (b) state update S_c = decay^L S_{c-1} + U_c
      if (!mbar_wait(bar(KV_FULL), c & 1, a.status, abort_flag)) break;
      tc_fence_after();
      const bool upd = !(LIT && Lc != 64);
      if (D == 128) {
        uint32_t u0[32], u1[32];
        tmem_ld_32x32b_x32(tmem + lane_off + kAccKV, u0);
        tmem_ld_32x32b_x32(tmem + lane_off + kAccKV + 32, u1);
          tc_fence_before();
        mbar_arrive(bar(KV_EMPTY));
        const float al = (Lc == 64) ? af[0] : at[0];
        for (int i = 0; i < 32; ++i) {
          S[0][i] = fmaf(al, S[0][i], __uint_as_float(u0[i]));
          S[0][32 + i] = fmaf(al, S[0][32 + i], __uint_as_float(u1[i]));
        }
      } else {
        tmem_ld_16x256b_x8(tmem + lane_off + kAccKV, r);
          tc_fence_before();
        mbar_arrive(bar(KV_EMPTY));
        if (upd) {
          for (int rr = 0; rr < NR; ++rr) {
            const float al = (Lc == 64) ? af[rr] : at[rr];
            for (int j = 0; j < 8; ++j) {
              S[rr][2 * j] = fmaf(al, S[rr][2 * j], __uint_as_float(r[4 * j + 2 * rr]));
              S[rr][2 * j + 1] = fmaf(al, S[rr][2 * j + 1], __uint_as_float(r[4 * j + 2 * rr + 1]));
            }
          }
        }
      }
      write_state();

      // (c) output y_c = g_c * O_c
      if (!mbar_wait(bar(O_FULL), c & 1, a.status, abort_flag)) break;
      if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
      tc_fence_after();
      tmem_ld_16x256b_x8(tmem + lane_off + kAccO, r);
      tc_fence_before();
      mbar_arrive(bar(O_EMPTY));
      uint32_t out[16];
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * j + cq;
        float o00 = __uint_as_float(r[4 * j]), o01 = __uint_as_float(r[4 * j + 1]);
        float o10 = __uint_as_float(r[4 * j + 2]), o11 = __uint_as_float(r[4 * j + 3]);
        if (gate) {
          const float2 g0 = unpack2(ld_shared_u32(st + L::ST_G + swz(r0, col)), BF);
          const float2 g1 = unpack2(ld_shared_u32(st + L::ST_G + swz(r0 + 8, col)), BF);
          o00 *= g0.x; o01 *= g0.y; o10 *= g1.x; o11 *= g1.y;
        }
        out[2 * j] = pack2(o00, o01, BF);
        out[2 * j + 1] = pack2(o10, o11, BF);
      }
      if (et == 0) tma_store_wait_read0();   // previous chunk's store has read the staging tile
      named_bar_sync(1, 128);
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * j + cq;
        st_shared_u32(sb + L::Y + swz(r0, col), out[2 * j]);
        st_shared_u32(sb + L::Y + swz(r0 + 8, col), out[2 * j + 1]);
      }
      fence_async_smem();
      named_bar_sync(1, 128);
      if (et == 0) {
        tma_store_4d(&ty, sb + L::Y, dv0, c * 64, h, b);
        tma_store_commit();
        mbar_arrive(bar(EMPTY + s));
      }
    }
    if (a.s_out)
      for (int rr = 0; rr < NR; ++rr)
        for (int i = 0; i < NV; ++i)
          a.s_out[sbase + (size_t)rows[rr] * D + dv0 + col_of(i)] = S[rr][i];
    if (et == 0) tma_store_wait_all();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D, bool LIT, int NS>
cudaError_t fwd_tc_launch(const FwdArgs &a, cudaStream_t st) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mg, my;
  const View gview = a.g.data ? a.g : a.q;
  if (!make_tmap_bhtd(&mq, a.q, a.B, a.H, a.T, a.D, BF) || !make_tmap_bhtd(&mk, a.k, a.B, a.H, a.T, a.D, BF) ||
      !make_tmap_bhtd(&mv, a.v, a.B, a.H, a.T, a.D, BF) || !make_tmap_bhtd(&mg, gview, a.B, a.H, a.T, a.D, BF) ||
      !make_tmap_bhtd(&my, a.y, a.B, a.H, a.T, a.D, BF))
    return cudaErrorInvalidValue;
  using L = FwdLayout<D, NS>;
  auto kern = fwd_tc_kernel<T, D, LIT, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(a.B * a.H, D / 64);
  kern<<<grid, kThreadsTc, L::SMEM, st>>>(mq, mk, mv, mg, my, a);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_tc(const FwdArgs &a, int dtype, cudaStream_t st) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if (a.D == 64) {
    if (a.literal) return bf ? fwd_tc_launch<__nv_bfloat16, 64, true, 2>(a, st) : fwd_tc_launch<__half, 64, true, 2>(a, st);
    return bf ? fwd_tc_launch<__nv_bfloat16, 64, false, 2>(a, st) : fwd_tc_launch<__half, 64, false, 2>(a, st);
  }
  return bf ? fwd_tc_launch<__nv_bfloat16, 128, false, 2>(a, st) : fwd_tc_launch<__half, 128, false, 2>(a, st);
}

}  // namespace kda
