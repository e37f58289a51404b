// KDA chunked-scan backward on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Two kernels, one CTA per (batch, head), each walking the chunks of 64 tokens
// with a fp32 D x D carry.  Gradients of the chunk loop in
// kernels/kda_kernel.py:269-296 (autograd there), with dO = dy * g,
// P = tril(Q K^T), dP = tril(dO V^T):
//
// forward direction (carry S_{c-1}, recomputed, never stored; it lives in
// tensor memory and the K^T V product accumulates into it):
//   O = P V + Q S              -> dg = dy * O
//   dq = dP K + dO S^T
//   S <- decay^L S + K^T V     (literal: K V^T)
//   decay gradient in forward mode: the tangent T = dS/dlog(decay) (row-wise)
//   obeys T <- decay^L (T + L S); dL/dlog decay[i] = sum_t q_t[i] (dO_t T^T)[i]
//   + <dS_T[i,:], T_T[i,:]>.  T is carried in registers, dO T^T is one more MMA.
// reverse direction (carry dS_c = dL/dS_c in registers):
//   dk = dP^T Q + V dS^T       (literal: dS V)
//   dv = P^T dO + K dS         (literal: dS^T K)
//   dS <- decay^L dS + Q^T dO
//
// Warp roles: warp 0 TMA producer, warp 1 tensor-memory owner and single MMA
// issuer, warps 2-9 epilogue (two warps per TMEM sub-partition, splitting the
// columns).  Every wait is bounded.
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

constexpr int kTile = 64 * 64 * 2;
constexpr int kBwdThreads = 320;
constexpr int kEpi = 256;
constexpr uint32_t kTmemCols = 512;

template <int D, int NS>
struct BwdLayout {
  static constexpr int KB = D / 64;
  static constexpr int BOX = KB * kTile;  // one [64 tokens x D] tile
  static constexpr int ST_Q = 0, ST_K = BOX, ST_V = 2 * BOX, ST_G = 3 * BOX, ST_DY = 4 * BOX;
  static constexpr int STAGE = 5 * BOX;
  static constexpr int P = NS * STAGE;
  static constexpr int DP = P + kTile;
  static constexpr int DO = DP + kTile;
  static constexpr int PANEL = D * 128;     // [D rows x 64 columns] of the carried state
  static constexpr int SB = DO + BOX;
  static constexpr int TB = SB + KB * PANEL;  // decay tangent operand (forward-direction pass)
  static constexpr int O1 = TB + KB * PANEL;
  static constexpr int O2 = O1 + BOX;
  static constexpr int RED = O2 + BOX;      // float [2][4][D]
  static constexpr int BAR = RED + 2 * 4 * D * 4;
  static constexpr int NBAR = 2 * NS + 24;
  static constexpr int TMEM_SLOT = BAR + NBAR * 8;
  static constexpr int ABORT = TMEM_SLOT + 8;
  static constexpr int SMEM = ABORT + 8 + 1024;
  // tensor-memory columns
  static constexpr uint32_t A_QK = 0, A_DP = 64, A_X = 128, A_Y = 128 + D, A_Z = 128 + 2 * D;
};

// M=64 accumulator fragment of W columns per thread group: thread holds rows
// r0 and r0+8, columns col0 + 8j + cq + {0,1}, value (e, j, k) at r[4j+2e+k].
template <int W>
struct Frag {
  uint32_t r[W / 2];
  __device__ __forceinline__ float v(int e, int j, int k) const { return __uint_as_float(r[4 * j + 2 * e + k]); }
};
__device__ __forceinline__ void ld_frag(uint32_t taddr, Frag<32> &f) { tmem_ld_16x256b_x4(taddr, f.r); }
__device__ __forceinline__ void ld_frag(uint32_t taddr, Frag<64> &f) { tmem_ld_16x256b_x8(taddr, f.r); }

// address of element (row, col) of a [64 rows x (64*KB) cols] tile stored as KB boxes
__device__ __forceinline__ uint32_t box_addr(uint32_t base, int row, int col) {
  return base + (uint32_t)((col >> 6) * kTile) + swz(row, col & 63);
}
// address of element (row, col) of a KB-panel [D rows x 64] state operand
template <int D>
__device__ __forceinline__ uint32_t panel_addr(uint32_t base, int row, int col) {
  return base + (uint32_t)((col >> 6) * D * 128) + swz(row, col & 63);
}

// Epilogue thread geometry.
struct Epi {
  int et, lane, sp, half, r0, cq;
  uint32_t lane_off;
  __device__ Epi() {
    et = threadIdx.x - 64;
    lane = threadIdx.x & 31;
    sp = (threadIdx.x >> 5) & 3;
    half = et >> 7;
    r0 = 16 * sp + (lane >> 2);
    cq = 2 * (lane & 3);
    lane_off = (uint32_t)(32 * sp) << 16;
  }
};

// fp32 carry (S or dS) owned by one epilogue thread.
//   D=128 (M=128 accumulators): row 32*sp + lane, columns 64*half + [0, 64)
//   D=64  (M=64 accumulators) : rows r0, r0+8, columns 32*half + 8j + cq + k (j < 4)
template <int D>
struct Carry {
  static constexpr int NR = (D == 128) ? 1 : 2;
  static constexpr int NV = (D == 128) ? 64 : 8;
  float x[NR][NV];
  int row[NR];
  __device__ __forceinline__ int col(const Epi &e, int i) const {
    return (D == 128) ? 64 * e.half + i : 32 * e.half + 8 * (i >> 1) + e.cq + (i & 1);
  }
  __device__ void init(const Epi &e) {
    if (D == 128) row[0] = 32 * e.sp + e.lane;
    else { row[0] = e.r0; row[NR - 1] = e.r0 + 8; }
  }
  __device__ void load(const Epi &e, const float *src) {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) x[r][i] = src ? src[(size_t)row[r] * D + col(e, i)] : 0.f;
  }
  __device__ void store(const Epi &e, float *dst) const {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) dst[(size_t)row[r] * D + col(e, i)] = x[r][i];
  }
  // x = alpha[row] * x + acc (accumulator of M = D rows at tensor-memory column base)
  __device__ void update(const Epi &e, uint32_t tmem, uint32_t acc, const float (&al)[NR]) {
    Carry<D> t;
    t.tmem_load(e, tmem, acc);
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) x[r][i] = fmaf(al[r], x[r][i], t.x[r][i]);
  }
  // read / write the carry layout from / to tensor memory (M = D accumulator)
  __device__ void tmem_load(const Epi &e, uint32_t tmem, uint32_t acc) {
    if (D == 128) {
      uint32_t u0[32], u1[32];
      tmem_ld_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half, u0);
      tmem_ld_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half + 32, u1);
      for (int i = 0; i < 32; ++i) {
        x[0][i] = __uint_as_float(u0[i]);
        x[0][32 + i] = __uint_as_float(u1[i]);
      }
    } else {
      Frag<32> f;
      ld_frag(tmem + e.lane_off + acc + 32 * e.half, f);
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < 4; ++j)
          for (int k = 0; k < 2; ++k) x[r][2 * j + k] = f.v(r, j, k);
    }
  }
  __device__ void tmem_store(const Epi &e, uint32_t tmem, uint32_t acc) const {
    if (D == 128) {
      uint32_t u[32];
      for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(x[0][i]);
      tmem_st_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half, u);
      for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(x[0][32 + i]);
      tmem_st_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half + 32, u);
    } else {
      uint32_t u[16];
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < 4; ++j)
          for (int k = 0; k < 2; ++k) u[4 * j + 2 * r + k] = __float_as_uint(x[r][2 * j + k]);
      tmem_st_16x256b_x4(tmem + e.lane_off + acc + 32 * e.half, u);
    }
  }
  // bf16/fp16 copy into the state operand (KB panels of [D rows x 64])
  template <bool BF>
  __device__ void write(const Epi &e, uint32_t base) const {
    if (D == 128) {
      const int rr = row[0];
      const uint32_t pb = base + (uint32_t)(e.half * D * 128);
      for (int j = 0; j < 8; ++j)
        st_shared_v4(pb + swz(rr, 8 * j), pack2(x[0][8 * j], x[0][8 * j + 1], BF),
                     pack2(x[0][8 * j + 2], x[0][8 * j + 3], BF), pack2(x[0][8 * j + 4], x[0][8 * j + 5], BF),
                     pack2(x[0][8 * j + 6], x[0][8 * j + 7], BF));
    } else {
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < 4; ++j)
          st_shared_u32(panel_addr<D>(base, row[r], 32 * e.half + 8 * j + e.cq),
                        pack2(x[r][2 * j], x[r][2 * j + 1], BF));
    }
  }
};

// dO = dy * g (or dy) into the DO tile; all 256 epilogue threads.
template <int D, bool BF>
__device__ void make_do(const Epi &e, uint32_t g_tile, uint32_t dy_tile, uint32_t do_tile, bool gate) {
  const int row = e.et >> 2, q4 = e.et & 3;
  for (int ch = q4; ch < 8 * (D / 64); ch += 4) {
    const uint32_t off = (uint32_t)((ch >> 3) * kTile) + (uint32_t)(row * 128) + ((((ch & 7) ^ (row & 7)) & 7) << 4);
    uint4 y = ld_shared_v4(dy_tile + off);
    if (gate) {
      const uint4 g = ld_shared_v4(g_tile + off);
      uint32_t *py = &y.x;
      const uint32_t *pg = &g.x;
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack2(py[i], BF), b = unpack2(pg[i], BF);
        py[i] = pack2(a.x * b.x, a.y * b.y, BF);
      }
    }
    st_shared_v4(do_tile + off, y.x, y.y, y.z, y.w);
  }
}

// Masked (col <= row) M=64, N=64 accumulator -> 16-bit [64 x 64] tile; each half owns 32 columns.
template <bool BF>
__device__ void masked_tile(const Epi &e, uint32_t taddr, uint32_t dst) {
  Frag<32> f;
  ld_frag(taddr + 32 * e.half, f);
  tc_fence_before();
  for (int j = 0; j < 4; ++j) {
    const int col = 32 * e.half + 8 * j + e.cq;
    for (int ee = 0; ee < 2; ++ee) {
      const int row = e.r0 + 8 * ee;
      const float a0 = col <= row ? f.v(ee, j, 0) : 0.f;
      const float a1 = col + 1 <= row ? f.v(ee, j, 1) : 0.f;
      st_shared_u32(dst + swz(row, col), pack2(a0, a1, BF));
    }
  }
}

// Output fragment (M=64, W = D/2 columns per half) -> staging tile -> TMA store.
template <int D, bool BF>
__device__ void store_out(const Epi &e, const float (&val)[D / 2], uint32_t stage_tile, const CUtensorMap *map,
                          int h, int b, int t0) {
  if (e.et == 0) tma_store_wait_read0();
  named_bar_sync(1, kEpi);
  for (int j = 0; j < D / 16; ++j) {
    const int col = (D / 2) * e.half + 8 * j + e.cq;
    st_shared_u32(box_addr(stage_tile, e.r0, col), pack2(val[4 * j], val[4 * j + 1], BF));
    st_shared_u32(box_addr(stage_tile, e.r0 + 8, col), pack2(val[4 * j + 2], val[4 * j + 3], BF));
  }
  fence_async_smem();
  named_bar_sync(1, kEpi);
  if (e.et == 0) {
    for (int kb = 0; kb < D / 64; ++kb) tma_store_4d(map, stage_tile + kb * kTile, 64 * kb, t0, h, b);
    tma_store_commit();
  }
}

// ===========================================================================
// forward-direction pass: dq, dg, decay gradient
// ===========================================================================
template <typename T, int D, bool LIT, int NS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_fwddir_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                         const __grid_constant__ CUtensorMap tdy, const __grid_constant__ CUtensorMap tdq,
                         const __grid_constant__ CUtensorMap tdg, const BwdArgs a) {
  using L = BwdLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr int KB = L::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  enum {
    QK_FULL = 2 * NS, QK_FREE, S_READY, DQ_FREE, KV_FULL, P_FULL, O_FULL, DO_FULL, DP_FREE, W_FREE, DPW_FULL,
    DPM_FULL, O_FREE, DQ_FULL, FIN
  };
  const int FULL = 0, EMPTY = NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int nchunks = (a.T + 63) / 64;
  const bool gate = a.g.data != nullptr;
  const bool want_dd = a.ddecay != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 2);
    }
    const int cnt[] = {1, kEpi, 1, kEpi, 1, 1, 1, 1, kEpi, kEpi, 1, 1, kEpi, 1, 1};
    for (int i = 0; i < 15; ++i) mbar_init(bar(QK_FULL + i), cnt[i]);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(sb + L::TMEM_SLOT, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::TMEM_SLOT);

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = (uint32_t)((4 + (gate ? 1 : 0)) * L::BOX);
      int c = 0;
      for (; c < nchunks; ++c) {
        const int s = c % NS, use = c / NS;
        if (!mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag)) break;
        const uint32_t st = sb + s * L::STAGE;
        mbar_arrive_expect_tx(bar(FULL + s), tx);
        for (int kb = 0; kb < KB; ++kb) {
          const int x = 64 * kb, t0 = 64 * c;
          tma_load_4d(st + L::ST_Q + kb * kTile, &tq, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_K + kb * kTile, &tk, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_V + kb * kTile, &tv, bar(FULL + s), x, t0, h, b);
          if (gate) tma_load_4d(st + L::ST_G + kb * kTile, &tg, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_DY + kb * kTile, &tdy, bar(FULL + s), x, t0, h, b);
        }
      }
      for (int d = c - 1; d >= 0 && d >= c - NS; --d)
        mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);   // Q K^T
      const uint32_t id_qs = idesc_f16(64, D, BF, false, true);     // Q S      (B = S, MN-major)
      const uint32_t id_kv = LIT ? idesc_f16(64, 64, BF, false, false) : idesc_f16(D, D, BF, true, true);
      const uint32_t id_pv = idesc_f16(64, D, BF, false, true);     // P V      (B = V, MN-major)
      const uint32_t id_dp = idesc_f16(64, 64, BF, false, false);   // dO V^T
      const uint32_t id_st = idesc_f16(64, D, BF, false, false);    // dO S^T, dO T^T (B = rows, K-major)
      const uint32_t id_dq = idesc_f16(64, D, BF, false, true);     // dP K     (B = K, MN-major)
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % NS, use = c / NS, ph = c & 1;
        const uint32_t st = sb + s * L::STAGE;
        if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(QK_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + L::A_QK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
        }
        mma_commit(bar(QK_FULL));
        // S_{c-1} operand written and decay^L S_{c-1} stored in tensor memory
        if (!mbar_wait(bar(S_READY), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DQ_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + L::A_X, sdesc_k(st + L::ST_Q + off), sdesc_mn(sb + L::SB + ks * 2048, L::PANEL), id_qs,
                  ks > 0);
        }
        for (int ks = 0; ks < 4; ++ks) {  // S_c = decay^L S_{c-1} + U_c, accumulated in place
          if (LIT)
            mma_f16(tmem + L::A_Z, sdesc_k(st + L::ST_K + ks * 32), sdesc_k(st + L::ST_V + ks * 32), id_kv, 1);
          else
            mma_f16(tmem + L::A_Z, sdesc_mn(st + L::ST_K + ks * 2048, kTile), sdesc_mn(st + L::ST_V + ks * 2048, kTile),
                    id_kv, 1);
        }
        mma_commit(bar(KV_FULL));
        if (!mbar_wait(bar(P_FULL), ph, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks)
          mma_f16(tmem + L::A_X, sdesc_k(sb + L::P + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_pv, 1);
        mma_commit(bar(O_FULL));
        if (!mbar_wait(bar(DO_FULL), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DP_FREE), ph ^ 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(W_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
          mma_f16(tmem + L::A_DP, sdesc_k(sb + L::DO + off), sdesc_k(st + L::ST_V + off), id_dp, ks > 0);
          if (want_dd)
            mma_f16(tmem + L::A_Y, sdesc_k(sb + L::DO + off), sdesc_k(sb + L::TB + poff), id_st, ks > 0);
        }
        mma_commit(bar(DPW_FULL));
        if (!mbar_wait(bar(DPM_FULL), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(O_FREE), ph, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {  // dq = dO S^T + dP K
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
          mma_f16(tmem + L::A_X, sdesc_k(sb + L::DO + off), sdesc_k(sb + L::SB + poff), id_st, ks > 0);
        }
        for (int ks = 0; ks < 4; ++ks)
          mma_f16(tmem + L::A_X, sdesc_k(sb + L::DP + ks * 32), sdesc_mn(st + L::ST_K + ks * 2048, kTile), id_dq, 1);
        mma_commit(bar(DQ_FULL));
        mma_commit(bar(EMPTY + s));
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else {
    const Epi e;
    const size_t sbase = ((size_t)b * a.H + h) * D * D;
    Carry<D> Td;  // decay tangent, registers
    Td.init(e);
    Td.load(e, nullptr);
    float af[Carry<D>::NR], at[Carry<D>::NR];
    const int Ltail = a.T - (nchunks - 1) * 64;
    for (int r = 0; r < Carry<D>::NR; ++r) {
      af[r] = chunk_alpha(a.decay, b, h, Td.row[r], 64, 64);
      at[r] = chunk_alpha(a.decay, b, h, Td.row[r], Ltail, 64);
    }
    double dlog = 0.0;  // thread et < D owns key channel et
    float *red = reinterpret_cast<float *>(smem + L::RED);

    for (int c = 0; c < nchunks; ++c) {
      const int s = c % NS, use = c / NS, ph = c & 1;
      const uint32_t st = sb + s * L::STAGE;
      const int t0 = 64 * c, Lc = min(64, a.T - t0);
      // state step: S_{c-1} -> operand; decay^L S_{c-1} -> tensor memory; tangent update.
      // Done in slices of the thread's columns to keep register pressure low.
      if (c > 0) {
        if (!mbar_wait(bar(KV_FULL), (c - 1) & 1, a.status, abort_flag)) break;
        tc_fence_after();
      }
      {
        float alr[Carry<D>::NR];
        for (int r = 0; r < Carry<D>::NR; ++r) alr[r] = (Lc == 64) ? af[r] : at[r];
        const float Lf = (float)Lc;
        if (D == 128) {
          const int row = Td.row[0];
          const uint32_t pb = (uint32_t)(e.half * D * 128);
          for (int sl = 0; sl < 2; ++sl) {
            const uint32_t col0 = 64 * e.half + 32 * sl;
            uint32_t u[32];
            if (c == 0) {
              for (int i = 0; i < 32; ++i)
                u[i] = __float_as_uint(a.s_in ? a.s_in[sbase + (size_t)row * D + col0 + i] : 0.f);
            } else {
              tmem_ld_32x32b_x32(tmem + e.lane_off + L::A_Z + col0, u);
            }
            for (int j = 0; j < 4; ++j) {
              const int jj = 4 * sl + j;
              st_shared_v4(sb + L::SB + pb + swz(row, 8 * jj), pack2(__uint_as_float(u[8 * j]), __uint_as_float(u[8 * j + 1]), BF),
                           pack2(__uint_as_float(u[8 * j + 2]), __uint_as_float(u[8 * j + 3]), BF),
                           pack2(__uint_as_float(u[8 * j + 4]), __uint_as_float(u[8 * j + 5]), BF),
                           pack2(__uint_as_float(u[8 * j + 6]), __uint_as_float(u[8 * j + 7]), BF));
              if (want_dd)
                st_shared_v4(sb + L::TB + pb + swz(row, 8 * jj), pack2(Td.x[0][8 * jj], Td.x[0][8 * jj + 1], BF),
                             pack2(Td.x[0][8 * jj + 2], Td.x[0][8 * jj + 3], BF),
                             pack2(Td.x[0][8 * jj + 4], Td.x[0][8 * jj + 5], BF),
                             pack2(Td.x[0][8 * jj + 6], Td.x[0][8 * jj + 7], BF));
            }
            for (int i = 0; i < 32; ++i) {
              const float sv = __uint_as_float(u[i]);
              Td.x[0][32 * sl + i] = alr[0] * fmaf(Lf, sv, Td.x[0][32 * sl + i]);
              u[i] = __float_as_uint(alr[0] * sv);
            }
            tmem_st_32x32b_x32(tmem + e.lane_off + L::A_Z + col0, u);
          }
        } else {
          Carry<D> Sp;
          Sp.row[0] = Td.row[0];
          Sp.row[Carry<D>::NR - 1] = Td.row[Carry<D>::NR - 1];
          if (c == 0) Sp.load(e, a.s_in ? a.s_in + sbase : nullptr);
          else Sp.tmem_load(e, tmem, L::A_Z);
          Sp.template write<BF>(e, sb + L::SB);
          if (want_dd) Td.template write<BF>(e, sb + L::TB);
          for (int r = 0; r < Carry<D>::NR; ++r)
            for (int i = 0; i < Carry<D>::NV; ++i) {
              Td.x[r][i] = alr[r] * fmaf(Lf, Sp.x[r][i], Td.x[r][i]);
              Sp.x[r][i] *= alr[r];
            }
          Sp.tmem_store(e, tmem, L::A_Z);
        }
        fence_async_smem();
        tc_fence_before();
        named_bar_sync(1, kEpi);
        if (e.et == 0) mbar_arrive(bar(S_READY));
      }
      if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
      // (0) dO
      make_do<D, BF>(e, st + L::ST_G, st + L::ST_DY, sb + L::DO, gate);
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(DO_FULL));
      // (a) P
      if (!mbar_wait(bar(QK_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      masked_tile<BF>(e, tmem + e.lane_off + L::A_QK, sb + L::P);
      mbar_arrive(bar(QK_FREE));
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(P_FULL));
      // (b) O -> dg
      if (!mbar_wait(bar(O_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      {
        Frag<D / 2> fo;
        ld_frag(tmem + e.lane_off + L::A_X + (D / 2) * e.half, fo);
        tc_fence_before();
        mbar_arrive(bar(O_FREE));
        if (gate) {
          float dg[D / 2];
          for (int j = 0; j < D / 16; ++j)
            for (int ee = 0; ee < 2; ++ee) {
              const int col = (D / 2) * e.half + 8 * j + e.cq;
              const float2 y = unpack2(ld_shared_u32(box_addr(st + L::ST_DY, e.r0 + 8 * ee, col)), BF);
              dg[4 * j + 2 * ee] = y.x * fo.v(ee, j, 0);
              dg[4 * j + 2 * ee + 1] = y.y * fo.v(ee, j, 1);
            }
          store_out<D, BF>(e, dg, sb + L::O1, &tdg, h, b, t0);
        }
      }
      // (d) dP (masked); decay term sum_t q_t . (dO T^T)_t
      if (!mbar_wait(bar(DPW_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      masked_tile<BF>(e, tmem + e.lane_off + L::A_DP, sb + L::DP);
      mbar_arrive(bar(DP_FREE));
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(DPM_FULL));
      if (want_dd) {
        Frag<D / 2> fw;
        ld_frag(tmem + e.lane_off + L::A_Y + (D / 2) * e.half, fw);
        tc_fence_before();
        mbar_arrive(bar(W_FREE));
        float part[D / 8];
        for (int j = 0; j < D / 16; ++j) {
          const int col = (D / 2) * e.half + 8 * j + e.cq;
          const float2 q0 = unpack2(ld_shared_u32(box_addr(st + L::ST_Q, e.r0, col)), BF);
          const float2 q1 = unpack2(ld_shared_u32(box_addr(st + L::ST_Q, e.r0 + 8, col)), BF);
          part[2 * j] = q0.x * fw.v(0, j, 0) + q1.x * fw.v(1, j, 0);
          part[2 * j + 1] = q0.y * fw.v(0, j, 1) + q1.y * fw.v(1, j, 1);
        }
        for (int i = 0; i < D / 8; ++i) {
          float v = part[i];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          part[i] = v;
        }
        float *rb = red + (c & 1) * 4 * D;
        if (e.lane < 4)
          for (int j = 0; j < D / 16; ++j)
            for (int k = 0; k < 2; ++k) rb[e.sp * D + (D / 2) * e.half + 8 * j + e.cq + k] = part[2 * j + k];
        named_bar_sync(1, kEpi);
        if (e.et < D) dlog += (double)(rb[e.et] + rb[D + e.et] + rb[2 * D + e.et] + rb[3 * D + e.et]);
      } else {
        tc_fence_before();
        mbar_arrive(bar(W_FREE));
        named_bar_sync(1, kEpi);
      }
      if (e.et == 0) mbar_arrive(bar(EMPTY + s));  // Q, G, dY of this stage no longer read
      // (e) dq
      if (!mbar_wait(bar(DQ_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      {
        Frag<D / 2> fd;
        ld_frag(tmem + e.lane_off + L::A_X + (D / 2) * e.half, fd);
        tc_fence_before();
        mbar_arrive(bar(DQ_FREE));
        float dq[D / 2];
        for (int i = 0; i < D / 2; ++i) dq[i] = __uint_as_float(fd.r[i]);
        store_out<D, BF>(e, dq, sb + L::O2, &tdq, h, b, t0);
      }
    }
    if (want_dd) {
      // final-state term <dS_T[i,:], T_T[i,:]>, then dL/d decay = dL/dlog decay / decay
      float *rowsum = red;
      named_bar_sync(1, kEpi);
      if (e.et < D) rowsum[e.et] = 0.f;
      named_bar_sync(1, kEpi);
      if (a.ds_out) {
        for (int r = 0; r < Carry<D>::NR; ++r) {
          float p = 0.f;
          for (int i = 0; i < Carry<D>::NV; ++i)
            p += a.ds_out[sbase + (size_t)Td.row[r] * D + Td.col(e, i)] * Td.x[r][i];
          atomicAdd(&rowsum[Td.row[r]], p);
        }
      }
      named_bar_sync(1, kEpi);
      if (e.et < D) {
        dlog += (double)rowsum[e.et];
        const double av = (double)decay_value(a.decay, b, h, e.et);
        a.ddecay[((size_t)b * a.H + h) * D + e.et] = (av != 0.0) ? (float)(dlog / av) : 0.f;
      }
    }
    if (e.et == 0) tma_store_wait_all();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ===========================================================================
// reverse pass: dk, dv, d(initial state)
// ===========================================================================
template <typename T, int D, bool LIT, int NS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_revdir_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tg,
                         const __grid_constant__ CUtensorMap tdy, const __grid_constant__ CUtensorMap tdk,
                         const __grid_constant__ CUtensorMap tdv, const BwdArgs a) {
  using L = BwdLayout<D, NS>;
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  constexpr int KB = L::KB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  auto bar = [&](int i) { return sb + L::BAR + 8u * i; };
  enum {
    QK_FULL = 2 * NS, QK_FREE, DO_FULL, DP_FULL, DP_FREE, DS_FULL, DKI_FREE, DVI_FREE, INTER_FULL, QDO_FREE,
    QDO_FULL, P_FULL, DPM_FULL, KV_FULL, FIN
  };
  const int FULL = 0, EMPTY = NS;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::ABORT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  const int nchunks = (a.T + 63) / 64;
  const bool gate = a.g.data != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(bar(FULL + s), 1);
      mbar_init(bar(EMPTY + s), 2);
    }
    const int cnt[] = {1, kEpi, 1, 1, kEpi, 1, kEpi, kEpi, 1, kEpi, 1, 1, 1, 1, 1};
    for (int i = 0; i < 15; ++i) mbar_init(bar(QK_FULL + i), cnt[i]);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(sb + L::TMEM_SLOT, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(smem + L::TMEM_SLOT);

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = (uint32_t)((4 + (gate ? 1 : 0)) * L::BOX);
      int it = 0;
      for (; it < nchunks; ++it) {
        const int c = nchunks - 1 - it, s = it % NS, use = it / NS;
        if (!mbar_wait(bar(EMPTY + s), (use & 1) ^ 1, a.status, abort_flag)) break;
        const uint32_t st = sb + s * L::STAGE;
        mbar_arrive_expect_tx(bar(FULL + s), tx);
        for (int kb = 0; kb < KB; ++kb) {
          const int x = 64 * kb, t0 = 64 * c;
          tma_load_4d(st + L::ST_Q + kb * kTile, &tq, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_K + kb * kTile, &tk, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_V + kb * kTile, &tv, bar(FULL + s), x, t0, h, b);
          if (gate) tma_load_4d(st + L::ST_G + kb * kTile, &tg, bar(FULL + s), x, t0, h, b);
          tma_load_4d(st + L::ST_DY + kb * kTile, &tdy, bar(FULL + s), x, t0, h, b);
        }
      }
      for (int d = it - 1; d >= 0 && d >= it - NS; --d)
        mbar_wait(bar(FULL + d % NS), (d / NS) & 1, a.status, abort_flag);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = idesc_f16(64, 64, BF, false, false);
      const uint32_t id_dp = idesc_f16(64, 64, BF, false, false);
      // inter terms
      const uint32_t id_dki = LIT ? idesc_f16(64, 64, BF, false, true) : idesc_f16(64, D, BF, false, false);
      const uint32_t id_dvi = LIT ? idesc_f16(64, 64, BF, true, true) : idesc_f16(64, D, BF, false, true);
      const uint32_t id_qdo = idesc_f16(D, D, BF, true, true);  // Q^T dO
      const uint32_t id_t = idesc_f16(64, D, BF, true, true);   // dP^T Q and P^T dO
      for (int it = 0; it < nchunks; ++it) {
        const int s = it % NS, use = it / NS, ph = it & 1;
        const uint32_t st = sb + s * L::STAGE;
        if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(QK_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + L::A_QK, sdesc_k(st + L::ST_Q + off), sdesc_k(st + L::ST_K + off), id_qk, ks > 0);
        }
        mma_commit(bar(QK_FULL));
        if (!mbar_wait(bar(DO_FULL), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DP_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
          mma_f16(tmem + L::A_DP, sdesc_k(sb + L::DO + off), sdesc_k(st + L::ST_V + off), id_dp, ks > 0);
        }
        mma_commit(bar(DP_FULL));
        if (!mbar_wait(bar(DS_FULL), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DKI_FREE), ph ^ 1, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DVI_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        if (LIT) {
          for (int ks = 0; ks < 4; ++ks) {
            // dS V: A = dS (rows p, K = q), B = V (N = d, K = q rows)
            mma_f16(tmem + L::A_X, sdesc_k(sb + L::SB + ks * 32), sdesc_mn(st + L::ST_V + ks * 2048, kTile), id_dki,
                    ks > 0);
            // dS^T K: A = dS^T (M = q columns, K = p rows), B = K (N = d, K = p rows)
            mma_f16(tmem + L::A_Y, sdesc_mn(sb + L::SB + ks * 2048, L::PANEL),
                    sdesc_mn(st + L::ST_K + ks * 2048, kTile), id_dvi, ks > 0);
          }
        } else {
          for (int ks = 0; ks < D / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kTile + (ks & 3) * 32;
            const uint32_t poff = (ks >> 2) * L::PANEL + (ks & 3) * 32;
            // V dS^T: A = V (M = tokens, K = dv), B = dS rows (N = dk, K = dv)
            mma_f16(tmem + L::A_X, sdesc_k(st + L::ST_V + off), sdesc_k(sb + L::SB + poff), id_dki, ks > 0);
            // K dS: A = K (M = tokens, K = dk), B = dS (N = dv, K = dk rows)
            mma_f16(tmem + L::A_Y, sdesc_k(st + L::ST_K + off), sdesc_mn(sb + L::SB + ks * 2048, L::PANEL), id_dvi,
                    ks > 0);
          }
        }
        mma_commit(bar(INTER_FULL));
        if (!mbar_wait(bar(QDO_FREE), ph ^ 1, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks)
          mma_f16(tmem + L::A_Z, sdesc_mn(st + L::ST_Q + ks * 2048, kTile), sdesc_mn(sb + L::DO + ks * 2048, kTile),
                  id_qdo, ks > 0);
        mma_commit(bar(QDO_FULL));
        if (!mbar_wait(bar(P_FULL), ph, a.status, abort_flag)) break;
        if (!mbar_wait(bar(DPM_FULL), ph, a.status, abort_flag)) break;
        tc_fence_after();
        for (int ks = 0; ks < 4; ++ks) {
          mma_f16(tmem + L::A_X, sdesc_mn(sb + L::DP + ks * 2048, kTile), sdesc_mn(st + L::ST_Q + ks * 2048, kTile),
                  id_t, 1);
          mma_f16(tmem + L::A_Y, sdesc_mn(sb + L::P + ks * 2048, kTile), sdesc_mn(sb + L::DO + ks * 2048, kTile),
                  id_t, 1);
        }
        mma_commit(bar(KV_FULL));
        mma_commit(bar(EMPTY + s));
      }
      mma_commit(bar(FIN));
      mbar_wait(bar(FIN), 0, a.status, abort_flag);
    }
    __syncwarp();
  } else {
    const Epi e;
    const size_t sbase = ((size_t)b * a.H + h) * D * D;
    Carry<D> dS;
    dS.init(e);
    dS.load(e, a.ds_out ? a.ds_out + sbase : nullptr);
    dS.template write<BF>(e, sb + L::SB);
    fence_async_smem();
    named_bar_sync(1, kEpi);
    if (e.et == 0) mbar_arrive(bar(DS_FULL));
    float af[Carry<D>::NR], at[Carry<D>::NR];
    const int Ltail = a.T - (nchunks - 1) * 64;
    for (int r = 0; r < Carry<D>::NR; ++r) {
      af[r] = chunk_alpha(a.decay, b, h, dS.row[r], 64, 64);
      at[r] = chunk_alpha(a.decay, b, h, dS.row[r], Ltail, 64);
    }

    for (int it = 0; it < nchunks; ++it) {
      const int c = nchunks - 1 - it, s = it % NS, use = it / NS, ph = it & 1;
      const uint32_t st = sb + s * L::STAGE;
      const int t0 = 64 * c, Lc = min(64, a.T - t0);
      if (!mbar_wait(bar(FULL + s), use & 1, a.status, abort_flag)) break;
      make_do<D, BF>(e, st + L::ST_G, st + L::ST_DY, sb + L::DO, gate);
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(DO_FULL));
      // (a) P
      if (!mbar_wait(bar(QK_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      masked_tile<BF>(e, tmem + e.lane_off + L::A_QK, sb + L::P);
      mbar_arrive(bar(QK_FREE));
      // (b) dP
      if (!mbar_wait(bar(DP_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      masked_tile<BF>(e, tmem + e.lane_off + L::A_DP, sb + L::DP);
      mbar_arrive(bar(DP_FREE));
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) {
        mbar_arrive(bar(P_FULL));
        mbar_arrive(bar(DPM_FULL));
      }
      // (c) the inter MMAs have read dS_c
      if (!mbar_wait(bar(INTER_FULL), ph, a.status, abort_flag)) break;
      if (e.et == 0) mbar_arrive(bar(EMPTY + s));  // G and dY of this stage no longer read
      // (d) dS <- alpha dS + Q^T dO  (the inter MMAs have consumed dS)
      if (!mbar_wait(bar(QDO_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      {
        float al[Carry<D>::NR];
        for (int r = 0; r < Carry<D>::NR; ++r) al[r] = (Lc == 64) ? af[r] : at[r];
        dS.update(e, tmem, L::A_Z, al);
      }
      tc_fence_before();
      mbar_arrive(bar(QDO_FREE));
      dS.template write<BF>(e, sb + L::SB);
      fence_async_smem();
      named_bar_sync(1, kEpi);
      if (e.et == 0) mbar_arrive(bar(DS_FULL));
      // (e) dk, dv
      if (!mbar_wait(bar(KV_FULL), ph, a.status, abort_flag)) break;
      tc_fence_after();
      {
        Frag<D / 2> fk, fv;
        ld_frag(tmem + e.lane_off + L::A_X + (D / 2) * e.half, fk);
        ld_frag(tmem + e.lane_off + L::A_Y + (D / 2) * e.half, fv);
        tc_fence_before();
        mbar_arrive(bar(DKI_FREE));
        mbar_arrive(bar(DVI_FREE));
        float o[D / 2];
        for (int i = 0; i < D / 2; ++i) o[i] = __uint_as_float(fk.r[i]);
        store_out<D, BF>(e, o, sb + L::O1, &tdk, h, b, t0);
        for (int i = 0; i < D / 2; ++i) o[i] = __uint_as_float(fv.r[i]);
        store_out<D, BF>(e, o, sb + L::O2, &tdv, h, b, t0);
      }
    }
    if (a.ds_in) dS.store(e, a.ds_in + sbase);
    if (e.et == 0) tma_store_wait_all();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D, bool LIT, int NS>
cudaError_t bwd_tc_launch(const BwdArgs &a, cudaStream_t st) {
  constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
  CUtensorMap mq, mk, mv, mg, mdy, mdq, mdk, mdv, mdg;
  const View gview = a.g.data ? a.g : a.q;
  const View dgview = a.g.data ? a.dg : a.dq;
  bool ok = make_tmap_bhtd(&mq, a.q, a.B, a.H, a.T, a.D, BF) && make_tmap_bhtd(&mk, a.k, a.B, a.H, a.T, a.D, BF) &&
            make_tmap_bhtd(&mv, a.v, a.B, a.H, a.T, a.D, BF) && make_tmap_bhtd(&mg, gview, a.B, a.H, a.T, a.D, BF) &&
            make_tmap_bhtd(&mdy, a.dy, a.B, a.H, a.T, a.D, BF) && make_tmap_bhtd(&mdq, a.dq, a.B, a.H, a.T, a.D, BF) &&
            make_tmap_bhtd(&mdk, a.dk, a.B, a.H, a.T, a.D, BF) && make_tmap_bhtd(&mdv, a.dv, a.B, a.H, a.T, a.D, BF) &&
            make_tmap_bhtd(&mdg, dgview, a.B, a.H, a.T, a.D, BF);
  if (!ok) return cudaErrorInvalidValue;
  using L = BwdLayout<D, NS>;
  auto k1 = bwd_fwddir_tc_kernel<T, D, LIT, NS>;
  auto k2 = bwd_revdir_tc_kernel<T, D, LIT, NS>;
  cudaError_t e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return e;
  k1<<<a.B * a.H, kBwdThreads, L::SMEM, st>>>(mq, mk, mv, mg, mdy, mdq, mdg, a);
  count_launches(1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k2<<<a.B * a.H, kBwdThreads, L::SMEM, st>>>(mq, mk, mv, mg, mdy, mdk, mdv, a);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_bwd_tc(const BwdArgs &a, int dtype, cudaStream_t st) {
  const bool bf = dtype == KDA_DTYPE_BF16;
  if (a.D == 64) {
    if (a.literal) return bf ? bwd_tc_launch<__nv_bfloat16, 64, true, 2>(a, st) : bwd_tc_launch<__half, 64, true, 2>(a, st);
    return bf ? bwd_tc_launch<__nv_bfloat16, 64, false, 2>(a, st) : bwd_tc_launch<__half, 64, false, 2>(a, st);
  }
  return bf ? bwd_tc_launch<__nv_bfloat16, 128, false, 1>(a, st) : bwd_tc_launch<__half, 128, false, 1>(a, st);
}

}  // namespace kda
