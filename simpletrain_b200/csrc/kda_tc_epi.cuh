// Shared pieces of the sm_100a KDA kernels: epilogue thread geometry, tensor-
// memory fragments, the fp32 carry (state) layout, smem tile helpers, direct
// global stores, and the persistent work queue with chained state handoff.
//
// Scheduling.  A "stream" is one (batch, head).  The stream-major sequence of
// all (stream, chunk) pairs is cut into `nranges` contiguous ranges of equal
// length (to one chunk), one per persistent CTA slot; CTAs take range tickets
// from an atomic counter in the workspace.  A range is split at stream
// boundaries into pieces: at most a partial first piece (the end of a stream
// begun by the range before), whole streams, and at most a partial last piece
// (the start of a stream finished by the range after).  The carried state
// crosses a range boundary through one slot per boundary.  Pieces run in an
// order that makes the boundary wait cheap: in the forward direction the last
// piece (a stream start, no wait) runs first and publishes its end state, the
// first piece (which waits for the previous range's publish) runs last; the
// reverse direction mirrors this with the ranges ticketed last-to-first.  A
// range therefore only waits for a range ticketed before it, which a running
// CTA holds (no deadlock), and usually for a piece finished long before.
// Every wait is bounded.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "kda_internal.h"
#include "tc_common.cuh"

// Development tracing: built only with -DKDA_TRACE (python -m simpletrain_b200.build
// --trace writes a separate library); records clock64() of pipeline events of
// CTA 0 into a per-kernel-file device array [chunk][32 slots], and the global
// timer (ns) of per-CTA milestones into [CTA][16 slots] (slot 7: SM id).
#ifdef KDA_TRACE
#define KDA_TRACE_DEFINE                                      \
  static __device__ unsigned long long g_kda_trace[128 * 32]; \
  static __device__ unsigned long long g_kda_trace_cta[1024 * 16];
#define KDA_TRACE_EVENT(slot, chunk)                                                    \
  do {                                                                                  \
    if (blockIdx.x == 0 && (chunk) < 128) g_kda_trace[(chunk) * 32 + (slot)] = clock64(); \
  } while (0)
#define KDA_TRACE_CTA(slot, value)                                               \
  do {                                                                           \
    if (blockIdx.x < 1024) g_kda_trace_cta[blockIdx.x * 16 + (slot)] = (value); \
  } while (0)
// cycles spent in `expr` (a wait) added to `acc`
#define KDA_TIMED(acc, expr)                  \
  ([&]() {                                    \
    const long long kda_t0_ = clock64();      \
    const auto kda_r_ = (expr);               \
    (acc) += clock64() - kda_t0_;             \
    return kda_r_;                            \
  }())
#define KDA_CLK(v) const long long v = clock64()
#define KDA_ADD(acc, from) (acc) += clock64() - (from)
__device__ __forceinline__ unsigned long long kda_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned kda_smid() {
  unsigned r;
  asm volatile("mov.u32 %0, %smid;" : "=r"(r));
  return r;
}
#else
#define KDA_TRACE_DEFINE
#define KDA_TRACE_EVENT(slot, chunk) \
  do {                               \
  } while (0)
#define KDA_TRACE_CTA(slot, value) \
  do {                             \
  } while (0)
#define KDA_TIMED(acc, expr) (expr)
#define KDA_CLK(v)
#define KDA_ADD(acc, from)
#endif

namespace kda {
namespace tc {

constexpr int kTile = 64 * 64 * 2;  // one [64 x 64] 16-bit box, 8 KB
constexpr int kQ = 2;               // epilogue warps per TMEM sub-partition: column groups
constexpr int kEpi = 128 * kQ;      // epilogue threads (warps 2 .. 1 + 4 kQ)
constexpr int kThreads = 64 + kEpi; // + TMA warp + MMA warp

// ------------------------------------------------------------- geometry --
// kQ epilogue warps per TMEM sub-partition (TMEM lanes 32 sp .. 32 sp + 31);
// column group `cg` owns 1 / kQ of every accumulator's columns.
struct Epi {
  int et, lane, sp, cg, r0, cq;
  uint32_t lane_off;
  __device__ Epi() : Epi((int)threadIdx.x) {}
  // the geometry of CTA thread `tid` of the main kernels (warps 2 ..), for
  // kernels that keep the carry layout without the producer warps
  __device__ explicit Epi(int tid) {
    et = tid - 64;
    lane = tid & 31;
    sp = (tid >> 5) & 3;
    cg = et >> 7;
    r0 = 16 * sp + (lane >> 2);
    cq = 2 * (lane & 3);
    lane_off = (uint32_t)(32 * sp) << 16;
  }
};

// M=64 accumulator fragment of W columns per warp: rows r0 and r0+8,
// columns W*cg + 8j + cq + {0,1}; value (e, j, k) at r[4j + 2e + k].
template <int W>
struct Frag {
  uint32_t r[W / 2];
  __device__ __forceinline__ float v(int e, int j, int k) const { return __uint_as_float(r[4 * j + 2 * e + k]); }
};
__device__ __forceinline__ void ld_frag(uint32_t taddr, Frag<16> &f) { tmem_ld_16x256b_x2(taddr, f.r); }
__device__ __forceinline__ void ld_frag(uint32_t taddr, Frag<32> &f) { tmem_ld_16x256b_x4(taddr, f.r); }
__device__ __forceinline__ void ld_frag(uint32_t taddr, Frag<64> &f) { tmem_ld_16x256b_x8(taddr, f.r); }

// (row, col) of a [64 rows x 64*KB cols] tile stored as KB swizzled boxes
__device__ __forceinline__ uint32_t box_addr(uint32_t base, int row, int col) {
  return base + (uint32_t)((col >> 6) * kTile) + swz(row, col & 63);
}
// (row, col) of a state operand stored as panels of [D rows x 64 cols]
template <int D>
__device__ __forceinline__ uint32_t panel_addr(uint32_t base, int row, int col) {
  return base + (uint32_t)((col >> 6) * D * 128) + swz(row, col & 63);
}

// ------------------------------------------------------------------ carry --
// fp32 D x D carry (state or its gradient / tangent) owned by the epilogue,
// W = D / kQ columns per thread group:
//   D=128 (M=128 accumulators): row 32*sp + lane, columns W*cg + [0, W)
//   D=64  (M=64 accumulators) : rows r0, r0+8, columns W*cg + 8j + cq + k (j < W/8)
template <int D>
struct Carry {
  static constexpr int W = D / kQ;
  static constexpr int NR = (D == 128) ? 1 : 2;
  static constexpr int NV = (D == 128) ? W : W / 4;
  static constexpr int FLOATS = NR * NV;  // per thread
  float x[NR][NV];
  int row[NR];
  // carry layout: register column i of a thread is matrix column col_of(e, i);
  // its register row r is matrix row row_of(e, r)
  static __device__ __forceinline__ int col_of(const Epi &e, int i) {
    return (D == 128) ? W * e.cg + i : W * e.cg + 8 * (i >> 1) + e.cq + (i & 1);
  }
  static __device__ __forceinline__ int row_of(const Epi &e, int r) {
    return (D == 128) ? 32 * e.sp + e.lane : e.r0 + 8 * r;
  }
  __device__ __forceinline__ int col(const Epi &e, int i) const { return col_of(e, i); }
  __device__ void init_rows(const Epi &e) {
    for (int r = 0; r < NR; ++r) row[r] = row_of(e, r);
  }
  __device__ void zero() {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) x[r][i] = 0.f;
  }
  // row-major [D][D] fp32 (user-facing states, 16-byte aligned), in the widest
  // accesses the layout allows: float4 runs of a row (D=128), float2 pairs (D=64)
  __device__ void load_rm(const Epi &e, const float *src) {
    if (src == nullptr) {
      zero();
      return;
    }
    if constexpr (D == 128) {
      const float4 *s4 = reinterpret_cast<const float4 *>(src + (size_t)row[0] * D + W * e.cg);
      for (int i = 0; i < NV / 4; ++i) {
        const float4 v = __ldg(s4 + i);
        x[0][4 * i] = v.x; x[0][4 * i + 1] = v.y; x[0][4 * i + 2] = v.z; x[0][4 * i + 3] = v.w;
      }
    } else {
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < NV / 2; ++j) {
          const float2 v = __ldg(reinterpret_cast<const float2 *>(src + (size_t)row[r] * D + col(e, 2 * j)));
          x[r][2 * j] = v.x;
          x[r][2 * j + 1] = v.y;
        }
    }
  }
  __device__ void store_rm(const Epi &e, float *dst) const {
    if constexpr (D == 128) {
      float4 *d4 = reinterpret_cast<float4 *>(dst + (size_t)row[0] * D + W * e.cg);
      for (int i = 0; i < NV / 4; ++i)
        d4[i] = make_float4(x[0][4 * i], x[0][4 * i + 1], x[0][4 * i + 2], x[0][4 * i + 3]);
    } else {
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < NV / 2; ++j)
          *reinterpret_cast<float2 *>(dst + (size_t)row[r] * D + col(e, 2 * j)) = make_float2(x[r][2 * j], x[r][2 * j + 1]);
    }
  }
  // handoff slot layout: float4 index i4 of thread et at slot[i4 * kEpi + et]
  __device__ void store_slot(const Epi &e, float4 *slot) const {
    const float *f = &x[0][0];
    for (int i4 = 0; i4 < FLOATS / 4; ++i4)
      __stcg(slot + i4 * kEpi + e.et, make_float4(f[4 * i4], f[4 * i4 + 1], f[4 * i4 + 2], f[4 * i4 + 3]));
  }
  __device__ void load_slot(const Epi &e, const float4 *slot) {
    float *f = &x[0][0];
    for (int i4 = 0; i4 < FLOATS / 4; ++i4) {
      const float4 v = __ldcg(slot + i4 * kEpi + e.et);
      f[4 * i4] = v.x; f[4 * i4 + 1] = v.y; f[4 * i4 + 2] = v.z; f[4 * i4 + 3] = v.w;
    }
  }
  // tensor memory (M = D accumulator at column base `acc`)
  __device__ void tmem_load(const Epi &e, uint32_t tmem, uint32_t acc) {
    if constexpr (D == 128) {
      for (int sl = 0; sl < W / 32; ++sl) {
        uint32_t u[32];
        tmem_ld_32x32b_x32(tmem + e.lane_off + acc + W * e.cg + 32 * sl, u);
        for (int i = 0; i < 32; ++i) x[0][32 * sl + i] = __uint_as_float(u[i]);
      }
    } else {
      Frag<W> f;
      ld_frag(tmem + e.lane_off + acc + W * e.cg, f);
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < W / 8; ++j)
          for (int k = 0; k < 2; ++k) x[r][2 * j + k] = f.v(r, j, k);
    }
  }
  __device__ void tmem_store(const Epi &e, uint32_t tmem, uint32_t acc) const {
    if constexpr (D == 128) {
      for (int sl = 0; sl < W / 32; ++sl) {
        uint32_t u[32];
        for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(x[0][32 * sl + i]);
        tmem_st_32x32b_x32(tmem + e.lane_off + acc + W * e.cg + 32 * sl, u);
      }
    } else {
      uint32_t u[W / 2];
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < W / 8; ++j)
          for (int k = 0; k < 2; ++k) u[4 * j + 2 * r + k] = __float_as_uint(x[r][2 * j + k]);
      if constexpr (W == 16) tmem_st_16x256b_x2(tmem + e.lane_off + acc + W * e.cg, u);
      else tmem_st_16x256b_x4(tmem + e.lane_off + acc + W * e.cg, u);
    }
  }
  // 16-bit copy of sc * carry into a state operand (panels of [D rows x 64 cols])
  template <bool BF>
  __device__ __forceinline__ void write_operand(const Epi &e, uint32_t base, float sc = 1.f) const {
    if constexpr (D == 128) {
      for (int j = 0; j < W / 8; ++j) {
        const float *f = &x[0][8 * j];
        st_shared_v4(panel_addr<D>(base, row[0], W * e.cg + 8 * j), pack2(sc * f[0], sc * f[1], BF),
                     pack2(sc * f[2], sc * f[3], BF), pack2(sc * f[4], sc * f[5], BF), pack2(sc * f[6], sc * f[7], BF));
      }
    } else {
      for (int r = 0; r < NR; ++r)
        for (int j = 0; j < W / 8; ++j)
          st_shared_u32(panel_addr<D>(base, row[r], W * e.cg + 8 * j + e.cq),
                        pack2(sc * x[r][2 * j], sc * x[r][2 * j + 1], BF));
    }
  }
};
static_assert(kQ == 2 || kQ == 4, "column groups of 64 or 32 (D=128) and 32 or 16 (D=64)");

// ---------------------------------------------------------- tile helpers --
// Row of the DO tile that epilogue thread `et` writes in make_do.
__device__ __forceinline__ int make_do_row(int et) { return et / (kEpi / 64); }

// dO = dy * g (or dy) into the DO tile; all epilogue threads, eight per row.
// ROWF: also times rowf, this thread's row factor (per-step mode).
template <int D, bool BF, bool ROWF = false>
__device__ void make_do(const Epi &e, uint32_t g_tile, uint32_t dy_tile, uint32_t do_tile, bool gate,
                        float rowf = 1.f) {
  constexpr int TPR = kEpi / 64;            // threads per row
  constexpr int N = 8 * (D / 64) / TPR;    // 16-byte chunks per thread
  const int row = make_do_row(e.et), q = e.et % TPR;
  uint32_t off[N];
  uint4 y[N], g[N];
  for (int i = 0; i < N; ++i) {  // all loads first: the shared-memory accesses are ordered asm
    const int ch = q + TPR * i;
    off[i] = (uint32_t)((ch >> 3) * kTile) + (uint32_t)(row * 128) + ((((ch & 7) ^ (row & 7)) & 7) << 4);
    y[i] = ld_shared_v4(dy_tile + off[i]);
    if (gate) g[i] = ld_shared_v4(g_tile + off[i]);
  }
  for (int i = 0; i < N; ++i) {
    if (gate) {
      uint32_t *py = &y[i].x;
      const uint32_t *pg = &g[i].x;
      for (int k = 0; k < 4; ++k) {
        const float2 a = unpack2(py[k], BF), b = unpack2(pg[k], BF);
        py[k] = ROWF ? pack2(rowf * (a.x * b.x), rowf * (a.y * b.y), BF) : pack2(a.x * b.x, a.y * b.y, BF);
      }
    } else if (ROWF) {
      uint32_t *py = &y[i].x;
      for (int k = 0; k < 4; ++k) {
        const float2 a = unpack2(py[k], BF);
        py[k] = pack2(rowf * a.x, rowf * a.y, BF);
      }
    }
    st_shared_v4(do_tile + off[i], y[i].x, y[i].y, y[i].z, y[i].w);
  }
}

// Masked (col <= row) M=64, N=64 accumulator -> 16-bit [64 x 64] tile; each
// column group owns 64 / kQ columns.  Ends with tcgen05.fence::before_thread_sync
// (the accumulator may be reused after a barrier).
template <bool BF>
__device__ void masked_tile(const Epi &e, uint32_t taddr, uint32_t dst) {
  constexpr int W = 64 / kQ;
  Frag<W> f;
  ld_frag(taddr + W * e.cg, f);
  tc_fence_before();
  for (int j = 0; j < W / 8; ++j) {
    const int col = W * e.cg + 8 * j + e.cq;
    for (int ee = 0; ee < 2; ++ee) {
      const int row = e.r0 + 8 * ee;
      const float a0 = col <= row ? f.v(ee, j, 0) : 0.f;
      const float a1 = col + 1 <= row ? f.v(ee, j, 1) : 0.f;
      st_shared_u32(dst + swz(row, col), pack2(a0, a1, BF));
    }
  }
}

// M=64 accumulator of D columns at `taddr` -> 16-bit tile at `tile` (KB boxes),
// each value optionally scaled by the 16-bit tile `scale` at the same place
// (which may be `tile` itself) and by a factor per row (rs[0] for row r0,
// rs[1] for row r0 + 8).  Loads go first: the shared-memory accesses are
// ordered asm.
template <int D, bool BF>
__device__ __forceinline__ void frag_to_tile(const Epi &e, uint32_t taddr, uint32_t tile, uint32_t scale,
                                             bool scaled, const float (&rs)[2] = {1.f, 1.f}) {
  constexpr int W = D / kQ;
  Frag<W> f;
  ld_frag(taddr + W * e.cg, f);
  uint32_t sv[W / 4];
  if (scaled)
    for (int j = 0; j < W / 8; ++j)
      for (int ee = 0; ee < 2; ++ee) sv[2 * j + ee] = ld_shared_u32(box_addr(scale, e.r0 + 8 * ee, W * e.cg + 8 * j + e.cq));
  for (int j = 0; j < W / 8; ++j)
    for (int ee = 0; ee < 2; ++ee) {
      float v0 = rs[ee] * f.v(ee, j, 0), v1 = rs[ee] * f.v(ee, j, 1);
      if (scaled) {
        const float2 s2 = unpack2(sv[2 * j + ee], BF);
        v0 *= s2.x;
        v1 *= s2.y;
      }
      st_shared_u32(box_addr(tile, e.r0 + 8 * ee, W * e.cg + 8 * j + e.cq), pack2(v0, v1, BF));
    }
}

// 8x8 16-bit matrices stored transposed from the mma fragment layout (thread t
// holds row t/4, columns 2(t%4) and 2(t%4)+1 of each); thread t gives the
// address of stored row t%8 of matrix t/8 (16 bytes, 16-byte aligned).
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0),
               "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}

// M=128, N=64 accumulator (tensor-memory lane = row m, column n) at column base
// `acc` -> the 16-bit tile of its transpose, [64 rows n x 128 columns m] in two
// swizzled boxes.  Warp (sp, cg) converts lanes 32 sp .. 32 sp + 31 and columns
// 32 cg .. 32 cg + 31: 16x256b loads deliver the 8x8 fragment layout, which
// stmatrix .trans writes out as 16-byte runs of 8 consecutive m for one n.
template <bool BF>
__device__ __forceinline__ void tile_from_transposed(const Epi &e, uint32_t tmem, uint32_t acc, uint32_t tile) {
  const int mat = e.lane >> 3, rho = e.lane & 7;
  for (int hh = 0; hh < 2; ++hh) {  // the two 16-lane halves of this warp's lanes
    uint32_t r[16];  // value (row half ee, column block j, k) at r[4 j + 2 ee + k]
    tmem_ld_16x256b_x4(tmem + e.lane_off + ((uint32_t)(16 * hh) << 16) + acc + 32 * e.cg, r);
    for (int k = 0; k < 4; k += 2) {  // matrices (ee, k), (ee, k + 1) for ee = 0, 1
      const int ee = mat & 1, kk = k + (mat >> 1);
      const int m0 = 32 * e.sp + 16 * hh + 8 * ee, n = 32 * e.cg + 8 * kk + rho;
      const uint32_t addr = tile + (uint32_t)((m0 >> 6) * kTile) + swz(n, m0 & 63);
      auto pk = [&](int i) { return pack2(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), BF); };
      stmatrix_x4_trans(addr, pk(4 * k), pk(4 * k + 2), pk(4 * (k + 1)), pk(4 * (k + 1) + 2));
    }
  }
}

// ------------------------------------------------------ per-step decay --
// Per-step semantics (one decay a per stream, s_t = a s_{t-1} + k_t^T v_t)
// run on the chunk kernels with a row-scaled k tile,
//   K~ = diag(a^(kRef-1-j)) K,   so that q_i . k~_j = a^(i-j) * a^(kRef-1-i) q_i . k_j,
// a factor a^(i+1-kRef) on each output row (or on the rows of dO, which the
// backward then carries as dO^ = diag(a^(i+1-kRef)) g dy), and scalar factors
// on the carried state.  Every factor stays within [a^kRef, a^-kRef].
constexpr int kRef = 32;

// a^e for the per-step decay of a stream (log2 a given)
__device__ __forceinline__ float pow_log2(float l2a, float e) { return exp2f(l2a * e); }

// A factor f as a pair of 16-bit pairs (f_hi, f_lo): f_hi = f rounded,
// f_lo = the remainder f - f_hi rounded, each in both halves.
template <bool BF>
__device__ __forceinline__ uint2 split_factor(float f) {
  const uint32_t hi = pack2(f, f, BF);
  const float r = f - unpack2(hi, BF).x;
  return make_uint2(hi, pack2(r, r, BF));
}

// x * f for a pair of 16-bit values: fma(x, f_hi, x f_lo) rounds once, and
// x f_lo carries the factor's rounding error to within ~2^-16 of x f, so the
// result is x * f rounded to nearest (two packed instructions per pair).
template <bool BF>
__device__ __forceinline__ uint32_t mul2_split(uint32_t x, uint2 f) {
  uint32_t d;
  if constexpr (BF)
    asm("{\n\t.reg .b32 t;\n\tmul.rn.bf16x2 t, %1, %3;\n\tfma.rn.bf16x2 %0, %1, %2, t;\n\t}"
        : "=r"(d) : "r"(x), "r"(f.x), "r"(f.y));
  else
    asm("{\n\t.reg .b32 t;\n\tmul.rn.f16x2 t, %1, %3;\n\tfma.rn.f16x2 %0, %1, %2, t;\n\t}"
        : "=r"(d) : "r"(x), "r"(f.x), "r"(f.y));
  return d;
}

// Scales row `row` of a [64 x 64 KB] 16-bit tile (KB swizzled boxes) in place
// by f (split_factor form).  A row is one 128-byte line of each box whatever
// the swizzle, so a row factor needs no column mapping; lanes holding rows
// that share banks start at different 16-byte chunks so that a warp's
// accesses cover all banks.
template <int KB, bool BF>
__device__ __forceinline__ void scale_tile_row(uint32_t tile, int row, uint2 f) {
  for (int kb = 0; kb < KB; ++kb) {
    const uint32_t line = tile + (uint32_t)(kb * kTile) + (uint32_t)(row * 128);
    uint4 v[8];
    for (int c = 0; c < 8; ++c) v[c] = ld_shared_v4(line + (((c + row) & 7) << 4));
    for (int c = 0; c < 8; ++c)
      st_shared_v4(line + (((c + row) & 7) << 4), mul2_split<BF>(v[c].x, f), mul2_split<BF>(v[c].y, f),
                   mul2_split<BF>(v[c].z, f), mul2_split<BF>(v[c].w, f));
  }
}

// Per-step factor a^(kRef-1-row) of row `row` of the k tile (log2 a given)
template <bool BF>
__device__ __forceinline__ uint2 k_row_factor(float l2a, int row) {
  return split_factor<BF>(pow_log2(l2a, (float)(kRef - 1 - row)));
}

// ------------------------------------------------------------ scheduling --
struct Queue {
  int *ticket;     // tickets taken so far (cleared by the host before the launch)
  int *flags;      // [nranges + 1]: boundary slot publish level (cleared by the host):
                   // 1 = carried state, 2 = also the decay-gradient partial
  float4 *slots;   // [nranges + 1][slot_f4 * kEpi]: carried state at range boundary r
  int slot_f4;     // float4 per thread per slot
  int nstreams, nchunks, nranges;
  float4 *agg;     // [nranges][agg_f4 * kEpi]: aggregates of the publishing pieces, or null
  int agg_f4;
};

struct Piece {
  int stream, c_begin, c_end;  // chunks [c_begin, c_end) of one stream
  int wait_slot;               // boundary slot holding the entry state, or -1 (stream end / start)
  int pub_slot;                // boundary slot for the exit state, or -1
  int range;
  // with precomputed aggregates (long streams) the entry carries of all range
  // boundaries are folded from them before the main kernel starts
  // (entry_fold_kernel), so a piece reads its entry without waiting and
  // publishes no exit carry
  __device__ __forceinline__ bool folds(const Queue &qu) const { return qu.agg != nullptr; }
};

// Range of ticket t: stream-major positions [N t / R, N (t+1) / R), N = streams x chunks.
struct Span {
  int r, s0, c0, s1, c1;  // first piece (s0, [c0, ...)), last piece (s1, [..., c1))
  __device__ __forceinline__ int npieces() const { return s1 - s0 + 1; }
};

__device__ __forceinline__ Span span_of(const Queue &qu, int t, bool reverse) {
  Span sp;
  sp.r = reverse ? qu.nranges - 1 - t : t;
  const long long n = (long long)qu.nstreams * qu.nchunks;
  const long long lo = n * sp.r / qu.nranges, hi = n * (sp.r + 1) / qu.nranges;
  sp.s0 = (int)(lo / qu.nchunks);
  sp.c0 = (int)(lo - (long long)sp.s0 * qu.nchunks);
  sp.s1 = (int)((hi - 1) / qu.nchunks);
  sp.c1 = (int)(hi - (long long)sp.s1 * qu.nchunks);
  return sp;
}

// Piece p (in processing order) of a span.  Forward: last piece, the whole
// streams, first piece.  Reverse: first piece, whole streams, last piece.
__device__ __forceinline__ Piece piece_of(const Queue &qu, const Span &sp, int p, bool reverse) {
  const int m = sp.npieces();
  int s;
  if (reverse || m == 1) s = sp.s0 + p;
  else s = p == 0 ? sp.s1 : (p == m - 1 ? sp.s0 : sp.s0 + p);
  Piece pc;
  pc.stream = s;
  pc.c_begin = s == sp.s0 ? sp.c0 : 0;
  pc.c_end = s == sp.s1 ? sp.c1 : qu.nchunks;
  const int at_begin = pc.c_begin > 0 ? sp.r : -1, at_end = pc.c_end < qu.nchunks ? sp.r + 1 : -1;
  pc.wait_slot = reverse ? at_end : at_begin;
  pc.pub_slot = reverse ? at_begin : at_end;
  pc.range = sp.r;
  return pc;
}

// The piece of a range that publishes a carry (forward: the last piece, when it
// ends mid-stream; reverse: the first, when it starts mid-stream) as its stream
// and chunks [cb, ce); false when the range publishes nothing.  Its aggregate
// is stored at the range's index.
__device__ __forceinline__ bool published_piece(const Queue &qu, const Span &sp, bool reverse, int &s, int &cb,
                                                int &ce) {
  if (!reverse) {
    if (sp.c1 == qu.nchunks) return false;
    s = sp.s1;
    cb = sp.npieces() == 1 ? sp.c0 : 0;
    ce = sp.c1;
  } else {
    if (sp.c0 == 0) return false;
    s = sp.s0;
    cb = sp.c0;
    ce = sp.npieces() == 1 ? sp.c1 : qu.nchunks;
  }
  return true;
}

// Range whose work holds global chunk x = stream * nchunks + chunk.
__device__ __forceinline__ int range_of(const Queue &qu, long long x) {
  const long long n = (long long)qu.nstreams * qu.nchunks;
  int r = (int)(x * qu.nranges / n);
  while (r + 1 < qu.nranges && n * (r + 1) / qu.nranges <= x) ++r;
  while (r > 0 && n * r / qu.nranges > x) --r;
  return r;
}

__device__ __forceinline__ float4 *slot_ptr(const Queue &qu, int slot) {
  return qu.slots + (size_t)slot * qu.slot_f4 * kEpi;
}
__device__ __forceinline__ const float4 *agg_ptr(const Queue &qu, int range) {
  return qu.agg + (size_t)range * qu.agg_f4 * kEpi;
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epilogue: wait until boundary `slot` has been published to `level` (one
// thread spins, bounded), then barrier.  slot < 0: no wait.  Returns false on
// timeout.
__device__ __forceinline__ bool chain_wait(const Epi &e, const Queue &qu, int slot, int32_t *status,
                                           volatile int *abort_flag, int level = 1) {
  __shared__ int ok_flag;
  if (e.et == 0) {
    int ok = 1;
    if (slot >= 0 && ld_acquire(qu.flags + slot) < level) {
      const long long t0 = clock64();
      while (ld_acquire(qu.flags + slot) < level) {
        if (*abort_flag || clock64() - t0 > kWaitCycles) {
          if (status) atomicOr(status, KDA_ERR_DEVICE_TIMEOUT);
          *abort_flag = 1;
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    ok_flag = ok;
  }
  named_bar_sync(1, kEpi);
  return ok_flag != 0;
}

// Epilogue: wait until every boundary slot in [lo, hi) has been published to
// `level`, the slots spread over the epilogue threads so that the waits overlap
// (each bounded), then barrier.  Returns false on timeout.
__device__ __forceinline__ bool shares_wait(const Epi &e, const Queue &qu, int lo, int hi, int32_t *status,
                                            volatile int *abort_flag, int level = 2) {
  __shared__ int all_ok;
  if (e.et == 0) all_ok = 1;
  named_bar_sync(1, kEpi);
  for (int s = lo + e.et; s < hi; s += kEpi) {
    if (ld_acquire(qu.flags + s) >= level) continue;
    const long long t0 = clock64();
    while (ld_acquire(qu.flags + s) < level) {
      if (*abort_flag || clock64() - t0 > kWaitCycles) {
        if (status) atomicOr(status, KDA_ERR_DEVICE_TIMEOUT);
        *abort_flag = 1;
        all_ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  named_bar_sync(1, kEpi);
  return all_ok != 0;
}

// Epilogue: after every thread stored its part of the slot, publish it.  The
// barrier orders the other threads' stores before the publishing thread's fence,
// which is cumulative, so one fence suffices.  The last epilogue thread publishes:
// thread 0 waits for the next piece's boundary flag (chain_wait), so the fence's
// round trip and that flag's overlap instead of adding up.
__device__ __forceinline__ void chain_publish(const Epi &e, const Queue &qu, int slot, int level = 1) {
  named_bar_sync(1, kEpi);
  if (e.et == kEpi - 1) {
    __threadfence();
    atomicExch(qu.flags + slot, level);
  }
}

// Per-step mode: two warps scale the k tile of every stage (warp `half`
// rows 32 half .. 32 half + 31) after its TMA load and before its MMAs (which
// wait on `SCALED + stage`, one arrival per scaler warp).  Units come from
// the same two-entry ring as the other roles; each warp frees a ring entry
// with one arrival.
template <int D, bool BF, int NS>
__device__ void scaler_role(const Queue &qu, bool reverse, int H, const DecaySrc &dec, uint32_t sb,
                            int stage_bytes, uint32_t tile_off, int half, volatile int *ring,
                            volatile int *abort_flag, int32_t *status, uint32_t bar_base, int FULL, int SCALED,
                            int UNIT_FULL0, int UNIT_FREE0) {
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) { return bar_base + 8u * i; };
  int gc = 0;
  for (int i = 0;; ++i) {
    // every lane waits; the warp leaves together if any lane's wait gave up
    if (!__all_sync(0xffffffffu, mbar_wait(bar(UNIT_FULL0 + (i & 1)), (i >> 1) & 1, status, abort_flag))) break;
    const int t = ring[2 * (i & 1)], p = ring[2 * (i & 1) + 1];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(UNIT_FREE0 + (i & 1)));
    if (t >= qu.nranges) break;
    const Piece u = piece_of(qu, span_of(qu, t, reverse), p, reverse);
    const int b = u.stream / H, h = u.stream - b * H;
    const int row = lane + 32 * half;
    const uint2 f = k_row_factor<BF>(log2f(decay_value(dec, b, h, 0)), row);
    bool ok = true;
    for (int k = 0; k < u.c_end - u.c_begin; ++k, ++gc) {
      const int s = gc % NS, use = gc / NS;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(bar(FULL + s), use & 1, status, abort_flag)))) break;
      scale_tile_row<D / 64, BF>(sb + (uint32_t)(s * stage_bytes) + tile_off, row, f);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(SCALED + s));
    }
    if (!ok) break;
  }
}

}  // namespace tc
}  // namespace kda
