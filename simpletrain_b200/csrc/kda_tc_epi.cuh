// Shared pieces of the sm_100a KDA kernels: epilogue thread geometry, tensor-
// memory fragments, the fp32 carry (state) layout, smem tile helpers, direct
// global stores, and the persistent work queue with chained state handoff.
//
// Scheduling.  The scan over T is cut into segments of G chunks.  A "stream"
// is one (batch, head); a unit is (stream, segment).  Persistent CTAs take
// unit tickets from an atomic counter in the workspace; tickets are issued
// segment-major in chain order, so a unit only ever waits for a unit with a
// smaller ticket, which some running CTA holds (no deadlock).  A unit starts
// from the state its chain predecessor published (or from the initial state),
// and publishes its own end state into a two-slot ring per stream.  Every
// wait is bounded.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "kda_internal.h"
#include "tc_common.cuh"

namespace kda {
namespace tc {

constexpr int kTile = 64 * 64 * 2;  // one [64 x 64] 16-bit box, 8 KB
constexpr int kEpi = 256;           // epilogue threads (warps 2..9)
constexpr int kThreads = 320;       // + TMA warp + MMA warp

// ------------------------------------------------------------- geometry --
// Two epilogue warps per TMEM sub-partition: `half` splits the columns.
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

// M=64 accumulator fragment, W columns per half: rows r0 and r0+8,
// columns col0 + 8j + cq + {0,1}; value (e, j, k) at r[4j + 2e + k].
template <int W>
struct Frag {
  uint32_t r[W / 2];
  __device__ __forceinline__ float v(int e, int j, int k) const { return __uint_as_float(r[4 * j + 2 * e + k]); }
};
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
// fp32 D x D carry (state or its gradient / tangent) owned by the epilogue:
//   D=128 (M=128 accumulators): row 32*sp + lane, columns 64*half + [0, 64)
//   D=64  (M=64 accumulators) : rows r0, r0+8, columns 32*half + 8j + cq + k (j < 4)
template <int D>
struct Carry {
  static constexpr int NR = (D == 128) ? 1 : 2;
  static constexpr int NV = (D == 128) ? 64 : 8;
  static constexpr int FLOATS = NR * NV;  // per thread
  float x[NR][NV];
  int row[NR];
  __device__ __forceinline__ int col(const Epi &e, int i) const {
    return (D == 128) ? 64 * e.half + i : 32 * e.half + 8 * (i >> 1) + e.cq + (i & 1);
  }
  __device__ void init_rows(const Epi &e) {
    if (D == 128) row[0] = 32 * e.sp + e.lane;
    else { row[0] = e.r0; row[NR - 1] = e.r0 + 8; }
  }
  __device__ void zero() {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) x[r][i] = 0.f;
  }
  // row-major [D][D] fp32 (user-facing states)
  __device__ void load_rm(const Epi &e, const float *src) {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) x[r][i] = src ? src[(size_t)row[r] * D + col(e, i)] : 0.f;
  }
  __device__ void store_rm(const Epi &e, float *dst) const {
    for (int r = 0; r < NR; ++r)
      for (int i = 0; i < NV; ++i) dst[(size_t)row[r] * D + col(e, i)] = x[r][i];
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
    if (D == 128) {
      uint32_t u[32];
      tmem_ld_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half, u);
      for (int i = 0; i < 32; ++i) x[0][i] = __uint_as_float(u[i]);
      tmem_ld_32x32b_x32(tmem + e.lane_off + acc + 64 * e.half + 32, u);
      for (int i = 0; i < 32; ++i) x[0][32 + i] = __uint_as_float(u[i]);
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
  // 16-bit copy into a state operand (panels of [D rows x 64 cols])
  template <bool BF>
  __device__ void write_operand(const Epi &e, uint32_t base) const {
    if (D == 128) {
      const uint32_t pb = base + (uint32_t)(e.half * D * 128);
      for (int j = 0; j < 8; ++j)
        st_shared_v4(pb + swz(row[0], 8 * j), pack2(x[0][8 * j], x[0][8 * j + 1], BF),
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

// ---------------------------------------------------------- tile helpers --
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
// Ends with tcgen05.fence::before_thread_sync (the accumulator may be reused after a barrier).
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

// Store an M=64 fragment of W = D/2 fp32 values per thread (rows r0, r0+8 of a
// 64-token chunk; columns (D/2)*half + 8j + cq + k) to global memory as 16-bit
// values.  A 4x4 transpose inside each lane quad gives every thread whole
// 16-byte groups of 8 columns.  Rows >= L (ragged last chunk) are skipped.
template <int D, bool BF>
__device__ void store_frag_global(const Epi &e, const float (&val)[D / 2], const View &v, int b, int h, int t0,
                                  int L) {
  constexpr int NJ = D / 16;  // 8-column groups per half
  const int q = e.lane & 3;
  uint32_t p[2][NJ];          // packed pairs: row sel, group j
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    p[0][j] = pack2(val[4 * j], val[4 * j + 1], BF);
    p[1][j] = pack2(val[4 * j + 2], val[4 * j + 3], BF);
  }
#pragma unroll
  for (int ee = 0; ee < 2; ++ee) {
    const int row = e.r0 + 8 * ee;
#pragma unroll
    for (int m = 0; m < NJ / 4; ++m) {
      // after the exchange, w[k] = pair k (columns 2k, 2k+1) of group 4m+q;
      // every index below is a compile-time constant (no local memory)
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int sel = (q - r) & 3;
        uint32_t sv = p[ee][4 * m];
#pragma unroll
        for (int jj = 1; jj < 4; ++jj) sv = (sel == jj) ? p[ee][4 * m + jj] : sv;
        const uint32_t got = __shfl_sync(0xffffffffu, sv, (e.lane & ~3) | ((q + r) & 3));
        const int dst = (q + r) & 3;
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = (dst == k) ? got : w[k];
      }
      if (row < L) {
        const int col = (D / 2) * e.half + 8 * (4 * m + q);
        uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(v.data) + b * v.sb + h * v.sh +
                                               (int64_t)(t0 + row) * v.st + col);
        *dst = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
}

// ------------------------------------------------------------ scheduling --
struct Queue {
  int *ticket;     // tickets taken so far (cleared by the host before the launch)
  int *flags;      // [nstreams]: chain positions published per stream (cleared by the host)
  float4 *slots;   // [nstreams][2][slot_f4 * kEpi]
  int slot_f4;     // float4 per thread per slot
  int nstreams, nseg, G, nchunks, nunits;
};

struct Unit {
  int stream, seg, order, c_begin, c_end;  // chunks [c_begin, c_end)
};

__device__ __forceinline__ Unit decode_unit(const Queue &qu, int t, bool reverse) {
  Unit u;
  u.order = t / qu.nstreams;
  u.stream = t - u.order * qu.nstreams;
  u.seg = reverse ? qu.nseg - 1 - u.order : u.order;
  u.c_begin = u.seg * qu.G;
  u.c_end = min(qu.nchunks, u.c_begin + qu.G);
  return u;
}

__device__ __forceinline__ float4 *slot_ptr(const Queue &qu, int stream, int order) {
  return qu.slots + ((size_t)stream * 2 + (order & 1)) * (size_t)qu.slot_f4 * kEpi;
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epilogue: wait until the chain predecessor of `order` has published (one
// thread spins, bounded), then barrier.  Returns false on timeout.
__device__ __forceinline__ bool chain_wait(const Epi &e, const Queue &qu, int stream, int order, int32_t *status,
                                           volatile int *abort_flag) {
  __shared__ int ok_flag;
  if (e.et == 0) {
    int ok = 1;
    if (order > 0 && ld_acquire(qu.flags + stream) < order) {
      const long long t0 = clock64();
      while (ld_acquire(qu.flags + stream) < order) {
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

// Epilogue: after every thread stored its part of the slot, publish it.
__device__ __forceinline__ void chain_publish(const Epi &e, const Queue &qu, int stream, int order) {
  __threadfence();
  named_bar_sync(1, kEpi);
  if (e.et == 0) atomicExch(qu.flags + stream, order + 1);
}

}  // namespace tc
}  // namespace kda
