// Fused low-bit dequantize + GEMV for B200 (sm_100a): the direct kernel, for
// group-wise formats whose activations fit in one CTA's shared memory.
//
// y[m, n] = fp16( sum_k x[m, k] * (q[n, k] - off[n, k/g]) * scale[n, k/g] ),
// fp32 accumulation, 1 <= M <= 8, the reference packer's format
// (KrishnaI2424/Dequant_Project dequant/packer.py:7-29); it replaces the
// reference kernel kernels/dequant_gemv.cu:144-217 for those shapes.
//
// Design (one CTA per SM, every warp a worker, no copy-issuing warp, no
// shared-memory ring and no mbarriers):
//   * A CTA owns a block of output rows (balanced to within one row), cut
//     into 16-row tiles; a tile's K is cut into groups, padded to a whole
//     number of "units" of gslots = 8 / mp groups (mp = M rounded up to a
//     power of two). The CTA's units, tile by tile, are split into one
//     contiguous range per warp.
//   * Each lane streams its words of the warp's range straight from global
//     memory into its own ring in shared memory (cp.async, 16 bytes per lane
//     per row where the format allows, one commit group per step), R steps
//     ahead of the step it computes: the copies of step s + R are issued right
//     after step s is consumed. (A ring of registers filled by plain loads was
//     measured slower: its loads share a few dependency scoreboards, so the
//     first use of one waits for the later ones.) The first R steps (and their scales/zero-points) are issued
//     before the programmatic-dependent-launch wait: the packed weight is not
//     written by the previous grid, the activations may be.
//   * After the wait, all warps load the activations with plain loads, store
//     them into shared memory in tensor-core B-fragment order and take
//     per-step sums (asymmetric formats), then synchronise once.
//   * Per step: unpack to centred fp16 integers (q - c) with LOP3 + HADD2 /
//     HFMA2 (exact), mma.m16n8k16 with 16 weight rows as the M side and the
//     group slots (times activation rows) as the N side; per unit: scales and
//     zero-points in fp32, sum_k (q - z) x = P - (z - c) * Sx.
//   * Tile results: a warp that covers a whole tile writes y; the tiles at the
//     ends of a warp's range are shared with its neighbours and are summed,
//     after one CTA barrier, in warp order (deterministic).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"
#include "gemv_stream.cuh"

namespace dqg {
namespace direct {

using stream::b_slot;
using stream::kChains;
using stream::lds;
using stream::mma16816;
using stream::quad_sum;
using stream::sts;
using stream::unpack_centered;
using stream::XUnits;

// Non-coherent 4/8/16-byte global load (read-only data for the whole grid).
template <int NB>
__device__ __forceinline__ void ldg_nc(const uint8_t* p, uint32_t* r) {
  if constexpr (NB == 16) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "l"(p));
  } else if constexpr (NB == 8) {
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "l"(p));
  } else {
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r[0]) : "l"(p));
  }
}

__device__ __forceinline__ uint32_t ldg_nc_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Asynchronous global -> shared copy of NB bytes (4, 8 or 16) by this thread;
// src_bytes 0 fills zeros. Completion is tracked per thread by commit groups.
template <int NB>
__device__ __forceinline__ void cp_async(uint32_t dst, const void* src, uint32_t src_bytes) {
  if constexpr (NB == 16)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
                 "r"(src_bytes)
                 : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(dst), "l"(src), "n"(NB),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One step's MMAs: WPL words of rows gid and gid + 8 (already in registers)
// against the activations at px (this lane's fragment column, or a zero
// block when the column is not live).
template <int BITS, int WPL>
__device__ __forceinline__ void mma_regs(const uint32_t* wa, const uint32_t* wb, const uint8_t* px,
                                         float (&D)[kChains<BITS, WPL>][4]) {
  constexpr int NPAIR = 16 / BITS;
  constexpr int NF = NPAIR / 2;
  constexpr int NCH = kChains<BITS, WPL>;
  using XU = XUnits<BITS, WPL>;
  uint32_t bx[WPL * NPAIR];
#pragma unroll
  for (int u = 0; u < XU::NU; ++u) lds<XU::U>(px + u * 4 * XU::U, bx + u * (XU::U / 4));
#pragma unroll
  for (int j = 0; j < WPL; ++j) {
    uint32_t ua[NPAIR], ub[NPAIR];
    unpack_centered<BITS>(wa[j], ua);
    unpack_centered<BITS>(wb[j], ub);
#pragma unroll
    for (int mi = 0; mi < NF; ++mi) {
      const int t = j * NF + mi;
      mma16816(D[t % NCH], ua[2 * mi], ub[2 * mi], ua[2 * mi + 1], ub[2 * mi + 1],
               bx[j * NPAIR + 2 * mi], bx[j * NPAIR + 2 * mi + 1]);
    }
  }
}

template <int BITS, bool SYM, bool INTER, int WPL, int GS>
__global__ void __launch_bounds__(kDirectThreads, 1)
    gemv_direct_kernel(const __grid_constant__ DirectParams p) {
  constexpr int MP = 8 / GS;            // activation-row columns per group slot
  constexpr int PP = 32 / BITS;         // codes per word
  constexpr int NPAIR = PP / 2;         // B registers per word
  constexpr int SC = 4 * WPL * PP;      // codes per step (= the group size)
  constexpr int WB = PP * 2;            // activation bytes per word
  constexpr int STEP_XB = SC * 2;       // activation bytes per step
  constexpr int SW = 4 * WPL;           // words per step and row
  constexpr int NCH = kChains<BITS, WPL>;
  constexpr int R = kDirectRingBytes / (64 * WPL * 4);  // steps in flight per warp
  constexpr int MU = R / GS;            // units per ring block
  constexpr int NMETA = (MP == 1 ? 4 : 2) * (SYM ? 1 : 2);  // u16 values per unit
  constexpr int kRowStepBytes = 4 * SW;  // packed bytes of one step of one row
  constexpr float kBias = static_cast<float>(1 << (BITS - 1));
  using XU = XUnits<BITS, WPL>;
  static_assert(R % GS == 0, "ring blocks hold whole units");

  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2;
  const int c = lane & 3;
  const int G = p.G;
  const int Gp = p.Gp;
  // Rows are balanced across CTAs to within one row; in SwiGLU mode to within
  // one tile (a CTA's rows start on a tile, so that every tile pairs its gate
  // rows 0-7 with its up rows 8-15).
  const int row_begin =
      p.swiglu ? static_cast<int>(static_cast<int64_t>(p.N / kTile) * blockIdx.x / gridDim.x) * kTile
               : static_cast<int>(static_cast<int64_t>(p.N) * blockIdx.x / gridDim.x);
  const int row_end =
      p.swiglu
          ? static_cast<int>(static_cast<int64_t>(p.N / kTile) * (blockIdx.x + 1) / gridDim.x) * kTile
          : static_cast<int>(static_cast<int64_t>(p.N) * (blockIdx.x + 1) / gridDim.x);
  const int T = (row_end - row_begin + kTile - 1) / kTile;
  // Warps split the CTA's steps evenly (to within one step): live steps are
  // [l_lo, l_hi). The loop runs over whole units around them, [s_lo, s_hi);
  // the steps outside the live range load and compute nothing, and their
  // group slots are left out of the unit epilogue.
  const int S_all = T * Gp;
  const int l_lo = static_cast<int>(static_cast<int64_t>(S_all) * warp / kDirectNW);
  const int l_hi = static_cast<int>(static_cast<int64_t>(S_all) * (warp + 1) / kDirectNW);
  const int s_lo = l_lo / GS * GS;
  const int s_hi = l_hi > l_lo ? (l_hi + GS - 1) / GS * GS : s_lo;
  auto live_step = [&](int s) { return s >= l_lo && s < l_hi; };
  const int64_t row_bytes = static_cast<int64_t>(p.K) * BITS / 8;
  const uint8_t* qw = reinterpret_cast<const uint8_t*>(p.qw) + c * (WPL * 4);

  // A cursor over this warp's steps: tile t, (padded) group g.
  struct Cursor {
    int t, g;
  };
  auto cursor_at = [&](int s) { return Cursor{s / Gp, s - (s / Gp) * Gp}; };
  auto advance = [&](Cursor& q) {
    if (++q.g == Gp) {
      q.g = 0;
      ++q.t;
    }
  };

  // Per-warp ring of packed words in shared memory: step base + j lives in
  // slot j; each lane copies (cp.async) and later reads back only its own
  // bytes of rows gid and gid + 8, laid out [slot][row half][lane] so that a
  // warp's reads are contiguous.
  constexpr int kLaneBytes = WPL * 4;
  const uint32_t ring_base =
      smem_u32(smem + p.off_ring) + static_cast<uint32_t>(warp * R * 64 * kLaneBytes);
  auto slot_addr = [&](int j, int half) {
    return ring_base + static_cast<uint32_t>(((j * 2 + half) * 32 + lane) * kLaneBytes);
  };
  uint32_t meta[MU][NMETA];
  // The copy cursor: step s, its tile and group, and this lane's source
  // addresses in rows gid and gid + 8 of the tile, advanced by one group's
  // bytes per step (recomputed only when the tile changes).
  struct LoadCur {
    int s, t, g;
    bool oka, okb;
    const uint8_t* pa;
    const uint8_t* pb;
  };
  auto lc_set = [&](LoadCur& L, int s) {
    L.s = s;
    L.t = s / Gp;
    L.g = s - L.t * Gp;
    const int ra = row_begin + L.t * kTile + gid;
    L.oka = ra < row_end;
    L.okb = ra + 8 < row_end;
    const uint8_t* g0 = qw + static_cast<int64_t>(L.g) * kRowStepBytes;
    L.pa = g0 + (L.oka ? ra : row_begin) * row_bytes;
    L.pb = g0 + (L.okb ? ra + 8 : row_begin) * row_bytes;
  };
  auto lc_next = [&](LoadCur& L) {
    ++L.s;
    L.pa += kRowStepBytes;
    L.pb += kRowStepBytes;
    if (++L.g == Gp) lc_set(L, L.s);
  };
  // Copies of the cursor's step into the ring slot at byte address `slot`
  // (zero fill where the step is outside this warp's live range, past the
  // last group or past the CTA's rows), one commit group per step.
  auto issue = [&](uint32_t slot, const LoadCur& L) {
    const bool ok = live_step(L.s) && L.g < G;
    const bool oka = ok && L.oka, okb = ok && L.okb;
    cp_async<kLaneBytes>(slot, oka ? L.pa : qw, oka ? kLaneBytes : 0u);
    cp_async<kLaneBytes>(slot + 32 * kLaneBytes, okb ? L.pb : qw, okb ? kLaneBytes : 0u);
    cp_async_commit();
  };
  // Scales (and zero-points) of the unit that starts at cursor q: for
  // M = 1 the lane's two columns are groups 2c and 2c + 1 of the unit,
  // otherwise both columns are the unit's group 2c / mp (two activation rows).
  auto load_meta = [&](uint32_t* dst, Cursor q, bool live) {
    const int ra = row_begin + q.t * kTile + gid;
#pragma unroll
    for (int i = 0; i < NMETA; ++i) dst[i] = 0u;
    if (!live) return;
    constexpr int NG = MP == 1 ? 2 : 1;
#pragma unroll
    for (int gi = 0; gi < NG; ++gi) {
      const int g = q.g + (MP == 1 ? 2 * c + gi : (2 * c) / MP);
      if (g >= G) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = ra + 8 * h;
        if (row >= row_end) continue;
        const int64_t e = static_cast<int64_t>(row) * G + g;
        dst[gi * 2 + h] = ldg_nc_u16(p.scales + e);
        if constexpr (!SYM) dst[NG * 2 + gi * 2 + h] = ldg_nc_u16(p.zeros + e);
      }
    }
  };

  // Issue the first ring: weights and metadata are not written by the
  // previous grid (with p.prefetch), so this runs before its dependency wait.
  if (!p.prefetch) pdl_wait_prior_grid();
  LoadCur lq;
  lc_set(lq, s_lo);
#pragma unroll
  for (int j = 0; j < R; ++j) {
    if (j % GS == 0) load_meta(meta[j / GS], Cursor{lq.t, lq.g}, s_lo + j < s_hi);
    issue(slot_addr(j, 0), lq);
    lc_next(lq);
  }
  if (threadIdx.x == 0) pdl_launch_dependents();

  // Activations: after this thread's dependency wait, plain loads into
  // B-fragment order with per-step (= per-group) sums for asymmetric formats.
  float* sx = reinterpret_cast<float*>(smem + p.off_sx);
  for (int i = threadIdx.x; i < STEP_XB / 16; i += kDirectThreads)
    reinterpret_cast<uint4*>(smem + p.off_zero)[i] = make_uint4(0u, 0u, 0u, 0u);
  pdl_wait_prior_grid();
  {
    constexpr int kCT = kDirectThreads;
    constexpr int kU = 128 / WB;
    const int wpr = p.K / PP;
    const int wtot = p.M * wpr;
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x);
    const int64_t xrow_bytes = static_cast<int64_t>(p.K) * 2;
    const uint32_t wmagic = 0xFFFFFFFFu / static_cast<uint32_t>(wpr) + 1u;
    for (int w0 = warp * 32; w0 < wtot; w0 += kU * kCT) {
      uint32_t v[kU][NPAIR];
      int mrow[kU], wcol[kU];
#pragma unroll
      for (int uu = 0; uu < kU; ++uu) {
        const int wf = w0 + uu * kCT + lane;
        const int m = static_cast<int>(__umulhi(static_cast<uint32_t>(wf), wmagic));
        mrow[uu] = m;
        wcol[uu] = wf - m * wpr;
        if (wf < wtot) {
          stream::ldg_l2<WB>(xg + m * xrow_bytes + wcol[uu] * WB, v[uu]);
        } else {
#pragma unroll
          for (int r = 0; r < NPAIR; ++r) v[uu][r] = 0u;
        }
      }
#pragma unroll
      for (int uu = 0; uu < kU; ++uu) {
        if (w0 + uu * kCT + lane >= wtot) continue;
        uint32_t o[NPAIR];
#pragma unroll
        for (int r = 0; r < NPAIR; ++r) {
          const int lo = slot_logical(BITS, INTER, b_slot(BITS, r, 0));
          const int hi = slot_logical(BITS, INTER, b_slot(BITS, r, 1));
          o[r] = prmt(v[uu][lo >> 1], v[uu][hi >> 1],
                      ((lo & 1) ? 0x32u : 0x10u) | ((hi & 1) ? 0x7600u : 0x5400u));
        }
        const int wi = wcol[uu];
        const int q = wi & (SW - 1);
        const int cc = q / WPL;
        const int j = q - cc * WPL;
        constexpr int PB = WB < XU::U ? WB : XU::U;
        uint8_t* sbase = smem + p.off_x + mrow[uu] * p.xp + (wi / SW) * STEP_XB + cc * XU::U;
#pragma unroll
        for (int pc = 0; pc < WB / PB; ++pc) {
          const int lb = j * WB + pc * PB;
          sts<PB>(sbase + (lb / XU::U) * 4 * XU::U + (lb % XU::U), o + pc * (PB / 4));
        }
      }
      if constexpr (!SYM) {
        float sum[kU];
#pragma unroll
        for (int uu = 0; uu < kU; ++uu) sum[uu] = quad_sum<NPAIR>(v[uu]);
#pragma unroll
        for (int off = SW / 2; off >= 4; off >>= 1)
#pragma unroll
          for (int uu = 0; uu < kU; ++uu) sum[uu] += __shfl_xor_sync(0xffffffffu, sum[uu], off);
#pragma unroll
        for (int uu = 0; uu < kU; ++uu) {
          if ((lane & (SW - 1)) == 0 && w0 + uu * kCT + lane < wtot)
            sx[mrow[uu] * G + wcol[uu] / SW] = sum[uu];
        }
      }
    }
  }
  __syncthreads();

  // Row-parallel mode: this rank's fp32 partial of y goes to its exchange
  // buffer (parity of this call's epoch) instead of y.
  const bool ar = p.ar_world > 1;
  const uint32_t ep = ar ? *reinterpret_cast<volatile const uint32_t*>(p.ar_ctl) + 1u : 0u;
  // Parity halves are a fixed cap apart, so that calls of different shapes
  // never write into the half a slower peer may still read.
  const int64_t ar_par = static_cast<int64_t>(ep & 1u) * p.ar_cap;
  // SwiGLU mode: act[xrow, orow] from the gate and up sums, each rounded to
  // fp16 as the GEMV's output is, then silu_mul_kernel's arithmetic
  // (decode_ops.cu): fp16(g / (1 + exp(-g)) * u) in fp32.
  auto store_swiglu = [&](int xrow, int orow, float gs, float us) {
    const float g = __half2float(__float2half_rn(gs));
    const float u = __half2float(__float2half_rn(us));
    const float sg = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
    p.y[static_cast<int64_t>(xrow) * (p.N / 2) + orow] =
        __half_as_ushort(__float2half_rn(__fmul_rn(sg, u)));
  };
  auto store_out = [&](int xrow, int row, float v) {
    const int64_t e = static_cast<int64_t>(xrow) * p.N + row;
    if (ar)
      reinterpret_cast<float*>(p.ar_data[p.ar_rank])[ar_par + e] = v;
    else
      p.y[e] = __half_as_ushort(__float2half_rn(v));
  };

  // ---------------------------------------------------------------- main loop
  const int my_slot = gid / MP;
  const int my_xrow = gid - my_slot * MP;
  const bool x_ok = my_xrow < p.M;
  const uint8_t* xrow_base = smem + p.off_x + (x_ok ? my_xrow : 0) * p.xp + c * XU::U;
  const uint8_t* zero_base = smem + p.off_zero + c * XU::U;
  float* red = reinterpret_cast<float*>(smem + p.off_red) + warp * (2 * kTile * 8);
  int* tiles = reinterpret_cast<int*>(smem + p.off_tiles);  // [warp][2]: tiles held in red
  float D[NCH][4];
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
    for (int e = 0; e < 4; ++e) D[ch][e] = 0.f;
  auto h2f = [](uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v))); };

  // Unit epilogue: scales and zero-points of the unit's groups (from g0)
  // applied in fp32 to the chains' sums, added into acc.
  auto epilogue = [&](const uint32_t* md, int g0, int tile_step) {
    float P[4];
    stream::combine<NCH>(D, P);
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int e = 0; e < 4; ++e) D[ch][e] = 0.f;
    bool ev[4];
    float sv[4], zv[4], sxv[4];
    if constexpr (MP >= 2) {
      const int slot = (2 * c) / MP;
      const int xr0 = 2 * c - slot * MP;
      const int g = g0 + slot;
      const bool gok = g < G && live_step(tile_step + g);
      ev[0] = ev[2] = gok && xr0 < p.M;
      ev[1] = ev[3] = gok && xr0 + 1 < p.M;
      sv[0] = sv[1] = h2f(md[0]);
      sv[2] = sv[3] = h2f(md[1]);
      if constexpr (!SYM) {
        zv[0] = zv[1] = h2f(md[2]);
        zv[2] = zv[3] = h2f(md[3]);
        const int gg = gok ? g : 0;
        sxv[0] = sxv[2] = sx[(ev[0] ? xr0 : 0) * G + gg];
        sxv[1] = sxv[3] = sx[(ev[1] ? xr0 + 1 : 0) * G + gg];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int gi = e & 1, h = e >> 1;
        const int g = g0 + 2 * c + gi;
        ev[e] = g < G && live_step(tile_step + g);
        sv[e] = h2f(md[gi * 2 + h]);
        if constexpr (!SYM) {
          zv[e] = h2f(md[4 + gi * 2 + h]);
          sxv[e] = sx[ev[e] ? g : 0];
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (ev[e]) {
        float t = P[e];
        if constexpr (!SYM) t = fmaf(-(zv[e] - kBias), sxv[e], t);
        acc[e] = fmaf(sv[e], t, acc[e]);
      }
    }
  };

  // Tile end: columns of one activation row summed across lanes; a tile this
  // warp covered whole goes to y, a shared one to this warp's slot in red.
  const int first_tile = s_lo / Gp;
  auto tile_flush = [&](int t) {
    float a[4] = {acc[0], acc[1], acc[2], acc[3]};
    if constexpr (MP == 1) {
      a[0] += a[1];
      a[2] += a[3];
    }
    if constexpr (MP <= 2) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a[e] += __shfl_xor_sync(0xffffffffu, a[e], 1);
        a[e] += __shfl_xor_sync(0xffffffffu, a[e], 2);
      }
    } else if constexpr (MP == 4) {
#pragma unroll
      for (int e = 0; e < 4; ++e) a[e] += __shfl_xor_sync(0xffffffffu, a[e], 2);
    }
    constexpr int cmask = MP <= 2 ? 3 : (MP == 4 ? 2 : 0);
    const bool whole = t * Gp >= l_lo && (t + 1) * Gp <= l_hi;
    const int r0 = row_begin + t * kTile;
    const int slot = t == first_tile ? 0 : 1;
    float* rs = red + slot * (kTile * 8);
    if ((c & cmask) == 0) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (MP == 1 && (e & 1)) continue;
        const int row = gid + 8 * (e >> 1);
        const int xrow = (2 * c + (e & 1)) & (MP - 1);
        if (xrow < p.M) {
          if (whole) {
            if (p.swiglu) {
              if ((e >> 1) == 0) store_swiglu(xrow, (r0 >> 1) + gid, a[e], a[e + 2]);
            } else if (r0 + row < row_end) {
              store_out(xrow, r0 + row, a[e]);
            }
          } else {
            rs[row * 8 + xrow] = a[e];
          }
        }
      }
    }
    if (!whole && lane == 0) tiles[warp * 2 + slot] = t;
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  };

  if (lane == 0) tiles[warp * 2] = tiles[warp * 2 + 1] = -1;
  __syncwarp();
  const uint32_t smem_base = smem_u32(smem);
  constexpr uint32_t kSlotBytes = 64 * kLaneBytes;  // one step's ring slot, both row halves
  if constexpr (GS >= 4) {
    // Batch of at most two activation rows (four or eight group slots): a
    // unit's steps are unrolled with the ring slot of the unit computed
    // once, and each unit's scales/zero-points are loaded one unit ahead
    // (the unit after next, into `mnxt`, while this one is computed).
    uint32_t mnxt[NMETA];
    if constexpr (MU >= 2) {
#pragma unroll
      for (int i = 0; i < NMETA; ++i) mnxt[i] = meta[1][i];
    } else {
      load_meta(mnxt, cursor_at(s_lo + GS), s_lo + GS < s_hi);
    }
    int t = s_lo / Gp, g0 = s_lo - (s_lo / Gp) * Gp;
    int ru = 0;  // ring position of the unit, in units
    for (int u0 = s_lo; u0 < s_hi; u0 += GS) {
      const uint32_t ring_u = ring_base + lane * kLaneBytes + ru * GS * kSlotBytes;
#pragma unroll
      for (int jj = 0; jj < GS; ++jj) {
        const uint32_t sa = ring_u + jj * kSlotBytes;
        cp_async_wait<R - 1>();  // step u0 + jj has landed (this lane's copies)
        if (g0 + jj < G && live_step(u0 + jj)) {
          uint32_t w[2 * WPL];
          lds<kLaneBytes>(smem + (sa - smem_base), w);
          lds<kLaneBytes>(smem + (sa + 32 * kLaneBytes - smem_base), w + WPL);
          const bool live = x_ok && my_slot == jj;
          mma_regs<BITS, WPL>(w, w + WPL, live ? xrow_base + (g0 + jj) * STEP_XB : zero_base, D);
        }
        issue(sa, lq);  // step u0 + jj + R into the slot just read
        lc_next(lq);
      }
      epilogue(meta[0], g0, t * Gp);
#pragma unroll
      for (int i = 0; i < NMETA; ++i) meta[0][i] = mnxt[i];
      const int un = u0 + 2 * GS;
      if (un < s_hi) load_meta(mnxt, cursor_at(un), true);
      if (g0 + GS == Gp || u0 + GS == s_hi) tile_flush(t);
      g0 += GS;
      if (g0 == Gp) {
        g0 = 0;
        ++t;
      }
      ru = ru + 1 == MU ? 0 : ru + 1;
    }
  } else {
    Cursor cq = cursor_at(s_lo);      // the step computed
    Cursor mq = cursor_at(s_lo + R);  // start of the unit whose metadata is loaded next
    for (int base = s_lo; base < s_hi; base += R) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int s = base + j;
        if (s < s_hi) {
          cp_async_wait<R - 1>();  // step s has landed (this lane's copies)
          if (cq.g < G && live_step(s)) {
            uint32_t w[2 * WPL];
            lds<kLaneBytes>(smem + (slot_addr(j, 0) - smem_base), w);
            lds<kLaneBytes>(smem + (slot_addr(j, 1) - smem_base), w + WPL);
            const bool live = x_ok && my_slot == j % GS;
            mma_regs<BITS, WPL>(w, w + WPL, live ? xrow_base + cq.g * STEP_XB : zero_base, D);
          }
          issue(slot_addr(j, 0), lq);
          lc_next(lq);
          if (j % GS == GS - 1) {
            epilogue(meta[j / GS], cq.g - (GS - 1), cq.t * Gp);
            load_meta(meta[j / GS], mq, s + 1 - GS + R < s_hi);
#pragma unroll
            for (int k2 = 0; k2 < GS; ++k2) advance(mq);
            if (cq.g == Gp - 1 || s == s_hi - 1) tile_flush(cq.t);
          }
          advance(cq);
        }
      }
    }
  }

  // Tiles shared between warps: the lowest warp holding a tile adds every
  // holder's partial in warp order and writes y. The holder table is read
  // into registers once and the loops over warps are unrolled, so that the
  // partials' shared-memory loads are independent of one another.
  __syncthreads();
  int tl[2 * kDirectNW];
#pragma unroll
  for (int i = 0; i < 2 * kDirectNW; ++i) tl[i] = tiles[i];
  const float* red_all = reinterpret_cast<const float*>(smem + p.off_red);
#pragma unroll
  for (int slot = 0; slot < 2; ++slot) {
    const int t = tiles[warp * 2 + slot];
    if (t < 0) continue;
    bool lowest = true;
#pragma unroll
    for (int w = 0; w < kDirectNW; ++w)
      if (w < warp) lowest = lowest && tl[2 * w] != t && tl[2 * w + 1] != t;
    if (!lowest) continue;
    const int r0 = row_begin + t * kTile;
    auto tile_sum = [&](int row, int xrow) {
      float part[2 * kDirectNW];
#pragma unroll
      for (int w = 0; w < kDirectNW; ++w) {
        const float* rw = red_all + w * (2 * kTile * 8) + row * 8 + xrow;
        part[2 * w] = w >= warp && tl[2 * w] == t ? rw[0] : 0.f;
        part[2 * w + 1] = w >= warp && tl[2 * w + 1] == t ? rw[kTile * 8] : 0.f;
      }
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 2 * kDirectNW; ++i) sum += part[i];
      return sum;
    };
    if (p.swiglu) {
      for (int idx = lane; idx < (kTile / 2) * p.M; idx += 32) {
        const int row = idx / p.M, xrow = idx - (idx / p.M) * p.M;
        store_swiglu(xrow, (r0 >> 1) + row, tile_sum(row, xrow), tile_sum(row + 8, xrow));
      }
    } else {
      for (int idx = lane; idx < kTile * p.M; idx += 32) {
        const int row = idx / p.M, xrow = idx - (idx / p.M) * p.M;
        const float sum = tile_sum(row, xrow);
        if (r0 + row < row_end) store_out(xrow, r0 + row, sum);
      }
    }
  }
  if (!ar) return;

  // Row-parallel exchange: once this CTA's rows are in its exchange buffer,
  // raise its flag on every rank, wait (bounded) for every rank's flag of
  // this CTA, and sum the ranks' partials of these rows in rank order.
  __syncthreads();
  if (threadIdx.x < p.ar_world) {
    fence_acq_rel_sys();
    st_relaxed_sys(reinterpret_cast<uint32_t*>(p.ar_flags[threadIdx.x]) +
                       blockIdx.x * p.ar_world + p.ar_rank,
                   ep);
  }
  bool ok = true;
  if (threadIdx.x < p.ar_world) {
    ok = wait_flag_sys(reinterpret_cast<const uint32_t*>(p.ar_flags[p.ar_rank]) +
                           blockIdx.x * p.ar_world + threadIdx.x,
                       ep, p.ar_wait_ns);
    fence_acq_rel_sys();
  }
  ok = __syncthreads_and(ok);
  const int rows = row_end - row_begin;
  if (ok) {
    for (int idx = threadIdx.x; idx < rows * p.M; idx += kDirectThreads) {
      const int xrow = idx / rows, row = row_begin + idx - (idx / rows) * rows;
      const int64_t e = ar_par + static_cast<int64_t>(xrow) * p.N + row;
      float sum = 0.f;
      for (int r = 0; r < p.ar_world; ++r)
        sum += __ldcg(reinterpret_cast<const float*>(p.ar_data[r]) + e);
      p.y[static_cast<int64_t>(xrow) * p.N + row] = __half_as_ushort(__float2half_rn(sum));
    }
  }
  // The last CTA of the call advances the epoch.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(p.ar_ctl + 1, 1u);
    if (t == gridDim.x - 1) {
      p.ar_ctl[1] = 0u;
      __threadfence();
      atomicExch(p.ar_ctl, ep);
    }
  }
}

}  // namespace direct
}  // namespace dqg

namespace dqg {
namespace direct {

template <int BITS, bool SYM, bool INTER, int WPL, int GS>
cudaError_t launch_one(const DirectParams& p, int grid, int smem, cudaStream_t stream) {
  auto kern = gemv_direct_kernel<BITS, SYM, INTER, WPL, GS>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDirectMaxSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDirectThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, bool SYM, bool INTER, int WPL>
cudaError_t launch_gs(int gs, const DirectParams& p, int grid, int smem, cudaStream_t stream) {
  switch (gs) {
    case 1: return launch_one<BITS, SYM, INTER, WPL, 1>(p, grid, smem, stream);
    case 2: return launch_one<BITS, SYM, INTER, WPL, 2>(p, grid, smem, stream);
    case 4: return launch_one<BITS, SYM, INTER, WPL, 4>(p, grid, smem, stream);
    case 8: return launch_one<BITS, SYM, INTER, WPL, 8>(p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

// All variants of one bit width (one translation unit per width).
template <int BITS>
cudaError_t launch_bits(int wpl, int gs, bool sym, bool inter, const DirectParams& p, int grid,
                        int smem, cudaStream_t stream) {
#define DQG_DIRECT_WPL(S, I)                                                 \
  switch (wpl) {                                                             \
    case 4: return launch_gs<BITS, S, I, 4>(gs, p, grid, smem, stream);      \
    case 2: return launch_gs<BITS, S, I, 2>(gs, p, grid, smem, stream);      \
    default: return launch_gs<BITS, S, I, 1>(gs, p, grid, smem, stream);     \
  }
  if (sym && inter) { DQG_DIRECT_WPL(true, true) }
  if (sym) { DQG_DIRECT_WPL(true, false) }
  if (inter) { DQG_DIRECT_WPL(false, true) }
  DQG_DIRECT_WPL(false, false)
#undef DQG_DIRECT_WPL
}

}  // namespace direct
}  // namespace dqg
