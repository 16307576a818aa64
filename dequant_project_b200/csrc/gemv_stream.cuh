// Fused low-bit dequantize + GEMV for B200 (sm_100a): the streaming kernel.
//
// y[m, n] = fp16( sum_k x[m, k] * (q[n, k] - off[n, k/g]) * scale[n, k/g] ),
// fp32 accumulation, 1 <= M <= 8, packed format of the reference packer
// (KrishnaI2424/Dequant_Project dequant/packer.py:7-29). It replaces the
// reference kernel kernels/dequant_gemv.cu:144-217 whenever the activations
// fit in shared memory.
//
// Design (one CTA per SM; rows balanced across CTAs to within one row):
//   * warp 0 (producer) streams the CTA's rows as (16-row tile, K slab)
//     stages into a ring of shared-memory slots: one bulk copy
//     (cp.async.bulk, no multicast) per packed row segment, plus each tile's
//     scales/zero-points as one contiguous span. The first ring is issued at
//     once, before the programmatic-dependent-launch wait (weights are not
//     written by the previous grid), so it streams while that grid drains.
//   * warps 2.. (consumers) load the activations with plain global loads
//     after the dependent-launch wait (off the bulk-copy queue, so they never
//     wait behind the weight ring), store them into shared memory in the
//     tensor-core B-fragment order and take per-step sums; then, per stage,
//     unpack codes in registers and run mma.m16n8k16 (fp16 x fp16 -> fp32)
//     with 16 weight rows as the M side.
//   * warp 1 (reducer) sums the consumer warps' partials of each tile in a
//     fixed order and writes y.
//
// Exact unpack with compile-time constants: a code pair at bit position p of
// the two 16-bit halves (p + bits <= 10) is dropped into the mantissa of fp16
// 1024 by one LOP3 and brought to (q - c), c = 2^(bits - 1), by one HADD2
// (p = 0) or one HFMA2 with the exact scale 2^-p (p > 0). Centring keeps the
// tensor-core partial sums as small as in a dequantized product. The offset is
// applied per group in fp32 through the group's activation sum:
//   sum_k (q - z) x = P - (z - c) * Sx,   P = sum_k (q - c) x,   Sx = sum_k x,
// so any zero-point (fractional, out of range) is handled the same way, and the
// scale multiplies the group's result in fp32 (as the reference kernel does per
// chunk, dequant_gemv.cu:199-200).
//
// Group slots: the MMA's N=8 side holds mp activation rows (mp = M rounded up
// to a power of two) times 8/mp consecutive groups; a lane's B fragment is
// zero unless its column's group is the one being streamed, so one MMA chain
// collects up to 8 group partials at once and their scale/offset work is
// spread over all lanes (for M=1 this is 8x fewer scale instructions than one
// group per chain).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {
namespace stream {

// B-fragment register r of a word holds the activations of slots
// (b_slot(r, 0), b_slot(r, 1)); unpack_sub produces the code pairs of the same
// slots in the same order.
__host__ __device__ constexpr int b_slot(int bits, int r, int hi) {
  if (bits == 4) return (r == 0 ? 0 : r == 1 ? 2 : r == 2 ? 1 : 3) + (hi ? 4 : 0);
  if (bits == 2) return (r >> 1) + ((r & 1) ? 4 : 0) + (hi ? 8 : 0);
  return r + (hi ? 2 : 0);
}

// Code pairs of one word as centred fp16 integers (q - c), c = 2^(bits - 1),
// in b_slot order: one LOP3 drops a pair at bit position p into the mantissa
// of 1024 (1024 + q * 2^p, exactly, p + bits <= 10) and one HADD2 (p = 0) or
// HFMA2 with 2^-p and -(1024 * 2^-p + c) (p > 0) leaves q - c, exactly (every
// intermediate is an integer or a power-of-two multiple below 2^11).
template <int BITS>
__device__ __forceinline__ void unpack_centered(uint32_t w, uint32_t* pa) {
  constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
  if constexpr (BITS == 4) {
    const uint32_t w8 = prmt(w, 0u, 0x4341u);  // (w >> 8) & 0x00FF00FF
    pa[0] = hadd2_u32(lop3_and_or(w, 0x000F000Fu, kMagic), 0xE408E408u);   // slots 0, 4: -1032
    pa[1] = hadd2_u32(lop3_and_or(w8, 0x000F000Fu, kMagic), 0xE408E408u);  // slots 2, 6
    pa[2] = hfma2_u32(lop3_and_or(w, 0x00F000F0u, kMagic), 0x2C002C00u,
                      0xD480D480u);                                         // slots 1, 5: /16 - 72
    pa[3] = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, kMagic), 0x2C002C00u,
                      0xD480D480u);                                         // slots 3, 7
  } else if constexpr (BITS == 2) {
    const uint32_t w8 = prmt(w, 0u, 0x4341u);
    // p = 2f: 2^-2f and -(1024 * 2^-2f + 2).
    constexpr uint32_t kS[4] = {0x3C003C00u, 0x34003400u, 0x2C002C00u, 0x24002400u};
    constexpr uint32_t kB[4] = {0xE402E402u, 0xDC08DC08u, 0xD420D420u, 0xCC80CC80u};
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      if (f == 0) {
        pa[0] = hadd2_u32(lop3_and_or(w, 0x00030003u, kMagic), kB[0]);   // slots 0, 8
        pa[1] = hadd2_u32(lop3_and_or(w8, 0x00030003u, kMagic), kB[0]);  // slots 4, 12
      } else {
        pa[2 * f] = hfma2_u32(lop3_and_or(w, 0x00030003u << (2 * f), kMagic), kS[f], kB[f]);
        pa[2 * f + 1] = hfma2_u32(lop3_and_or(w8, 0x00030003u << (2 * f), kMagic), kS[f], kB[f]);
      }
    }
  } else {
    pa[0] = hadd2_u32(prmt(w, kMagic, 0x7250u), 0xE480E480u);  // slots 0, 2
    pa[1] = hadd2_u32(prmt(w, kMagic, 0x7351u), 0xE480E480u);  // slots 1, 3
  }
}

// Not volatile: a pure function of its operands, so the compiler may schedule
// loads and unpacking of later steps around it.
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same MMA with a zero accumulator input (the first MMA of a chain).
__device__ __forceinline__ void mma16816_first(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Total of the fp16 values in one word's registers summed over the four lanes
// of a quad (lanes 4g .. 4g + 3), by MMAs against a matrix of ones: the
// registers are taken as A fragment registers, whose rows g and g + 8 collect
// the quad's a0/a2 and a1/a3 halves, so d0 + d2 (every column is the same) is
// the quad's total. The products are exact and the tensor core accumulates in
// fp32; one MMA replaces eight conversions, seven adds and two shuffle levels
// per word.
template <int NREG>
__device__ __forceinline__ float quad_sum(const uint32_t* v) {
  constexpr uint32_t kOnes = 0x3C003C00u;
  float d[4];
  if constexpr (NREG == 2) {
    mma16816_first(d, v[0], v[1], 0u, 0u, kOnes, kOnes);
  } else {
    mma16816_first(d, v[0], v[1], v[2], v[3], kOnes, kOnes);
#pragma unroll
    for (int i = 4; i < NREG; i += 4) mma16816(d, v[i], v[i + 1], v[i + 2], v[i + 3], kOnes, kOnes);
  }
  return d[0] + d[2];
}

template <int NB>
__device__ __forceinline__ void lds(const uint8_t* p, uint32_t* r) {
  if constexpr (NB == 4) {
    r[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (NB == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    r[0] = v.x;
    r[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + 16 * i);
      r[4 * i + 0] = v.x;
      r[4 * i + 1] = v.y;
      r[4 * i + 2] = v.z;
      r[4 * i + 3] = v.w;
    }
  }
}

// NB bytes (8, 16 or 32) from global memory into registers, cached in L2 only
// (never a stale L1 line of data the previous grid wrote).
template <int NB>
__device__ __forceinline__ void ldg_l2(const uint8_t* p, uint32_t* r) {
  if constexpr (NB == 8) {
    asm volatile("ld.global.cg.v2.u32 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "l"(p));
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i)
      asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(r[4 * i]), "=r"(r[4 * i + 1]), "=r"(r[4 * i + 2]), "=r"(r[4 * i + 3])
                   : "l"(p + 16 * i));
  }
}

template <int NB>
__device__ __forceinline__ void sts(uint8_t* p, const uint32_t* r) {
  if constexpr (NB == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(r[0], r[1]);
  } else {
#pragma unroll
    for (int i = 0; i < NB / 16; ++i)
      *reinterpret_cast<uint4*>(p + 16 * i) =
          make_uint4(r[4 * i + 0], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
  }
}

// Shared-memory layout of a step's activations (B-fragment order): lane c's
// LXB bytes are cut into U-byte units; unit u of lane c sits at u * 4U + c * U,
// so the four lanes of a fragment row read one contiguous 4U-byte run.
template <int BITS, int WPL>
struct XUnits {
  static constexpr int WB = 64 / BITS;          // activation bytes per word
  static constexpr int LXB = WPL * WB;          // per lane per step
  static constexpr int U = LXB >= 16 ? 16 : LXB;
  static constexpr int NU = LXB / U;
};

// Accumulator chains per lane: MMA t of a step goes to chain t % NCH (two
// independent chains hide the MMA latency).
template <int BITS, int WPL>
constexpr int kChains = (WPL * (16 / BITS) / 2) >= 2 ? 2 : 1;

// One step of one lane: WPL words of rows gid and gid + 8 and their
// activations (px points at the step's activations when this lane's fragment
// column is live, else at a zero block), NPAIR/2 MMAs per word. FIRST: the
// chains start here (their first MMA takes a zero accumulator).
template <int BITS, int WPL, bool FIRST>
__device__ __forceinline__ void mma_step(const uint8_t* pa, const uint8_t* pb, const uint8_t* px,
                                         float (&D)[kChains<BITS, WPL>][4]) {
  constexpr int NPAIR = 16 / BITS;
  constexpr int NF = NPAIR / 2;
  constexpr int NCH = kChains<BITS, WPL>;
  using XU = XUnits<BITS, WPL>;
  uint32_t wa[WPL], wb[WPL];
  lds<WPL * 4>(pa, wa);
  lds<WPL * 4>(pb, wb);
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
      if (FIRST && t < NCH)
        mma16816_first(D[t % NCH], ua[2 * mi], ub[2 * mi], ua[2 * mi + 1], ub[2 * mi + 1],
                       bx[j * NPAIR + 2 * mi], bx[j * NPAIR + 2 * mi + 1]);
      else
        mma16816(D[t % NCH], ua[2 * mi], ub[2 * mi], ua[2 * mi + 1], ub[2 * mi + 1],
                 bx[j * NPAIR + 2 * mi], bx[j * NPAIR + 2 * mi + 1]);
    }
  }
}

// sum_k (q - c) x of each accumulator element: the chains added in order.
template <int NCH>
__device__ __forceinline__ void combine(const float (&D)[NCH][4], float* P) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float v = D[0][e];
#pragma unroll
    for (int ch = 1; ch < NCH; ++ch) v += D[ch][e];
    P[e] = v;
  }
}

template <int BITS, bool SYM, bool INTER, int WPL, int GS>
__global__ void __launch_bounds__(kStreamThreads, kStreamMinBlocks)
    gemv_stream_kernel(const __grid_constant__ StreamParams p) {
  constexpr bool GROUPED = GS > 0;
  constexpr int MP = GROUPED ? 8 / GS : 8;  // activation-row columns per group slot
  constexpr int PP = 32 / BITS;         // codes per word
  constexpr int NPAIR = PP / 2;         // B registers per word
  constexpr int SC = 4 * WPL * PP;      // codes per step
  constexpr int WB = PP * 2;            // activation bytes per word
  constexpr int STEP_XB = SC * 2;       // activation bytes per step
  constexpr int SW = 4 * WPL;           // words per step
  constexpr int NCH = kChains<BITS, WPL>;  // accumulator chains
  constexpr float kBias = static_cast<float>(1 << (BITS - 1));

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + kMaxStages;
  uint64_t* meta_full = empty + kMaxStages;     // [kStreamMaxMeta]
  uint64_t* red_full = meta_full + kStreamMaxMeta;  // [kStreamNRB]
  uint64_t* red_empty = red_full + kStreamNRB;  // [kStreamNRB]
  uint64_t* sx_ready = red_empty + kStreamNRB;  // activation sums written (reducer)
  uint64_t* xfull = sx_ready + 1;               // [kStreamNRB] peers' partials landed (rank 0)
  uint64_t* xempty = xfull + kStreamNRB;        // [kStreamNRB] rank 0 done with a slot (rank > 0)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t lim = p.wait_ns;  // limit of every bounded wait
  const int S = p.stages;
  const int NMB = p.n_meta;
  // Split K: a cluster of C CTAs shares the same rows; CTA `rank` streams the
  // K slice [klo, klo + kn) with those activations resident, and rank 0 sums
  // the C partials of every tile through distributed shared memory.
  const int C = p.C;
  const int rank = C > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cid = static_cast<int>(blockIdx.x) / C;
  const int ncl = static_cast<int>(gridDim.x) / C;
  const int klo = rank * p.KC;
  const int kn = min(p.KC, p.K - klo);
  const int n_slabs = (kn + p.KS - 1) / p.KS;
  const int64_t row_bytes = static_cast<int64_t>(p.K) * BITS / 8;
  const int row_begin = static_cast<int>(static_cast<int64_t>(p.N) * cid / ncl);
  const int row_end = static_cast<int>(static_cast<int64_t>(p.N) * (cid + 1) / ncl);
  const int n_tiles = (row_end - row_begin + kTile - 1) / kTile;
  const int total = n_tiles * n_slabs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStreamNCW);
    }
    for (int b = 0; b < NMB; ++b) mbar_init(&meta_full[b], 1);
    for (int b = 0; b < kStreamNRB; ++b) {
      mbar_init(&red_full[b], kStreamNCW);
      mbar_init(&red_empty[b], 1);
    }
    mbar_init(sx_ready, 1);
    for (int b = 0; b < kStreamNRB; ++b) {
      mbar_init(&xfull[b], 32 * (C - 1));
      mbar_init(&xempty[b], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Peers arrive on each other's barriers: all of them must exist first.
  if (C > 1) cluster_sync_all();
  if (threadIdx.x == 0) pdl_launch_dependents();

  // Each role runs as a lambda: a role that gives up a bounded wait returns
  // from its lambda and still reaches the cluster barrier below.
  if (warp == 0) [&] {
    // ------------------------------------------------------------ producer
    if (p.starve) return;  // diagnostic: issue nothing, every wait gives up
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const uint8_t* qw = reinterpret_cast<const uint8_t*>(p.qw);
    // The last few scales/zeros elements past the tensors' last 16-byte
    // boundary cannot be bulk-copied; the last CTA reads them here and stores
    // them into its final tile's metadata buffer.
    uint16_t tail_s = 0, tail_z = 0;
    if (cid == ncl - 1 && lane < p.tail_n) {
      tail_s = p.scales[p.tail_first + lane];
      if (!SYM) tail_z = p.zeros[p.tail_first + lane];
    }
    // A tile's scales (and zeros): rows [r0, r0 + R) x all groups, one
    // contiguous span, copied from its enclosing 16-byte boundary a0.
    auto issue_meta = [&](int i) {
      const int r0 = row_begin + i * kTile;
      const int R = min(kTile, row_end - r0);
      const int64_t e0 = static_cast<int64_t>(r0) * p.G;
      const int64_t e1 = static_cast<int64_t>(r0 + R) * p.G;
      const int64_t a0 = (e0 * 2) & ~15ll;
      const int64_t a1 = min((e1 * 2 + 15) & ~15ll, p.tail_first * 2);
      const uint32_t bytes = a1 > a0 ? static_cast<uint32_t>(a1 - a0) : 0u;
      const int mb = i % NMB;
      uint8_t* dst = smem + p.off_meta + mb * p.meta_stride;
      if (e1 > p.tail_first) {
        const int64_t e = p.tail_first + lane;
        if (lane < p.tail_n && e >= e0 && e < e1) {
          *reinterpret_cast<uint16_t*>(dst + e * 2 - a0) = tail_s;
          if (!SYM) *reinterpret_cast<uint16_t*>(dst + p.meta_half + e * 2 - a0) = tail_z;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&meta_full[mb], SYM ? bytes : 2 * bytes);
      __syncwarp();
      if (bytes) {
        if (lane == 0)
          bulk_g2s(dst, reinterpret_cast<const uint8_t*>(p.scales) + a0, bytes, &meta_full[mb],
                   pol_x);
        if (!SYM && lane == 1)
          bulk_g2s(dst + p.meta_half, reinterpret_cast<const uint8_t*>(p.zeros) + a0, bytes,
                   &meta_full[mb], pol_x);
      }
    };
    auto issue_stage = [&](int s) {
      const int i = s / n_slabs, j = s - (s / n_slabs) * n_slabs;
      const int r0 = row_begin + i * kTile;
      const int R = min(kTile, row_end - r0);
      const int k0 = klo + j * p.KS;
      const int L = min(p.KS, klo + kn - k0);
      const uint32_t run = static_cast<uint32_t>(L) * BITS / 8;
      const int slot = s % S;
      uint8_t* st = smem + slot * p.stage_bytes;
      if (j == 0) issue_meta(i);
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], R * run);
      __syncwarp();
      if (lane < R)
        bulk_g2s(st + lane * p.w_pitch, qw + (r0 + lane) * row_bytes + k0 * BITS / 8, run,
                 &full[slot], pol_w);
    };
    // Packed weights and metadata are inputs the previous grid does not
    // write; the activations are loaded by the consumer warps with plain
    // loads after their own dependent-launch wait, so nothing queues behind
    // these copies. With p.prefetch the whole first ring is issued at once,
    // before this grid's dependency on the previous one is resolved (the
    // copies run while the previous grid drains); without it the producer
    // waits for the previous grid first.
    if (!p.prefetch) pdl_wait_prior_grid();
    int s = 0;
    for (; s < total && s < S && s / n_slabs < NMB; ++s) issue_stage(s);
    for (; s < total; ++s) {
      const int slot = s % S;
      if (s >= S && !warp_wait(&empty[slot], ((s / S) - 1) & 1, lim)) break;
      const int i = s / n_slabs;
      if (i >= NMB && s == i * n_slabs) {
        // Metadata buffer i % NMB is free once tile i - NMB is consumed: its
        // last stage t released (implied by the wait above when t <= s - S).
        const int t = (i - NMB + 1) * n_slabs - 1;
        if (t > s - S && !warp_wait(&empty[t % S], (t / S) & 1, lim)) break;
      }
      issue_stage(s);
    }
    // Drain: every copy this warp issued has landed before the CTA exits.
    for (int t = max(0, s - S); t < s; ++t) mbar_wait(&full[t % S], (t / S) & 1, lim);
    const int issued_tiles = (s + n_slabs - 1) / n_slabs;
    for (int ii = max(0, issued_tiles - NMB); ii < issued_tiles; ++ii)
      mbar_wait(&meta_full[ii % NMB], (ii / NMB) & 1, lim);
  }();
  else if (warp == 1) [&] {
    // ------------------------------------------------------------- reducer
    const float* sxg = reinterpret_cast<const float*>(smem + p.off_sx);
    for (int i = 0; i < n_tiles; ++i) {
      const int b = i % kStreamNRB;
      const int r0 = row_begin + i * kTile;
      const int R = min(kTile, row_end - r0);
      float sc = 0.f, zc = 0.f;
      if constexpr (!GROUPED) {
        // Per-channel: one scale (and zero) per row, applied here.
        if (lane < R) {
          sc = __half2float(__ushort_as_half(p.scales[r0 + lane]));
          zc = SYM ? kBias : __half2float(__ushort_as_half(p.zeros[r0 + lane]));
        }
      }
      if (!warp_wait(&red_full[b], (i / kStreamNRB) & 1, lim)) return;
      if constexpr (!GROUPED) {
        if (!warp_wait(sx_ready, 0, lim)) return;
      }
      const float* red = reinterpret_cast<const float*>(smem + p.off_red) +
                         b * (kStreamNCW * kTile * p.M);
      // This CTA's partial of each (row, activation row) of the tile: up to 4
      // elements per lane (16 rows x M <= 128).
      float part[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int idx = q * 32 + lane;
        const int row = idx & (kTile - 1);
        const int m = idx >> 4;
        const float s_row = __shfl_sync(0xffffffffu, sc, row);
        const float z_row = __shfl_sync(0xffffffffu, zc, row);
        part[q] = 0.f;
        if (idx < kTile * p.M && row < R) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kStreamNCW; ++w) sum += red[(w * kTile + row) * p.M + m];
          if constexpr (!GROUPED) sum = s_row * (SYM ? sum : fmaf(-(z_row - kBias), sxg[m], sum));
          part[q] = sum;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_empty[b]);
      float* xred = reinterpret_cast<float*>(smem + p.off_xred) + b * (C * kTile * p.M);
      if (C > 1 && rank > 0) {
        // Send the partial to rank 0's slot b (free once rank 0 released it
        // for tile i - kStreamNRB), then arrive there.
        if (i >= kStreamNRB && !warp_wait_cluster(&xempty[b], ((i / kStreamNRB) - 1) & 1, lim))
          return;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int idx = q * 32 + lane;
          const int row = idx & (kTile - 1);
          if (idx < kTile * p.M && row < R)
            st_cluster_f32(map_to_rank(xred + rank * kTile * p.M + (idx >> 4) * kTile + row, 0),
                           part[q]);
        }
        mbar_arrive_remote(map_to_rank(&xfull[b], 0));
        continue;
      }
      if (C > 1 && !warp_wait_cluster(&xfull[b], (i / kStreamNRB) & 1, lim)) return;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int idx = q * 32 + lane;
        const int row = idx & (kTile - 1);
        const int m = idx >> 4;
        if (idx < kTile * p.M && row < R) {
          float sum = part[q];
          for (int r = 1; r < C; ++r) sum += xred[r * kTile * p.M + m * kTile + row];
          p.y[static_cast<int64_t>(m) * p.N + r0 + row] = __half_as_ushort(__float2half_rn(sum));
        }
      }
      if (C > 1) {
        __syncwarp();
        if (lane >= 1 && lane < C) mbar_arrive_remote(map_to_rank(&xempty[b], lane));
      }
    }
    // A peer leaves only once rank 0 has released every slot it used, so no
    // remote arrive can target a CTA that has exited.
    if (C > 1 && rank > 0) {
      for (int i = max(0, n_tiles - kStreamNRB); i < n_tiles; ++i)
        if (!warp_wait_cluster(&xempty[i % kStreamNRB], (i / kStreamNRB) & 1, lim)) return;
    }
  }();
  else [&] {
    // ----------------------------------------------------------- consumers
    using XU = XUnits<BITS, WPL>;
    const int cw = warp - 2;
    const int tid = cw * 32 + lane;
    constexpr int kCT = kStreamNCW * 32;
    float* sstep = reinterpret_cast<float*>(smem + p.off_sstep);
    float* sxg = reinterpret_cast<float*>(smem + p.off_sx);
    const int spr = kn / SC;   // steps per activation row (this CTA's K slice)
    const int Gs = GROUPED ? kn / p.gsize : 1;  // groups in the slice
    const int g_lo = GROUPED ? klo / p.gsize : 0;

    // Prologue 1: activations from global memory into B-fragment order in
    // shared memory, with per-step sums (asymmetric formats only). The loads
    // come after this thread's dependent-launch wait (the previous grid may
    // have written x) and use the load/store path, not the bulk-copy queue
    // that carries the weight ring. The words of all M rows form one flat
    // index space; each lane loads kU words (128 bytes) per pass. Rows and
    // steps start on multiples of SW words and each pass's words are
    // contiguous in groups of 32 lanes, so a step's SW words lie in one
    // aligned group of SW lanes; a step's sum is the sum of its quads'
    // totals (quad_sum).
    for (int i = tid; i < STEP_XB / 16; i += kCT)
      reinterpret_cast<uint4*>(smem + p.off_zero)[i] = make_uint4(0u, 0u, 0u, 0u);
    pdl_wait_prior_grid();
    // Word wi of an activation row, permuted in registers and stored at its
    // place in the row's B-fragment order.
    auto put = [&](const uint32_t (&w)[NPAIR], uint8_t* row, int wi) {
      uint32_t o[NPAIR];
#pragma unroll
      for (int r = 0; r < NPAIR; ++r) {
        const int lo = slot_logical(BITS, INTER, b_slot(BITS, r, 0));
        const int hi = slot_logical(BITS, INTER, b_slot(BITS, r, 1));
        o[r] = prmt(w[lo >> 1], w[hi >> 1],
                    ((lo & 1) ? 0x32u : 0x10u) | ((hi & 1) ? 0x7600u : 0x5400u));
      }
      const int q = wi & (SW - 1);
      const int cc = q / WPL;
      const int j = q - cc * WPL;
      constexpr int PB = WB < XU::U ? WB : XU::U;
      uint8_t* sbase = row + (wi / SW) * STEP_XB + cc * XU::U;
#pragma unroll
      for (int pc = 0; pc < WB / PB; ++pc) {
        const int lb = j * WB + pc * PB;
        sts<PB>(sbase + (lb / XU::U) * 4 * XU::U + (lb % XU::U), o + pc * (PB / 4));
      }
    };
    constexpr int kU = 128 / WB;
    const int wpr = kn / PP;  // words per activation row
    const int wtot = p.M * wpr;
    const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.x + klo);
    const int64_t xrow_bytes = static_cast<int64_t>(p.K) * 2;
    // ceil(2^32 / wpr): umulhi(f, wmagic) == f / wpr for every f < 2^32 / wpr.
    const uint32_t wmagic = 0xFFFFFFFFu / static_cast<uint32_t>(wpr) + 1u;
    for (int w0 = cw * 32; w0 < wtot; w0 += kU * kCT) {
      uint32_t v[kU][NPAIR];
      int mrow[kU], wcol[kU];
#pragma unroll
      for (int uu = 0; uu < kU; ++uu) {
        const int wf = w0 + uu * kCT + lane;
        const int m = static_cast<int>(__umulhi(static_cast<uint32_t>(wf), wmagic));
        mrow[uu] = m;
        wcol[uu] = wf - m * wpr;
        if (wf < wtot) {
          ldg_l2<WB>(xg + m * xrow_bytes + wcol[uu] * WB, v[uu]);
        } else {
#pragma unroll
          for (int r = 0; r < NPAIR; ++r) v[uu][r] = 0u;
        }
      }
#pragma unroll
      for (int uu = 0; uu < kU; ++uu) {
        if (w0 + uu * kCT + lane < wtot) put(v[uu], smem + p.off_x + mrow[uu] * p.xp, wcol[uu]);
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
            sstep[mrow[uu] * spr + wcol[uu] / SW] = sum[uu];
        }
      }
    }
    named_sync(1, kStreamNCW * 32);
    // Prologue 2: the activation sum of every group (per-channel: of the
    // whole row); symmetric formats need none.
    // A group of one step (spg == 1) has its sum already: the per-step sums
    // are read as the group sums and this pass and its barrier are skipped.
    const bool group_is_step = GROUPED && p.gsize == SC;
    if constexpr (SYM) {
    } else if constexpr (GROUPED) {
      const int spg = p.gsize / SC;
      if (group_is_step) sxg = sstep;
      else
        for (int e = tid; e < p.M * Gs; e += kCT) {
          const int m = e / Gs;
          const int g = e - m * Gs;
          const float* src = sstep + m * spr + g * spg;
          float sum = 0.f;
          for (int t = 0; t < spg; ++t) sum += src[t];
          sxg[e] = sum;
        }
    } else {
      if (cw < p.M) {
        float sum = 0.f;
        for (int t = lane; t < spr; t += 32) sum += sstep[cw * spr + t];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        if (lane == 0) sxg[cw] = sum;
      }
    }
    if (!SYM && !group_is_step) named_sync(1, kStreamNCW * 32);
    if (tid == 0) mbar_arrive(sx_ready);

    // Main loop. Work units (grouped: gslots consecutive groups; per-channel:
    // one step) go to warps round-robin by their index over the whole CTA.
    const int gid = lane >> 2;
    const int c = lane & 3;
    constexpr int mp = MP;
    constexpr int gslots = GROUPED ? GS : 1;
    const int my_slot = gid / mp;
    const int my_xrow = gid - my_slot * mp;
    const bool x_ok = my_xrow < p.M;
    const uint8_t* xrow_base = smem + p.off_x + (x_ok ? my_xrow : 0) * p.xp + c * XU::U;
    // Lanes whose column is not live read zeros from a block 64 bytes off the
    // activations' bank phase (no bank conflict with the live lanes).
    const uint8_t* zero_base = smem + p.off_zero + c * XU::U;
    constexpr int kStepWB = SC * BITS / 8;  // packed bytes per step per row
    const int spg = p.gsize / SC;
    const int units_per_tile = GROUPED ? (Gs + gslots - 1) / gslots : spr;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float D[NCH][4];
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int e = 0; e < 4; ++e) D[ch][e] = 0.f;

    int s = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int r0 = row_begin + i * kTile;
      // (Waited for in every mode: the producer reuses a metadata buffer
      // only after its previous copy has been seen complete here.)
      if (!warp_wait(&meta_full[i % NMB], (i / NMB) & 1, lim)) return;
      const uint8_t* meta = smem + p.off_meta + (i % NMB) * p.meta_stride;
      const int64_t a0 = (static_cast<int64_t>(r0) * p.G * 2) & ~15ll;
      // Byte offsets of (row gid, group 0) and (row gid + 8, group 0).
      const int mo_a = static_cast<int>(static_cast<int64_t>(r0 + gid) * p.G * 2 - a0);
      const int mo_b = mo_a + 8 * p.G * 2;
      for (int j = 0; j < n_slabs; ++j, ++s) {
        const int slot = s % S;
        if (!warp_wait(&full[slot], (s / S) & 1, lim)) return;
        const int k0 = klo + j * p.KS;          // absolute K of the slab
        const int L = min(p.KS, klo + kn - k0);
        const int kx0 = k0 - klo;               // its offset in the resident slice
        const uint8_t* st = smem + slot * p.stage_bytes;
        const uint8_t* wa_row = st + gid * p.w_pitch + c * WPL * 4;
        const uint8_t* wb_row = wa_row + 8 * p.w_pitch;
        if constexpr (GROUPED) {
          const int g_slab = k0 / p.gsize;
          const int ng = L / p.gsize;
          const int units = (ng + gslots - 1) / gslots;
          const int ubase = i * units_per_tile + (g_slab - g_lo) / gslots;
          // M > 4 (one group per unit): two units per iteration overlap one
          // unit's epilogue with the next one's loads (measured faster there,
          // slower for the larger units of M <= 4).
#pragma unroll(MP == 8 ? 2 : 1)
          for (int u = (cw - ubase % kStreamNCW + kStreamNCW) % kStreamNCW; u < units;
               u += kStreamNCW) {
            // This unit's scales, zero-points and activation sums, loaded
            // before its MMAs.
            bool ev[4];
            float sv[4], zv[4], sxv[4];
            if constexpr (MP >= 2) {
              // A lane's two columns 2c, 2c + 1 are one group slot (and two
              // activation rows): one scale/zero per weight row, one sum per
              // activation row.
              const int slot = (2 * c) / MP;
              const int xr0 = 2 * c - slot * MP;
              const int gl = u * gslots + slot;
              const bool gok = gl < ng;
              const int g = g_slab + (gok ? gl : 0);
              ev[0] = ev[2] = gok && xr0 < p.M;
              ev[1] = ev[3] = gok && xr0 + 1 < p.M;
              sv[0] = sv[1] = __half2float(*reinterpret_cast<const __half*>(meta + mo_a + g * 2));
              sv[2] = sv[3] = __half2float(*reinterpret_cast<const __half*>(meta + mo_b + g * 2));
              if constexpr (!SYM) {
                const uint8_t* zm = meta + p.meta_half + g * 2;
                zv[0] = zv[1] = __half2float(*reinterpret_cast<const __half*>(zm + mo_a));
                zv[2] = zv[3] = __half2float(*reinterpret_cast<const __half*>(zm + mo_b));
                const float* sx = sxg + (g - g_lo);
                sxv[0] = sxv[2] = sx[(ev[0] ? xr0 : 0) * Gs];
                sxv[1] = sxv[3] = sx[(ev[1] ? xr0 + 1 : 0) * Gs];
              } else {
                zv[0] = zv[1] = zv[2] = zv[3] = 0.f;
                sxv[0] = sxv[1] = sxv[2] = sxv[3] = 0.f;
              }
            } else {
              // One activation row: the lane's two columns are two slots.
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int slot_e = 2 * c + (e & 1);
                const int gl = u * gslots + slot_e;
                ev[e] = gl < ng && x_ok;
                const int g = g_slab + (ev[e] ? gl : 0);
                const int mo = ((e >> 1) ? mo_b : mo_a) + g * 2;
                sv[e] = __half2float(*reinterpret_cast<const __half*>(meta + mo));
                if constexpr (!SYM) {
                  zv[e] = __half2float(*reinterpret_cast<const __half*>(meta + p.meta_half + mo));
                  sxv[e] = sxg[g - g_lo];
                } else {
                  zv[e] = 0.f;
                  sxv[e] = 0.f;
                }
              }
            }
            if (spg == 1 && (u + 1) * gslots <= ng) {
              // A whole unit of one-step groups: fully unrolled.
              const int st0 = u * gslots;
              const uint8_t* pwa = wa_row + st0 * kStepWB;
              const uint8_t* pwb = wb_row + st0 * kStepWB;
              const uint8_t* px = xrow_base + (kx0 / SC + st0) * STEP_XB;
#pragma unroll
              for (int gs = 0; gs < gslots; ++gs) {
                const uint8_t* pxg = (x_ok && my_slot == gs) ? px + gs * STEP_XB : zero_base;
                if (gs == 0)  // the unit's first step starts its chains
                  mma_step<BITS, WPL, true>(pwa, pwb, pxg, D);
                else
                  mma_step<BITS, WPL, false>(pwa + gs * kStepWB, pwb + gs * kStepWB, pxg, D);
              }
            } else {
#pragma unroll
              for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
                for (int e = 0; e < 4; ++e) D[ch][e] = 0.f;
              for (int gs = 0; gs < gslots; ++gs) {
                const int gl = u * gslots + gs;
                if (gl >= ng) break;
                const bool live = x_ok && my_slot == gs;
                const int st0 = gl * spg;         // first step of the group in the slab
                const int kst = kx0 / SC + st0;   // its step index in the slice
                for (int t = 0; t < spg; ++t) {
                  const int wofs = (st0 + t) * kStepWB;
                  mma_step<BITS, WPL, false>(wa_row + wofs, wb_row + wofs,
                                            live ? xrow_base + (kst + t) * STEP_XB : zero_base, D);
                }
              }
            }
            float P[4];
            combine<NCH>(D, P);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (ev[e]) {
                float t = P[e];
                if constexpr (!SYM) t = fmaf(-(zv[e] - kBias), sxv[e], t);
                acc[e] = fmaf(sv[e], t, acc[e]);
              }
            }
          }
        } else {
          const int steps = L / SC;
          const int st_glob0 = kx0 / SC;
          const int ubase = i * units_per_tile + st_glob0;
          int u = (cw - ubase % kStreamNCW + kStreamNCW) % kStreamNCW;
          // Two steps per iteration: the second one's loads overlap the first
          // one's MMAs.
          for (; u + kStreamNCW < steps; u += 2 * kStreamNCW) {
            mma_step<BITS, WPL, false>(wa_row + u * kStepWB, wb_row + u * kStepWB,
                                      x_ok ? xrow_base + (st_glob0 + u) * STEP_XB : zero_base, D);
            const int u2 = u + kStreamNCW;
            mma_step<BITS, WPL, false>(wa_row + u2 * kStepWB, wb_row + u2 * kStepWB,
                                      x_ok ? xrow_base + (st_glob0 + u2) * STEP_XB : zero_base, D);
          }
          if (u < steps)
            mma_step<BITS, WPL, false>(wa_row + u * kStepWB, wb_row + u * kStepWB,
                                      x_ok ? xrow_base + (st_glob0 + u) * STEP_XB : zero_base, D);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }

      // Tile end: per (row, activation row) partial of this warp.
      if constexpr (!GROUPED) {
        combine<NCH>(D, acc);
#pragma unroll
        for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
          for (int e = 0; e < 4; ++e) D[ch][e] = 0.f;
      }
      // Columns sharing an activation row (different group slots) are summed
      // across lanes: slots are the high bits of the column 2c + (e & 1).
      if (mp == 1) {
        acc[0] += acc[1];
        acc[2] += acc[3];
      }
      if (mp <= 2) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 1);
          acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 2);
        }
      } else if (mp == 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 2);
      }
      const int b = i % kStreamNRB;
      if (i >= kStreamNRB && !warp_wait(&red_empty[b], ((i / kStreamNRB) - 1) & 1, lim)) return;
      float* red = reinterpret_cast<float*>(smem + p.off_red) + b * (kStreamNCW * kTile * p.M) +
                   cw * kTile * p.M;
      const int cmask = mp <= 2 ? 3 : (mp == 4 ? 2 : 0);
      if ((c & cmask) == 0) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (mp == 1 && (e & 1)) continue;
          const int row = gid + 8 * (e >> 1);
          const int xrow = (2 * c + (e & 1)) & (mp - 1);
          if (xrow < p.M) red[row * p.M + xrow] = acc[e];
        }
      }
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[b]);
    }
  }();
  // No CTA of a cluster exits while a peer may still store into its shared
  // memory or arrive on its barriers: all threads of all CTAs meet here, also
  // after a wait gave up (every wait before this point is bounded).
  if (C > 1) cluster_sync_all_unaligned();
}


template <int BITS, bool SYM, bool INTER, int WPL, int GS>
cudaError_t launch_one(const StreamParams& p, int grid, int smem, cudaStream_t stream) {
  auto kern = gemv_stream_kernel<BITS, SYM, INTER, WPL, GS>;
  static int configured[64] = {0};  // max dynamic smem already raised, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemBytes);
    if (e != cudaSuccess) return e;
    // The whole carveout as shared memory, for every variant alike, so that a
    // CTA of the next launch can become resident beside one of this launch.
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: this grid may start while the previous
  // one drains; it waits for it before reading activations. Split-K runs as
  // clusters of p.C CTAs.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.C > 1 ? 2 : 1;
  if (p.C > 1) {
    // No more clusters than can be resident at once (the plan assumed every
    // SM; GPC boundaries can leave some out). Cached per device and size.
    static int cached_n[64][kStreamMaxCluster + 1] = {};
    int n = (dev >= 0 && dev < 64) ? cached_n[dev][p.C] : 0;
    if (n == 0) {
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return e;
      if (n < 1) return cudaErrorInvalidConfiguration;
      if (dev >= 0 && dev < 64) cached_n[dev][p.C] = n;
    }
    if (grid / p.C > n) cfg.gridDim = dim3(n * p.C);
  }
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, bool SYM, bool INTER, int WPL>
cudaError_t launch_gs(int gs, const StreamParams& p, int grid, int smem, cudaStream_t stream) {
  switch (gs) {
    case 0: return launch_one<BITS, SYM, INTER, WPL, 0>(p, grid, smem, stream);
    case 1: return launch_one<BITS, SYM, INTER, WPL, 1>(p, grid, smem, stream);
    case 2: return launch_one<BITS, SYM, INTER, WPL, 2>(p, grid, smem, stream);
    case 4: return launch_one<BITS, SYM, INTER, WPL, 4>(p, grid, smem, stream);
    case 8: return launch_one<BITS, SYM, INTER, WPL, 8>(p, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

// All variants of one bit width (one translation unit per width).
template <int BITS>
cudaError_t launch_bits(int wpl, int gs, bool sym, bool inter, const StreamParams& p, int grid,
                        int smem, cudaStream_t stream) {
#define DQG_WPL(S, I)                                                        \
  switch (wpl) {                                                             \
    case 4: return launch_gs<BITS, S, I, 4>(gs, p, grid, smem, stream);      \
    case 2: return launch_gs<BITS, S, I, 2>(gs, p, grid, smem, stream);      \
    default: return launch_gs<BITS, S, I, 1>(gs, p, grid, smem, stream);     \
  }
  if (sym && inter) { DQG_WPL(true, true) }
  if (sym) { DQG_WPL(true, false) }
  if (inter) { DQG_WPL(false, true) }
  DQG_WPL(false, false)
#undef DQG_WPL
}

}  // namespace stream
}  // namespace dqg
