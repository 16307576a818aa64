// Fused low-bit dequantize + GEMV for B200 (sm_100a).
//
// y[m, n] = fp16( sum_k x[m, k] * (q[n, k] - off[n, k/g]) * scale[n, k/g] ),
// fp32 accumulation, for 1 <= M <= 8 activation rows, with the packed format of
// the reference packer (KrishnaI2424/Dequant_Project dequant/packer.py:7-29):
// int32 words of 32/bits unsigned codes, fp16 scales [N, K/g] and, when
// asymmetric, fp16 zero-points [N, K/g]; off = 2^(bits-1) when symmetric.
// The reference kernel this replaces is kernels/dequant_gemv.cu:144-217.
//
// Design (one CTA per SM, warp-specialised):
//   * Every CTA owns a contiguous range of 16-row tiles (one m16 MMA tile
//     each), processed tile by tile in K slabs. One (tile, slab) pair is one
//     pipeline stage in a ring of shared-memory slots.
//   * warp 0 streams each stage: one untiled bulk copy (cp.async.bulk, no
//     multicast) per packed row segment into padded rows, the tile's scales
//     and zero-points as one contiguous span, and (when x is not resident)
//     the activation slab, all completing on mbarriers. Weights and metadata
//     are issued before the programmatic-dependent-launch wait; activations
//     after it.
//   * warps 1..kNAux prepare every stage together and in order: per (row,
//     group) they turn scale and zero-point into the fp16 unpack constant and
//     fp32 scale, and they rewrite x into the k-order the unpack produces
//     (once for the whole K when it fits, else per slab), with per-step sums.
//   * kNCW consumer warps unpack codes in registers and run mma.m16n8k16
//     (fp16 x fp16 -> fp32) with the weight rows as the M=16 side and the <= 8
//     activation rows as the N=8 side. Steps go to warps by their global index
//     along K, so every output row is summed in the same order for any M and
//     any slab length; a fixed-order shared-memory reduction ends each tile.
//   * Every wait on an mbarrier is bounded (a device-side status flag records a
//     timeout and the kernel returns).
//
// Exactness of the unpack: a code pair is dropped into the mantissa of
// 0x6400 (fp16 1024) with one LOP3, giving 1024 + 2^p q exactly; one HADD2 or
// HFMA2 with the per-group constant -(1024/2^p + z') then yields q - z'
// exactly, z' = clamp(rint(z), -1024, 1024). The residual (z' - z), non-zero
// only for out-of-range or fractional zero-points, is added back in fp32
// through per-step activation sums. Products (q - z') * x are exact in fp32;
// the scale multiplies each step's partial sum in fp32 (as the reference does
// per 16-byte chunk, dequant_gemv.cu:199-200).
//
// The k-order inside a step is free because the reduction is a sum: slot pair
// t of a word is (t, t + 32/bits/2) for every bit width and both layouts, and
// x is permuted to match (the interleaved layout only changes that
// permutation).
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {

namespace {

constexpr uint32_t kMagic = 0x64006400u;    // fp16 1024.0 in both halves
constexpr uint32_t kQuarter = 0x34003400u;  // fp16 0.25
constexpr uint32_t kSixteenth = 0x2C002C00u;  // fp16 0.0625

// Unpack one packed word into 16/bits half2 pairs holding (q - z') exactly.
// Pair t holds slots (t, t + PP/2). kc = {K0, K1, K2} are the half2
// constants -(1024 + z'), -(256 + z'), -(64 + z').
template <int BITS>
__device__ __forceinline__ void unpack_pairs(uint32_t w, uint32_t K0, uint32_t K1, uint32_t K2,
                                             uint32_t* pr) {
  if constexpr (BITS == 4) {
    pr[0] = hadd2_u32(lop3_and_or(w, 0x000F000Fu, kMagic), K0);
    pr[1] = hfma2_u32(lop3_and_or(w, 0x00F000F0u, kMagic), kSixteenth, K2);
    const uint32_t w8 = w >> 8;
    pr[2] = hadd2_u32(lop3_and_or(w8, 0x000F000Fu, kMagic), K0);
    pr[3] = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, kMagic), kSixteenth, K2);
  } else if constexpr (BITS == 8) {
    pr[0] = hadd2_u32(prmt(w, 0x64646464u, 0x4240u), K0);  // slots 0, 2
    pr[1] = hadd2_u32(prmt(w, 0x64646464u, 0x4341u), K0);  // slots 1, 3
  } else {
    pr[0] = hadd2_u32(lop3_and_or(w, 0x00030003u, kMagic), K0);
    pr[1] = hfma2_u32(lop3_and_or(w, 0x000C000Cu, kMagic), kQuarter, K1);
    pr[2] = hfma2_u32(lop3_and_or(w, 0x00300030u, kMagic), kSixteenth, K2);
    const uint32_t w6 = w >> 6;
    pr[3] = hadd2_u32(lop3_and_or(w6, 0x00030003u, kMagic), K0);
    pr[4] = hfma2_u32(lop3_and_or(w6, 0x000C000Cu, kMagic), kQuarter, K1);
    pr[5] = hfma2_u32(lop3_and_or(w6, 0x00300030u, kMagic), kSixteenth, K2);
    const uint32_t w12 = w >> 12;
    pr[6] = hadd2_u32(lop3_and_or(w12, 0x00030003u, kMagic), K0);
    pr[7] = hfma2_u32(lop3_and_or(w12, 0x000C000Cu, kMagic), kQuarter, K1);
  }
}

__device__ __forceinline__ void mma_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int N>
struct Vec;
template <>
struct Vec<4> {
  static __device__ __forceinline__ void ld(const uint8_t* p, uint32_t* r) {
    r[0] = *reinterpret_cast<const uint32_t*>(p);
  }
};
template <>
struct Vec<8> {
  static __device__ __forceinline__ void ld(const uint8_t* p, uint32_t* r) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    r[0] = v.x;
    r[1] = v.y;
  }
};
template <>
struct Vec<32> {
  static __device__ __forceinline__ void ld(const uint8_t* p, uint32_t* r) {
    const uint4 v0 = *reinterpret_cast<const uint4*>(p);
    const uint4 v1 = *reinterpret_cast<const uint4*>(p + 16);
    r[0] = v0.x;
    r[1] = v0.y;
    r[2] = v0.z;
    r[3] = v0.w;
    r[4] = v1.x;
    r[5] = v1.y;
    r[6] = v1.z;
    r[7] = v1.w;
  }
};
template <>
struct Vec<16> {
  static __device__ __forceinline__ void ld(const uint8_t* p, uint32_t* r) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    r[0] = v.x;
    r[1] = v.y;
    r[2] = v.z;
    r[3] = v.w;
  }
};

}  // namespace

constexpr uint32_t kH768 = 0x62006200u;   // fp16 768.0 in both halves
constexpr uint32_t kH960 = 0x63806380u;   // fp16 960.0 in both halves

// Permute one word's worth of activations (natural order in v[]) into the
// unpack's pair order: pair t = (x[logical(t)], x[logical(t + NPAIR)]).
template <int BITS, bool INTER, int NPAIR>
__device__ __forceinline__ void permute_word(const uint32_t* v, uint32_t* o) {
#pragma unroll
  for (int t = 0; t < NPAIR; ++t) {
    const int lo = slot_logical(BITS, INTER, t);
    const int hi = slot_logical(BITS, INTER, t + NPAIR);
    o[t] = prmt(v[lo >> 1], v[hi >> 1],
                ((lo & 1) ? 0x32u : 0x10u) | ((hi & 1) ? 0x7600u : 0x5400u));
  }
}

// Store the permuted pairs of word `wi` (index within a run of whole steps)
// into a permuted-activation row at `xp`: step st = wi / (4*WPL) occupies
// STEP_XB bytes; inside it lane c's WPL words are spread in U-byte units so
// that the four lanes of a row read adjacent units.
template <int WPL, int WB, int U>
__device__ __forceinline__ void store_perm(uint8_t* xp, int wi, const uint32_t* o) {
  constexpr int STEP_XB = 4 * WPL * WB;
  const int stp = wi / (4 * WPL);
  const int q = wi - stp * (4 * WPL);
  const int c = q / WPL;
  const int jj = q - c * WPL;
  uint8_t* base = xp + stp * STEP_XB + c * U;
  if constexpr (WB >= U) {
#pragma unroll
    for (int piece = 0; piece < WB / U; ++piece) {
      const int u = (jj * WB) / U + piece;
      if constexpr (U == 16) {
        *reinterpret_cast<uint4*>(base + u * 4 * U) =
            make_uint4(o[piece * 4 + 0], o[piece * 4 + 1], o[piece * 4 + 2], o[piece * 4 + 3]);
      } else {
        *reinterpret_cast<uint2*>(base + u * 4 * U) = make_uint2(o[0], o[1]);
      }
    }
  } else {
    const int u = (jj * WB) / U;
    *reinterpret_cast<uint2*>(base + u * 4 * U + (jj * WB) % U) = make_uint2(o[0], o[1]);
  }
}

// One activation row's step (SC codes): load all of it at once from `src`
// (natural order; global or shared memory), sum it in natural order (the
// zero-point residual needs per-step sums), and write it in the unpack's
// pair order into the step's region `dst` of a permuted-activation row.
template <int BITS, bool INTER, int WPL>
__device__ __forceinline__ float process_step(const uint8_t* src, uint8_t* dst) {
  constexpr int PP = 32 / BITS;
  constexpr int NPAIR = PP / 2;
  constexpr int WB = PP * 2;
  constexpr int LXB = WPL * WB;
  constexpr int U = LXB >= 16 ? 16 : LXB;
  constexpr int NW = 4 * WPL;  // words per step
  // Words held in registers at once (at most 64 registers of activations).
  constexpr int CW = NW * NPAIR <= 64 ? NW : 64 / NPAIR;
  float sum = 0.f;
#pragma unroll
  for (int w0 = 0; w0 < NW; w0 += CW) {
    uint32_t v[CW][NPAIR];
#pragma unroll
    for (int w = 0; w < CW; ++w) Vec<WB>::ld(src + (w0 + w) * WB, v[w]);
#pragma unroll
    for (int w = 0; w < CW; ++w) {
#pragma unroll
      for (int q = 0; q < NPAIR; ++q) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v[w][q]));
        sum += f.x;
        sum += f.y;
      }
    }
#pragma unroll
    for (int w = 0; w < CW; ++w) {
      uint32_t o[NPAIR];
      permute_word<BITS, INTER, NPAIR>(v[w], o);
      store_perm<WPL, WB, U>(dst, w0 + w, o);
    }
  }
  return sum;
}

template <int BITS, bool SYM, bool INTER, int WPL, bool XRES>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  constexpr int PP = 32 / BITS;           // codes per word
  constexpr int NPAIR = PP / 2;           // half2 pairs per word
  constexpr int SC = 4 * WPL * PP;        // codes per step (4 lanes x WPL words)
  constexpr int WB = PP * 2;              // activation bytes per word
  constexpr int LXB = WPL * WB;           // activation bytes per lane per step
  constexpr int U = LXB >= 16 ? 16 : LXB;  // shared-memory load width for x
  constexpr int NU = LXB / U;
  constexpr int STEP_XB = 4 * LXB;
  constexpr int BIAS = 1 << (BITS - 1);

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full_w = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* full_aux = full_w + kMaxStages;
  uint64_t* empty = full_aux + kMaxStages;
  uint64_t* red_bar = empty + kMaxStages;
  uint64_t* meta_full = red_bar + 2;
  uint64_t* x_ready = meta_full + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;
  const int64_t row_bytes = static_cast<int64_t>(p.K) * BITS / 8;

  // This CTA's 16-row tiles; one (tile, K slab) pair is one stage.
  const int T = (p.N + kTile - 1) / kTile;
  const int t_begin = static_cast<int>(static_cast<int64_t>(T) * blockIdx.x / gridDim.x);
  const int t_end = static_cast<int>(static_cast<int64_t>(T) * (blockIdx.x + 1) / gridDim.x);
  const int total = (t_end - t_begin) * p.n_slabs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&full_aux[s], kNAux);
      mbar_init(&empty[s], kNCW);
    }
    mbar_init(&red_bar[0], kNCW * 32);
    mbar_init(&red_bar[1], kNCW * 32);
    mbar_init(&meta_full[0], 1);
    mbar_init(&meta_full[1], 1);
    mbar_init(x_ready, kNAux);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const uint8_t* qw = reinterpret_cast<const uint8_t*>(p.qw);
    // Scales/zeros of a tile: rows [r0, r0 + R) x all groups are one
    // contiguous span starting 16-byte aligned (r0 is a multiple of 16).
    // The aligned prefix comes by bulk copy; the rest (only in the matrix's
    // last partial tile) is read by the aux warps from global memory.
    auto issue_meta = [&](int i) {
      const int r0 = (t_begin + i) * kTile;
      const int R = min(kTile, p.N - r0);
      const uint32_t bytes = static_cast<uint32_t>(R * static_cast<int64_t>(p.G) * 2) & ~15u;
      uint8_t* dst = smem + p.off_meta + (i & 1) * p.meta_stride;
      if (lane == 0) mbar_arrive_expect_tx(&meta_full[i & 1], SYM ? bytes : 2 * bytes);
      __syncwarp();
      if (bytes) {
        if (lane == 0)
          bulk_g2s(dst, p.scales + static_cast<int64_t>(r0) * p.G, bytes, &meta_full[i & 1], pol_x);
        if (!SYM && lane == 1)
          bulk_g2s(dst + p.meta_stride / 2, p.zeros + static_cast<int64_t>(r0) * p.G, bytes,
                   &meta_full[i & 1], pol_x);
      }
    };
    auto x_slab = [&](int s) {
      const int j = s % p.n_slabs;
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      uint8_t* st = smem + (s % S) * p.stage_bytes;
      if (lane < p.M)
        bulk_g2s(st + p.off_xraw + lane * (p.KS * 2), p.x + static_cast<int64_t>(lane) * p.K + k0,
                 static_cast<uint32_t>(L) * 2, &full_w[s % S], pol_x);
    };
    // One stage: a long bulk copy per packed row (the tile's rows are
    // consecutive, so HBM sees one contiguous run per tile when n_slabs = 1).
    auto issue_stage = [&](int s, bool with_x) {
      const int i = s / p.n_slabs, j = s - (s / p.n_slabs) * p.n_slabs;
      const int r0 = (t_begin + i) * kTile;
      const int R = min(kTile, p.N - r0);
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      const uint32_t run = static_cast<uint32_t>(L) * BITS / 8;
      const int slot = s % S;
      uint8_t* st = smem + slot * p.stage_bytes;
      if (p.meta_direct && j == 0) issue_meta(i);
      if (lane == 0)
        mbar_arrive_expect_tx(&full_w[slot], R * run + (XRES ? 0u : p.M * L * 2u));
      __syncwarp();
      if (lane < R)
        bulk_g2s(st + p.off_w + lane * p.w_pitch, qw + (r0 + lane) * row_bytes + k0 * BITS / 8, run,
                 &full_w[slot], pol_w);
      if (!XRES && with_x) x_slab(s);
    };
    // Weights and metadata do not depend on the previous grid: stream the
    // first stages before waiting for it; activations only after.
    int pre = min(S, total);
    if (p.meta_direct) pre = min(pre, 2 * p.n_slabs);
    for (int s = 0; s < pre; ++s) issue_stage(s, false);
    pdl_wait_prior_grid();
    if (!XRES)
      for (int s = 0; s < pre; ++s) x_slab(s);
    int s = pre;
    for (; s < total; ++s) {
      const int slot = s % S;
      if (s >= S && !warp_wait(&empty[slot], ((s / S) - 1) & 1)) break;
      const int i = s / p.n_slabs;
      if (p.meta_direct && i >= 2 && s == i * p.n_slabs) {
        // Metadata buffer (i & 1) is free once tile i - 2 is consumed, i.e.
        // its last stage t is released. For t <= s - S the ring wait above
        // already implied it (stages are released in order); otherwise t's
        // slot is still on its phase for stage t.
        const int t = (i - 1) * p.n_slabs - 1;
        if (t > s - S && !warp_wait(&empty[t % S], (t / S) & 1)) break;
      }
      issue_stage(s, true);
    }
    // Drain: every copy issued by this warp has landed before the CTA exits.
    for (int t = max(0, s - S); t < s; ++t) mbar_wait(&full_w[t % S], (t / S) & 1);
    if (p.meta_direct) {
      const int issued_tiles = (s + p.n_slabs - 1) / p.n_slabs;
      for (int ii = max(0, issued_tiles - 2); ii < issued_tiles; ++ii)
        mbar_wait(&meta_full[ii & 1], (ii >> 1) & 1);
    }
  } else if (warp <= kNAux) {
    // ----------------------------------------------------------------- aux
    // The kNAux warps process every stage together and strictly in order,
    // each taking a quarter of the rows, words and step sums. (In-order
    // processing is what makes every parity wait below unambiguous: when a
    // warp waits for stage t's phase, stage t - S is known to be consumed.)
    const int a = warp - 1;
    const int at = a * 32 + lane;  // 0 .. kNAux*32 - 1
    constexpr int kAT = kNAux * 32;
    if constexpr (XRES) {
      // Activations, permuted once for the whole K (every tile of this CTA
      // reads them), plus their per-step sums. They may come from the
      // previous grid. One (row, step) unit per thread: its loads are all in
      // flight together.
      pdl_wait_prior_grid();
      const int gsteps = p.K / SC;
      for (int e = at; e < p.M * gsteps; e += kAT) {
        const int n = e / gsteps;
        const int gs = e - n * gsteps;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x + static_cast<int64_t>(n) * p.K +
                                                              static_cast<int64_t>(gs) * SC);
        uint8_t* dst = smem + p.off_xres + n * p.xp_pitch + gs * STEP_XB;
        reinterpret_cast<float*>(smem + p.off_sxres)[n * gsteps + gs] =
            process_step<BITS, INTER, WPL>(src, dst);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);
    }
    for (int s = 0; s < total; ++s) {
      const int i = s / p.n_slabs, j = s - (s / p.n_slabs) * p.n_slabs;
      const int r0 = (t_begin + i) * kTile;
      const int R = min(kTile, p.N - r0);
      const int slot = s % S;
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      const int G0 = k0 / p.gsize;
      const int koff = k0 - G0 * p.gsize;
      const int gps = (koff + L - 1) / p.gsize + 1;
      if (s >= S && !warp_wait(&empty[slot], ((s / S) - 1) & 1)) return;
      const uint16_t* ms = reinterpret_cast<const uint16_t*>(smem + p.off_meta +
                                                              (i & 1) * p.meta_stride);
      const uint16_t* mz = ms + p.meta_stride / 4;
      int64_t in_smem = 0;
      if (p.meta_direct) {
        // meta_full[i & 1] completes once per tile using that buffer. Before
        // waiting on it by parity, make sure its previous user (tile i - 2)
        // finished, or the test would pass on the old phase: wait until tile
        // i - 2's last stage t is released (implied by the wait above when
        // t <= s - S).
        if (i >= 2) {
          const int t = (i - 1) * p.n_slabs - 1;
          if (t > s - S && !warp_wait(&empty[t % S], (t / S) & 1)) return;
        }
        if (!warp_wait(&meta_full[i & 1], (i >> 1) & 1)) return;
        in_smem = (static_cast<int64_t>(R) * p.G * 2 & ~15ll) / 2;
      }
      uint8_t* st = smem + slot * p.stage_bytes;
      uint2* ent = reinterpret_cast<uint2*>(st + p.off_ent);
      // Per (row, group): K0 = -(1024 + z') (fp16), the residual d = z' - z
      // (fp16, exact) and the fp32 scale, with z' = clamp(rint(z), +-1024).
      bool flag = false;
      for (int r = a; r < R; r += kNAux) {
        for (int gl = lane; gl < gps; gl += 32) {
          const int64_t li = static_cast<int64_t>(r) * p.G + G0 + gl;
          const int64_t gi = static_cast<int64_t>(r0) * p.G + li;
          const uint16_t sh = li < in_smem ? ms[li] : __ldg(p.scales + gi);
          float zf, zc;
          if constexpr (SYM) {
            zf = zc = static_cast<float>(BIAS);
          } else {
            const uint16_t zh = li < in_smem ? mz[li] : __ldg(p.zeros + gi);
            zf = __half2float(__ushort_as_half(zh));
            zc = fminf(fmaxf(rintf(zf), -1024.f), 1024.f);
          }
          const float d = zc - zf;
          const uint32_t k0h = __half_as_ushort(__float2half_rn(-(1024.f + zc)));
          const uint32_t dh = __half_as_ushort(__float2half_rn(d));
          ent[r * p.ep + gl] = make_uint2(k0h | (dh << 16),
                                          __float_as_uint(__half2float(__ushort_as_half(sh))));
          flag |= (d != 0.f);  // NaN compares unequal, so a NaN zero takes this path too
        }
      }
      flag = __any_sync(0xffffffffu, flag);

      if constexpr (!XRES) {
        // Activations for this slab: wait for the raw copy, then permute it
        // and take the per-step sums, one (row, step) unit per thread.
        if (!warp_wait(&full_w[slot], (s / S) & 1)) return;
        const int steps = L / SC;
        for (int e = at; e < p.M * steps; e += kAT) {
          const int n = e / steps;
          const int stp = e - n * steps;
          const uint8_t* src = st + p.off_xraw + n * (p.KS * 2) + stp * SC * 2;
          uint8_t* dst = st + p.off_xperm + n * p.xp_pitch + stp * STEP_XB;
          reinterpret_cast<float*>(st + p.off_sx)[n * p.steps_max + stp] =
              process_step<BITS, INTER, WPL>(src, dst);
        }
      }
      if (lane == 0) reinterpret_cast<int*>(st + p.off_flag)[a] = flag ? 1 : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_aux[slot]);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1 - kNAux;
    const int gid = lane >> 2;
    const int c = lane & 3;
    const bool has_x = gid < p.M;
    if constexpr (XRES) {
      if (!warp_wait(x_ready, 0)) return;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int s = 0;
    for (int i = 0; i < t_end - t_begin; ++i) {
      const int r0 = (t_begin + i) * kTile;
      const int R = min(kTile, p.N - r0);
      for (int j = 0; j < p.n_slabs; ++j, ++s) {
        const int slot = s % S;
        const uint32_t par = (s / S) & 1;
        if (!warp_wait(&full_w[slot], par) || !warp_wait(&full_aux[slot], par)) return;
        const int k0 = j * p.KS;
        const int L = min(p.KS, p.K - k0);
        const int steps = L / SC;
        const int G0 = k0 / p.gsize;
        const int koff_s = (k0 - G0 * p.gsize) / SC;
        const uint8_t* st = smem + slot * p.stage_bytes;
        const int4 flags = *reinterpret_cast<const int4*>(st + p.off_flag);
        const bool flag = (flags.x | flags.y | flags.z | flags.w) != 0;
        const float* sxs = XRES ? reinterpret_cast<const float*>(smem + p.off_sxres) + k0 / SC
                                : reinterpret_cast<const float*>(st + p.off_sx);
        const int sx_pitch = XRES ? p.K / SC : p.steps_max;
        const uint8_t* xrow = XRES ? smem + p.off_xres + gid * p.xp_pitch + (k0 / SC) * STEP_XB
                                   : st + p.off_xperm + gid * p.xp_pitch;
        const uint8_t* wrow_a = st + p.off_w + gid * p.w_pitch;
        const uint8_t* wrow_b = wrow_a + 8 * p.w_pitch;
        const uint2* ent = reinterpret_cast<const uint2*>(st + p.off_ent);

        // Steps go to warps by their global index along K, so each warp sums
        // the same steps in the same order however K is cut into slabs: the
        // result of a row does not depend on the slab length (nor on M).
        const int first = (cw - (k0 / SC) % kNCW + kNCW) % kNCW;
        for (int stp = first; stp < steps; stp += kNCW) {
          const int gl = static_cast<int>(fast_div(koff_s + stp, p.gq_magic));
          // B fragments: this lane's activation row (gid) at its k positions.
          uint32_t bx[WPL * NPAIR];
          if (has_x) {
            const uint8_t* xp = xrow + stp * STEP_XB + c * U;
#pragma unroll
            for (int u = 0; u < NU; ++u) Vec<U>::ld(xp + u * 4 * U, bx + u * (U / 4));
          } else {
#pragma unroll
            for (int q = 0; q < WPL * NPAIR; ++q) bx[q] = 0u;
          }
          const int wofs = (stp * 4 * WPL + c * WPL) * 4;
          uint32_t wa[WPL], wb[WPL];
          Vec<WPL * 4>::ld(wrow_a + wofs, wa);
          Vec<WPL * 4>::ld(wrow_b + wofs, wb);
          const uint2 ea = ent[gid * p.ep + gl];
          const uint2 eb = ent[(gid + 8) * p.ep + gl];
          const uint32_t k0a = prmt(ea.x, ea.x, 0x1010u);  // K0 in both halves
          const uint32_t k0b = prmt(eb.x, eb.x, 0x1010u);
          const uint32_t k1a = BITS == 2 ? hadd2_u32(k0a, kH768) : 0u;
          const uint32_t k1b = BITS == 2 ? hadd2_u32(k0b, kH768) : 0u;
          const uint32_t k2a = BITS != 8 ? hadd2_u32(k0a, kH960) : 0u;
          const uint32_t k2b = BITS != 8 ? hadd2_u32(k0b, kH960) : 0u;
          // Two independent accumulator chains halve the dependent-MMA latency.
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int jj = 0; jj < WPL; ++jj) {
            uint32_t pa[NPAIR], pb[NPAIR];
            unpack_pairs<BITS>(wa[jj], k0a, k1a, k2a, pa);
            unpack_pairs<BITS>(wb[jj], k0b, k1b, k2b, pb);
#pragma unroll
            for (int q = 0; q < NPAIR / 2; ++q) {
              float* chain = ((jj * (NPAIR / 2) + q) & 1) ? e : d;
              mma_16816(chain, pa[2 * q], pb[2 * q], pa[2 * q + 1], pb[2 * q + 1],
                        bx[jj * NPAIR + 2 * q], bx[jj * NPAIR + 2 * q + 1]);
            }
          }
          const float sa = __uint_as_float(ea.y);
          const float sb = __uint_as_float(eb.y);
          acc[0] = fmaf(sa, d[0] + e[0], acc[0]);
          acc[1] = fmaf(sa, d[1] + e[1], acc[1]);
          acc[2] = fmaf(sb, d[2] + e[2], acc[2]);
          acc[3] = fmaf(sb, d[3] + e[3], acc[3]);
          if (flag) {
            // Residual of out-of-range or fractional zero-points, in fp32.
            const float xa = (2 * c < p.M) ? sxs[(2 * c) * sx_pitch + stp] : 0.f;
            const float xb = (2 * c + 1 < p.M) ? sxs[(2 * c + 1) * sx_pitch + stp] : 0.f;
            const float qa = sa * __half2float(__ushort_as_half(static_cast<uint16_t>(ea.x >> 16)));
            const float qb = sb * __half2float(__ushort_as_half(static_cast<uint16_t>(eb.x >> 16)));
            acc[0] = fmaf(qa, xa, acc[0]);
            acc[1] = fmaf(qa, xb, acc[1]);
            acc[2] = fmaf(qb, xa, acc[2]);
            acc[3] = fmaf(qb, xb, acc[3]);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }

      // Tile done: fixed-order reduction across the consumer warps.
      const int buf = i & 1;
      float* red = reinterpret_cast<float*>(smem + p.off_red) + buf * (kNCW * kTile * kMaxM);
      float* rw = red + (cw * kTile + gid) * kMaxM + 2 * c;
      *reinterpret_cast<float2*>(rw) = make_float2(acc[0], acc[1]);
      *reinterpret_cast<float2*>(rw + 8 * kMaxM) = make_float2(acc[2], acc[3]);
      acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      mbar_arrive(&red_bar[buf]);
      if (!warp_wait(&red_bar[buf], (i >> 1) & 1)) return;
      for (int idx = cw * 32 + lane; idx < kTile * p.M; idx += kNCW * 32) {
        const int row = idx & (kTile - 1);
        const int col = idx / kTile;
        if (row < R) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kNCW; ++w) sum += red[(w * kTile + row) * kMaxM + col];
          p.y[static_cast<int64_t>(col) * p.N + r0 + row] = __half_as_ushort(__float2half_rn(sum));
        }
      }
    }
  }
}

// ------------------------------------------------------------------- host

namespace {

int round_up(int v, int m) { return (v + m - 1) / m * m; }

template <int BITS, bool SYM, bool INTER, int WPL, bool XRES>
cudaError_t launch_variant(const GemvParams& p, int grid, int smem, cudaStream_t stream) {
  auto kern = gemv_kernel<BITS, SYM, INTER, WPL, XRES>;
  static int configured[64] = {0};  // max dynamic smem already raised, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: this grid may start while the previous
  // one drains; the kernel waits for it before touching activations.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, bool SYM, bool INTER, int WPL>
cudaError_t dispatch_x(bool xres, const GemvParams& p, int grid, int smem, cudaStream_t stream) {
  return xres ? launch_variant<BITS, SYM, INTER, WPL, true>(p, grid, smem, stream)
              : launch_variant<BITS, SYM, INTER, WPL, false>(p, grid, smem, stream);
}

template <int BITS, bool SYM, bool INTER>
cudaError_t dispatch_wpl(int wpl, bool xres, const GemvParams& p, int grid, int smem,
                         cudaStream_t stream) {
  switch (wpl) {
    case 4: return dispatch_x<BITS, SYM, INTER, 4>(xres, p, grid, smem, stream);
    case 2: return dispatch_x<BITS, SYM, INTER, 2>(xres, p, grid, smem, stream);
    default: return dispatch_x<BITS, SYM, INTER, 1>(xres, p, grid, smem, stream);
  }
}

}  // namespace

cudaError_t read_device_status(int device, uint32_t* status, bool reset) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return e;
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) return e;
  cudaError_t (*readers[])(uint32_t*, bool) = {read_status_gemv, read_status_stream_b2,
                                                read_status_stream_b4, read_status_stream_b8,
                                                read_status_peer,        read_status_direct_b2,
                                                read_status_direct_b4,   read_status_direct_b8};
  *status = 0;
  for (auto rd : readers) {
    uint32_t v = 0;
    e = rd(&v, reset);
    if (e != cudaSuccess) break;
    *status |= v;
  }
  if (prev != device) cudaSetDevice(prev);
  return e;
}

int gemv_words_per_lane(int bits, int group_size, int K) {
  const int pp = 32 / bits;
  for (int wpl = 4; wpl >= 1; wpl >>= 1) {
    const int sc = 4 * wpl * pp;
    if (group_size % sc == 0 && K % sc == 0) return wpl;
  }
  return 0;
}

bool plan_gemv(int M, int N, int K, int bits, int group_size, int num_sms, GemvPlan* plan) {
  const int pp = 32 / bits;
  const int wpl = gemv_words_per_lane(bits, group_size, K);
  if (wpl == 0 || num_sms <= 0) return false;
  const int sc = 4 * wpl * pp;
  const int lxb = wpl * pp * 2;
  const int u = lxb >= 16 ? 16 : lxb;
  const int xpad = u == 16 ? 64 : 32;
  const int G = K / group_size;
  const int64_t row_bytes = static_cast<int64_t>(K) * bits / 8;
  // Activations resident for the whole K when they fit.
  const int xres_pitch = round_up(K * 2, 128) + xpad;
  const bool xres = static_cast<int64_t>(M) * xres_pitch <= kMaxXresBytes;
  // Slabs: split K so that a 16-row stage holds about kStageBytes of packed
  // weights (long per-row runs), in whole steps; with per-stage activations,
  // also keep their raw + permuted copies within kXStageBytes. (The result
  // does not depend on the slab length: steps go to warps by global index.)
  int n_slabs = static_cast<int>((kTile * row_bytes + kStageBytes - 1) / kStageBytes);
  if (n_slabs < 1) n_slabs = 1;
  int ks = round_up((K + n_slabs - 1) / n_slabs, sc);
  if (!xres) {
    int ks_x = (kXStageBytes / (4 * M)) / sc * sc;
    if (ks_x < sc) ks_x = sc;
    if (ks > ks_x) ks = ks_x;
  }
  if (ks > K) ks = K;
  n_slabs = (K + ks - 1) / ks;
  int gps_max = (ks % group_size == 0) ? ks / group_size : (ks + group_size - 1) / group_size + 1;
  if (gps_max > G) gps_max = G;
  if (gps_max < 1) gps_max = 1;
  const int ep = gps_max | 1;  // odd entry stride per row: conflict-free row reads
  GemvPlan pl;
  pl.wpl = wpl;
  pl.ks = ks;
  pl.n_slabs = n_slabs;
  pl.ep = ep;
  pl.steps_max = ks / sc;
  pl.xres = xres ? 1 : 0;
  pl.w_pitch = round_up(ks * bits / 8, 128) + 16 * wpl;
  pl.xp_pitch = xres ? xres_pitch : round_up(ks * 2, 128) + xpad;
  int off = 0;
  pl.off_w = off;
  off += kTile * pl.w_pitch;
  pl.off_xraw = off;
  if (!xres) off += round_up(M * ks * 2, 128);
  pl.off_xperm = off;
  if (!xres) off += round_up(M * pl.xp_pitch, 128);
  pl.off_ent = off;
  off += round_up(kTile * ep * 8, 128);
  pl.off_sx = off;
  if (!xres) off += round_up(M * pl.steps_max * 4, 128);
  pl.off_flag = off;
  off += 128;
  pl.stage_bytes = off;
  // Two tile metadata buffers, each [scales span | zeros span] of 16 rows x G.
  const int span = round_up(kTile * G * 2, 128);
  pl.meta_stride = 2 * span;
  pl.meta_direct = 2 * pl.meta_stride <= kMaxMetaBytes ? 1 : 0;
  const int meta_bytes = pl.meta_direct ? 2 * pl.meta_stride : 0;
  const int sxres_bytes = xres ? round_up(M * (K / sc) * 4, 128) : 0;
  const int xres_bytes = xres ? round_up(M * xres_pitch, 128) + sxres_bytes : 0;
  const int fixed = kRedBytes + kBarBytes + meta_bytes + xres_bytes;
  int stages = (kMaxSmemBytes - fixed) / off;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  pl.stages = stages;
  pl.off_xres = stages * off;
  pl.off_sxres = pl.off_xres + (xres ? round_up(M * xres_pitch, 128) : 0);
  pl.off_meta = pl.off_xres + xres_bytes;
  pl.off_red = pl.off_meta + meta_bytes;
  pl.off_bar = pl.off_red + kRedBytes;
  pl.smem = pl.off_bar + kBarBytes;
  const int tiles = (N + kTile - 1) / kTile;
  pl.grid = tiles < num_sms ? tiles : num_sms;
  *plan = pl;
  return true;
}

cudaError_t launch_gemv(const GemvArgs& a, const GemvPlan& pl, cudaStream_t stream) {
  GemvParams p;
  p.x = a.x;
  p.qw = a.qweight;
  p.scales = a.scales;
  p.zeros = a.zeros;
  p.y = a.y;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.G = a.K / a.group_size;
  p.gsize = a.group_size;
  p.KS = pl.ks;
  p.n_slabs = pl.n_slabs;
  p.stages = pl.stages;
  const int sc = 4 * pl.wpl * (32 / a.bits);
  const uint32_t gq = static_cast<uint32_t>(a.group_size / sc);
  p.gq_magic = gq <= 1 ? 0u : static_cast<uint32_t>((0x100000000ull + gq - 1) / gq);
  p.ep = pl.ep;
  p.steps_max = pl.steps_max;
  p.w_pitch = pl.w_pitch;
  p.xp_pitch = pl.xp_pitch;
  p.off_w = pl.off_w;
  p.off_xraw = pl.off_xraw;
  p.off_xperm = pl.off_xperm;
  p.off_ent = pl.off_ent;
  p.off_sx = pl.off_sx;
  p.off_flag = pl.off_flag;
  p.stage_bytes = pl.stage_bytes;
  p.off_xres = pl.off_xres;
  p.off_sxres = pl.off_sxres;
  p.off_meta = pl.off_meta;
  p.meta_stride = pl.meta_stride;
  // Metadata bulk copies need 16-byte-aligned tensors; otherwise the aux
  // warps read scales/zeros from global memory.
  p.meta_direct = pl.meta_direct && reinterpret_cast<uintptr_t>(a.scales) % 16 == 0 &&
                  (a.zeros == nullptr || reinterpret_cast<uintptr_t>(a.zeros) % 16 == 0);
  p.off_red = pl.off_red;
  p.off_bar = pl.off_bar;

#define DQG_GEMV_CASE(B, S, I) \
  if (a.bits == B && a.symmetric == S && a.interleaved == I) \
    return dispatch_wpl<B, S, I>(pl.wpl, pl.xres != 0, p, pl.grid, pl.smem, stream);
  DQG_GEMV_CASE(2, false, false)
  DQG_GEMV_CASE(2, false, true)
  DQG_GEMV_CASE(2, true, false)
  DQG_GEMV_CASE(2, true, true)
  DQG_GEMV_CASE(4, false, false)
  DQG_GEMV_CASE(4, false, true)
  DQG_GEMV_CASE(4, true, false)
  DQG_GEMV_CASE(4, true, true)
  DQG_GEMV_CASE(8, false, false)
  DQG_GEMV_CASE(8, false, true)
  DQG_GEMV_CASE(8, true, false)
  DQG_GEMV_CASE(8, true, true)
#undef DQG_GEMV_CASE
  return cudaErrorInvalidValue;
}

}  // namespace dqg

DQG_STATUS_READER(read_status_gemv)
