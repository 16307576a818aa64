// Fused low-bit dequantize + GEMV for B200 (sm_100a).
//
// y[m, n] = fp16( sum_k x[m, k] * (q[n, k] - off[n, k/g]) * scale[n, k/g] ),
// fp32 accumulation, for 1 <= M <= 8 activation rows, with the packed format of
// the reference packer (KrishnaI2424/Dequant_Project dequant/packer.py:7-29):
// int32 words of 32/bits unsigned codes, fp16 scales [N, K/g] and, when
// asymmetric, fp16 zero-points [N, K/g]; off = 2^(bits-1) when symmetric.
// The reference kernel this replaces is kernels/dequant_gemv.cu:144-217.
//
// Design (one persistent CTA per SM, warp-specialised):
//   * Every CTA owns a contiguous range of output rows (balanced to within one
//     row), processed in row blocks of <= 32 rows and, inside a block, in
//     K slabs. One (row block, slab) pair is one pipeline stage.
//   * warp 0 streams the stage: one untiled bulk copy (cp.async.bulk, no
//     multicast) per packed row segment plus one per activation row, all
//     completing on the stage's mbarrier.
//   * warps 1..kNAux each own every kNAux-th stage: they turn scales and
//     zero-points into the fp16 constants the unpack needs, and rewrite x into
//     the k-order the unpack produces, so that the tensor-core B fragments are
//     plain shared-memory loads.
//   * warps kNAux+1.. (kNCW of them) unpack codes in registers and run
//     mma.m16n8k16 (fp16 x fp16 -> fp32) with the weight rows as the M=16 side
//     and the <= 8 activation rows as the N=8 side.
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

// Interleaved slot orders (dequant/packer.py:37-41): slot s of a word holds
// logical code order[s] of that word.
__host__ __device__ constexpr int slot_logical(int bits, bool inter, int s) {
  if (!inter) return s;
  if (bits == 4) {
    constexpr int o[8] = {0, 2, 4, 6, 1, 3, 5, 7};
    return o[s];
  }
  if (bits == 2) {
    constexpr int o[16] = {0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15};
    return o[s];
  }
  constexpr int o[4] = {0, 2, 1, 3};
  return o[s];
}

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

// Physical row (within a 16-row tile) held by MMA row slot g (and g + 8). The
// packed rows arrive through a 128-byte-swizzled TMA box, where 16-byte unit u
// of row r sits at unit u ^ (r & 7); this slot order makes the rows that one
// shared-memory wavefront serves land on disjoint units for each load width.
template <int WPL>
__device__ __forceinline__ int slot_row(int g) {
  if constexpr (WPL == 4) return (g >> 1) | ((g & 1) << 2);   // 0 4 1 5 2 6 3 7
  else if constexpr (WPL == 2) return ((g & 3) << 1) | (g >> 2);  // 0 2 4 6 1 3 5 7
  else return g;
}

// Byte offset of packed byte `wb` of tile row `rl` (0..15) in the stage's W
// area, laid out as boxes [chunk q][tile h][16 rows x 128 B], swizzled.
__device__ __forceinline__ int w_offset(int h, int rl, int wb) {
  const int q = wb >> 7;
  const int u = (wb >> 4) & 7;
  return ((q * 2 + h) << 11) + (rl << 7) + ((u ^ (rl & 7)) << 4) + (wb & 15);
}

template <int BITS, bool SYM, bool INTER, int WPL>
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

  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled TMA boxes need 1024-byte aligned destinations.
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full_w = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* full_aux = full_w + kMaxStages;
  uint64_t* empty = full_aux + kMaxStages;
  uint64_t* red_bar = empty + kMaxStages;
  uint64_t* meta_full = red_bar + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = p.stages;

  // This CTA's tiles (16 rows each, aligned), grouped in row blocks of two.
  const int T = (p.N + kTile - 1) / kTile;
  const int t_begin = static_cast<int>(static_cast<int64_t>(T) * blockIdx.x / gridDim.x);
  const int t_end = static_cast<int>(static_cast<int64_t>(T) * (blockIdx.x + 1) / gridDim.x);
  const int n_rb = (t_end - t_begin + 1) / 2;
  const int total = n_rb * p.n_slabs;
  auto block_rows = [&](int b, int& r0, int& R, int& ntb) {
    const int t0 = t_begin + 2 * b;
    ntb = min(2, t_end - t0);
    r0 = t0 * kTile;
    R = min(ntb * kTile, p.N - r0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&full_aux[s], 1);
      mbar_init(&empty[s], kNCW);
    }
    mbar_init(&red_bar[0], kNCW * 32);
    mbar_init(&red_bar[1], kNCW * 32);
    mbar_init(&meta_full[0], 1);
    mbar_init(&meta_full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int64_t span_elems = static_cast<int64_t>(p.G);
    // Scales/zeros of a row block: rows [r0, r0 + R) x all groups are one
    // contiguous span; r0 is a multiple of 16, so it starts 16-byte aligned.
    // The 16-byte-aligned prefix comes by bulk copy, the rest (only in the
    // matrix's last partial tile) is read by the aux warps.
    auto issue_meta = [&](int b) {
      int r0, R, ntb;
      block_rows(b, r0, R, ntb);
      const uint32_t bytes = static_cast<uint32_t>(R * span_elems * 2) & ~15u;
      uint8_t* dst = smem + p.off_meta + (b & 1) * p.meta_stride;
      if (lane == 0)
        mbar_arrive_expect_tx(&meta_full[b & 1], SYM ? bytes : 2 * bytes);
      __syncwarp();
      if (bytes) {
        if (lane == 0)
          bulk_g2s(dst, p.scales + static_cast<int64_t>(r0) * span_elems, bytes, &meta_full[b & 1],
                   pol_x);
        if (!SYM && lane == 1)
          bulk_g2s(dst + p.meta_stride / 2, p.zeros + static_cast<int64_t>(r0) * span_elems, bytes,
                   &meta_full[b & 1], pol_x);
      }
    };
    auto issue_w = [&](int s, bool with_x) {
      const int b = s / p.n_slabs, j = s - (s / p.n_slabs) * p.n_slabs;
      int r0, R, ntb;
      block_rows(b, r0, R, ntb);
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      const int nch = (L * BITS / 8 + 127) >> 7;
      const int slot = s % S;
      uint8_t* st = smem + slot * p.stage_bytes;
      if (p.meta_direct && j == 0) issue_meta(b);
      if (lane == 0)
        mbar_arrive_expect_tx(&full_w[slot],
                              static_cast<uint32_t>(ntb * nch * 2048 + p.M * L * 2));
      __syncwarp();
      if (lane < nch * ntb) {
        const int q = lane / ntb, h = lane - (lane / ntb) * ntb;
        tma_load_2d(st + p.off_w + ((q * 2 + h) << 11), &p.tmap, k0 / PP + 32 * q,
                    r0 + kTile * h, &full_w[slot], pol_w);
      }
      (void)R;
      if (with_x && lane < p.M)
        bulk_g2s(st + p.off_xraw + lane * p.xraw_pitch, p.x + static_cast<int64_t>(lane) * p.K + k0,
                 static_cast<uint32_t>(L) * 2, &full_w[slot], pol_x);
    };
    auto issue_x = [&](int s) {
      const int j = s % p.n_slabs;
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      uint8_t* st = smem + (s % S) * p.stage_bytes;
      if (lane < p.M)
        bulk_g2s(st + p.off_xraw + lane * p.xraw_pitch, p.x + static_cast<int64_t>(lane) * p.K + k0,
                 static_cast<uint32_t>(L) * 2, &full_w[s % S], pol_x);
    };
    // A stage needs no wait if its slot is fresh and, when it starts a row
    // block, that block's metadata buffer is fresh too (blocks 0 and 1).
    int pre = min(S, total);
    if (p.meta_direct) pre = min(pre, 2 * p.n_slabs);
    // Packed weights and their metadata do not depend on the previous grid:
    // stream the first stages before waiting for it; activations only after.
    for (int s = 0; s < pre; ++s) issue_w(s, false);
    pdl_wait_prior_grid();
    for (int s = 0; s < pre; ++s) issue_x(s);
    int s = pre;
    for (; s < total; ++s) {
      const int slot = s % S;
      if (s >= S && !warp_wait(&empty[slot], ((s / S) - 1) & 1)) break;
      const int b = s / p.n_slabs;
      if (p.meta_direct && b >= 2 && s == b * p.n_slabs) {
        // Metadata buffer (b & 1) is free once block b - 2 is fully consumed,
        // i.e. its last stage t is released. When t <= s - S the ring wait
        // above already implied that (stages are released in order); only
        // otherwise is t's slot still on its phase for stage t.
        const int t = (b - 1) * p.n_slabs - 1;
        if (t > s - S && !warp_wait(&empty[t % S], (t / S) & 1)) break;
      }
      issue_w(s, true);
    }
    // Drain: every copy issued by this warp has landed before the CTA can exit.
    for (int t = max(0, s - S); t < s; ++t) mbar_wait(&full_w[t % S], (t / S) & 1);
    if (p.meta_direct) {
      const int nb_issued = (s + p.n_slabs - 1) / p.n_slabs;
      for (int bb = max(0, nb_issued - 2); bb < nb_issued; ++bb)
        mbar_wait(&meta_full[bb & 1], (bb >> 1) & 1);
    }
  } else if (warp <= kNAux) {
    // ----------------------------------------------------------------- aux
    const int a = warp - 1;
    for (int s = a; s < total; s += kNAux) {
      const int b = s / p.n_slabs, j = s - (s / p.n_slabs) * p.n_slabs;
      int r0, R, ntb;
      block_rows(b, r0, R, ntb);
      const int slot = s % S;
      const int k0 = j * p.KS;
      const int L = min(p.KS, p.K - k0);
      const int G0 = k0 / p.gsize;
      const int koff = k0 - G0 * p.gsize;
      const int gps = (koff + L - 1) / p.gsize + 1;
      const int n_ent = R * gps;
      const uint32_t gps_magic =
          gps == 1 ? 0u : static_cast<uint32_t>((0x100000000ull + gps - 1) / gps);
      uint16_t sv[kMaxEntPerLane], zv[kMaxEntPerLane];
      if (p.meta_direct) {
        // This row block's scales/zeros are in shared memory (bulk copy).
        if (!warp_wait(&meta_full[b & 1], (b >> 1) & 1)) return;
        const uint16_t* ms = reinterpret_cast<const uint16_t*>(smem + p.off_meta +
                                                                (b & 1) * p.meta_stride);
        const uint16_t* mz = ms + p.meta_stride / 4;
        const int64_t in_smem = (static_cast<int64_t>(R) * p.G * 2 & ~15ll) / 2;
#pragma unroll
        for (int i = 0; i < kMaxEntPerLane; ++i) {
          const int e = lane + 32 * i;
          if (e < n_ent) {
            const int r = static_cast<int>(fast_div(e, gps_magic));
            const int gl = e - r * gps;
            const int64_t li = static_cast<int64_t>(r) * p.G + G0 + gl;
            const int64_t idx = static_cast<int64_t>(r0) * p.G + li;
            sv[i] = li < in_smem ? ms[li] : __ldg(p.scales + idx);
            if constexpr (!SYM) zv[i] = li < in_smem ? mz[li] : __ldg(p.zeros + idx);
          }
        }
      } else {
        // Scales and zero-points are weights: fetch them before waiting for
        // the slot, so that their latency overlaps the wait.
#pragma unroll
        for (int i = 0; i < kMaxEntPerLane; ++i) {
          const int e = lane + 32 * i;
          if (e < n_ent) {
            const int r = static_cast<int>(fast_div(e, gps_magic));
            const int gl = e - r * gps;
            const int64_t idx = static_cast<int64_t>(r0 + r) * p.G + G0 + gl;
            sv[i] = __ldg(p.scales + idx);
            if constexpr (!SYM) zv[i] = __ldg(p.zeros + idx);
          }
        }
      }
      if (s >= S && !warp_wait(&empty[slot], ((s / S) - 1) & 1)) return;
      uint8_t* st = smem + slot * p.stage_bytes;
      bool flag = false;
#pragma unroll
      for (int i = 0; i < kMaxEntPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < n_ent) {
          const int r = static_cast<int>(fast_div(e, gps_magic));
          const int gl = e - r * gps;
          float zf, zc;
          if constexpr (SYM) {
            zf = zc = static_cast<float>(BIAS);
          } else {
            zf = __half2float(__ushort_as_half(zv[i]));
            zc = fminf(fmaxf(rintf(zf), -1024.f), 1024.f);
          }
          const float d = zc - zf;
          const float scale = __half2float(__ushort_as_half(sv[i]));
          const uint32_t h0 = __half_as_ushort(__float2half_rn(-(1024.f + zc)));
          const uint32_t h1 = __half_as_ushort(__float2half_rn(-(256.f + zc)));
          const uint32_t h2 = __half_as_ushort(__float2half_rn(-(64.f + zc)));
          uint4 ent;
          ent.x = h0 | (h0 << 16);
          ent.y = h1 | (h1 << 16);
          ent.z = h2 | (h2 << 16);
          ent.w = __float_as_uint(scale);
          // [group][row] layout: the 8 rows one consumer load reads are
          // 8 consecutive 16-byte entries (no bank conflicts).
          reinterpret_cast<uint4*>(st + p.off_const)[gl * kRowBlock + r] = ent;
          reinterpret_cast<float*>(st + p.off_corr)[gl * kRowBlock + r] = scale * d;
          flag |= (d != 0.f);  // NaN compares unequal, so a NaN zero takes this path too
        }
      }
      flag = __any_sync(0xffffffffu, flag);

      // Activations: wait for the raw slab, rewrite it in unpack order.
      if (!warp_wait(&full_w[slot], (s / S) & 1)) return;
      const int words = L / PP;
      for (int n = 0; n < p.M; ++n) {
        const uint8_t* xr = st + p.off_xraw + n * p.xraw_pitch;
        uint8_t* xp = st + p.off_xperm + n * p.xperm_pitch;
        for (int wi = lane; wi < words; wi += 32) {
          uint32_t v[NPAIR];  // natural order: v[i] = (x[2i], x[2i+1])
          Vec<WB>::ld(xr + wi * WB, v);
          uint32_t o[NPAIR];
#pragma unroll
          for (int t = 0; t < NPAIR; ++t) {
            const int lo = slot_logical(BITS, INTER, t);
            const int hi = slot_logical(BITS, INTER, t + NPAIR);
            // low half <- x[lo] from v[lo/2], high half <- x[hi] from v[hi/2]
            o[t] = prmt(v[lo >> 1], v[hi >> 1],
                        ((lo & 1) ? 0x32u : 0x10u) | ((hi & 1) ? 0x7600u : 0x5400u));
          }
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
                    make_uint4(o[piece * 4 + 0], o[piece * 4 + 1], o[piece * 4 + 2],
                               o[piece * 4 + 3]);
              } else {
                *reinterpret_cast<uint2*>(base + u * 4 * U) = make_uint2(o[0], o[1]);
              }
            }
          } else {
            // WB == 8 < U == 16: two words share one 16-byte unit.
            const int u = (jj * WB) / U;
            *reinterpret_cast<uint2*>(base + u * 4 * U + (jj * WB) % U) = make_uint2(o[0], o[1]);
          }
        }
      }
      if (flag) {
        // Per-step activation sums for the zero-point residual.
        const int steps = L / SC;
        for (int e = lane; e < p.M * steps; e += 32) {
          const int n = e / steps;
          const int stp = e - n * steps;
          const __half* xr =
              reinterpret_cast<const __half*>(st + p.off_xraw + n * p.xraw_pitch) + stp * SC;
          float sum = 0.f;
          for (int k = 0; k < SC; ++k) sum += __half2float(xr[k]);
          reinterpret_cast<float*>(st + p.off_sx)[n * p.steps_max + stp] = sum;
        }
      }
      if (lane == 0) *reinterpret_cast<int*>(st + p.off_flag) = flag ? 1 : 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_aux[slot]);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1 - kNAux;
    const int gid = lane >> 2;
    const int c = lane & 3;
    const int prow = slot_row<WPL>(gid);  // physical row of slot gid in a tile
    const bool has_x = gid < p.M;
    float acc[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;

    int s = 0;
    for (int b = 0; b < n_rb; ++b) {
      int r0, R, ntb;
      block_rows(b, r0, R, ntb);
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
        const bool flag = *reinterpret_cast<const volatile int*>(st + p.off_flag) != 0;

        for (int stp = cw; stp < steps; stp += kNCW) {
          const int gl = static_cast<int>(fast_div(koff_s + stp, p.gq_magic));
          // B fragments: this lane's activation row (gid) at its k positions.
          uint32_t bx[WPL * NPAIR];
          if (has_x) {
            const uint8_t* xp = st + p.off_xperm + gid * p.xperm_pitch + stp * STEP_XB + c * U;
#pragma unroll
            for (int u = 0; u < NU; ++u) Vec<U>::ld(xp + u * 4 * U, bx + u * (U / 4));
          } else {
#pragma unroll
            for (int i = 0; i < WPL * NPAIR; ++i) bx[i] = 0u;
          }
          const int wb = (stp * 4 * WPL + c * WPL) * 4;
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int ra = mt * kTile + prow;      // physical rows of slots gid, gid + 8
            const int rbw = ra + 8;
            uint32_t wa[WPL], wbv[WPL];
            Vec<WPL * 4>::ld(st + p.off_w + w_offset(mt, prow, wb), wa);
            Vec<WPL * 4>::ld(st + p.off_w + w_offset(mt, prow + 8, wb), wbv);
            const uint4 ca = reinterpret_cast<const uint4*>(st + p.off_const)[gl * kRowBlock + ra];
            const uint4 cb = reinterpret_cast<const uint4*>(st + p.off_const)[gl * kRowBlock + rbw];
            // Two independent accumulator chains (even / odd MMAs) halve the
            // dependent-MMA latency of a step; summed once at the end.
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            float e[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int jj = 0; jj < WPL; ++jj) {
              uint32_t pa[NPAIR], pb[NPAIR];
              unpack_pairs<BITS>(wa[jj], ca.x, ca.y, ca.z, pa);
              unpack_pairs<BITS>(wbv[jj], cb.x, cb.y, cb.z, pb);
#pragma unroll
              for (int i = 0; i < NPAIR / 2; ++i) {
                float* acc_chain = ((jj * (NPAIR / 2) + i) & 1) ? e : d;
                mma_16816(acc_chain, pa[2 * i], pb[2 * i], pa[2 * i + 1], pb[2 * i + 1],
                          bx[jj * NPAIR + 2 * i], bx[jj * NPAIR + 2 * i + 1]);
              }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) d[i] += e[i];
            const float sa = __uint_as_float(ca.w);
            const float sb = __uint_as_float(cb.w);
            acc[mt][0] = fmaf(sa, d[0], acc[mt][0]);
            acc[mt][1] = fmaf(sa, d[1], acc[mt][1]);
            acc[mt][2] = fmaf(sb, d[2], acc[mt][2]);
            acc[mt][3] = fmaf(sb, d[3], acc[mt][3]);
            if (flag) {
              const float* corr = reinterpret_cast<const float*>(st + p.off_corr);
              const float* sx = reinterpret_cast<const float*>(st + p.off_sx);
              const float xa = (2 * c < p.M) ? sx[(2 * c) * p.steps_max + stp] : 0.f;
              const float xb = (2 * c + 1 < p.M) ? sx[(2 * c + 1) * p.steps_max + stp] : 0.f;
              const float qa = corr[gl * kRowBlock + ra];
              const float qb = corr[gl * kRowBlock + rbw];
              acc[mt][0] = fmaf(qa, xa, acc[mt][0]);
              acc[mt][1] = fmaf(qa, xb, acc[mt][1]);
              acc[mt][2] = fmaf(qb, xa, acc[mt][2]);
              acc[mt][3] = fmaf(qb, xb, acc[mt][3]);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }

      // Row block done: fixed-order reduction across the consumer warps.
      const int buf = b & 1;
      float* red = reinterpret_cast<float*>(smem + p.off_red) + buf * (kNCW * kRowBlock * kMaxM);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float* rw = red + (cw * kRowBlock + mt * kTile + prow) * kMaxM + 2 * c;
        *reinterpret_cast<float2*>(rw) = make_float2(acc[mt][0], acc[mt][1]);
        *reinterpret_cast<float2*>(rw + 8 * kMaxM) = make_float2(acc[mt][2], acc[mt][3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
      }
      mbar_arrive(&red_bar[buf]);
      if (!warp_wait(&red_bar[buf], (b >> 1) & 1)) return;
      const int tc = cw * 32 + lane;
      for (int idx = tc; idx < kRowBlock * p.M; idx += kNCW * 32) {
        const int row = idx & (kRowBlock - 1);
        const int col = idx / kRowBlock;
        if (row < R) {
          float sum = 0.f;
#pragma unroll
          for (int w = 0; w < kNCW; ++w) sum += red[(w * kRowBlock + row) * kMaxM + col];
          p.y[static_cast<int64_t>(col) * p.N + r0 + row] = __half_as_ushort(__float2half_rn(sum));
        }
      }
    }
  }
}

// ------------------------------------------------------------------- host

namespace {

int round_up(int v, int m) { return (v + m - 1) / m * m; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

template <int BITS, bool SYM, bool INTER, int WPL>
cudaError_t launch_variant(const GemvParams& p, int grid, int smem, cudaStream_t stream) {
  auto kern = gemv_kernel<BITS, SYM, INTER, WPL>;
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

template <int BITS, bool SYM, bool INTER>
cudaError_t dispatch_wpl(int wpl, const GemvParams& p, int grid, int smem, cudaStream_t stream) {
  switch (wpl) {
    case 4: return launch_variant<BITS, SYM, INTER, 4>(p, grid, smem, stream);
    case 2: return launch_variant<BITS, SYM, INTER, 2>(p, grid, smem, stream);
    default: return launch_variant<BITS, SYM, INTER, 1>(p, grid, smem, stream);
  }
}

}  // namespace

cudaError_t read_device_status(int device, uint32_t* status, bool reset) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return e;
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(status, g_status, sizeof(uint32_t));
  if (e == cudaSuccess && reset) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(uint32_t));
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
  const int chunk_codes = 1024 / bits;  // codes in one 128-byte TMA box row
  const int budget = kMaxSmemBytes - kRedBytes - kBarBytes - kAlignSlack;
  // Slab length depends only on the format and K, never on M: the order in
  // which a row's products are summed is then the same for every batch size,
  // so each output row is bit-identical to the M = 1 call on that activation
  // row. Target 512 packed bytes per row per stage, in whole 128-byte boxes.
  int ks = 4096 / bits;
  while (ks > chunk_codes && (ks + group_size - 1) / group_size + 1 > kMaxEntPerLane)
    ks -= chunk_codes;
  if (ks > K) ks = K;
  if (ks % sc != 0) return false;
  const int G = K / group_size;
  int gps_max = (ks % group_size == 0) ? ks / group_size : (ks + group_size - 1) / group_size + 1;
  if (gps_max > G) gps_max = G;
  if (gps_max < 1) gps_max = 1;
  if (gps_max > kMaxEntPerLane) return false;
  GemvPlan pl;
  pl.wpl = wpl;
  pl.ks = ks;
  pl.gps_max = gps_max;
  pl.steps_max = ks / sc;
  pl.xraw_pitch = ks * 2;
  pl.xperm_pitch = round_up(ks * 2, 128) + (u == 16 ? 64 : 32);
  const int nch = (ks * bits / 8 + 127) / 128;
  // Two row-block metadata buffers, each [scales span | zeros span] of
  // 32 rows x G fp16 (the span is copied whole when it fits the budget).
  const int span = round_up(kRowBlock * G * 2, 128);
  const int meta_stride = 2 * span;
  const bool meta_direct = 2 * meta_stride <= kMaxMetaBytes;
  const int meta_bytes = meta_direct ? 2 * meta_stride : 0;
  int off = 0;
  pl.off_w = off;
  off += 2 * nch * 2048;
  pl.off_xraw = off;
  off += round_up(M * pl.xraw_pitch, 128);
  pl.off_xperm = off;
  off += round_up(M * pl.xperm_pitch, 128);
  pl.off_const = off;
  off += round_up(kRowBlock * gps_max * 16, 128);
  pl.off_corr = off;
  off += round_up(kRowBlock * gps_max * 4, 128);
  pl.off_sx = off;
  off += round_up(M * pl.steps_max * 4, 128);
  pl.off_flag = off;
  off += 128;
  off = round_up(off, 1024);
  pl.stage_bytes = off;
  int stages = (budget - meta_bytes) / off;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  pl.stages = stages;
  pl.meta_direct = meta_direct ? 1 : 0;
  pl.off_meta = stages * off;
  pl.meta_stride = meta_stride;
  pl.off_red = pl.off_meta + meta_bytes;
  pl.off_bar = pl.off_red + kRedBytes;
  pl.smem = pl.off_bar + kBarBytes + kAlignSlack;
  const int tiles = (N + kTile - 1) / kTile;
  pl.grid = tiles < num_sms ? tiles : num_sms;
  *plan = pl;
  return true;
}

cudaError_t launch_gemv(const GemvArgs& a, const GemvPlan& pl, cudaStream_t stream) {
  GemvParams p;
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return cudaErrorNotSupported;
  const cuuint64_t words = static_cast<cuuint64_t>(a.K) * a.bits / 32;
  const cuuint64_t dims[2] = {words, static_cast<cuuint64_t>(a.N)};
  const cuuint64_t strides[1] = {words * 4};
  const cuuint32_t box[2] = {32, kTile};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&p.tmap, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<uint32_t*>(a.qweight), dims,
          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
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
  p.n_slabs = (a.K + pl.ks - 1) / pl.ks;
  p.stages = pl.stages;
  const int sc = 4 * pl.wpl * (32 / a.bits);
  const uint32_t gq = static_cast<uint32_t>(a.group_size / sc);
  p.gq_magic = gq <= 1 ? 0u : static_cast<uint32_t>((0x100000000ull + gq - 1) / gq);
  p.gps_max = pl.gps_max;
  p.steps_max = pl.steps_max;
  p.xraw_pitch = pl.xraw_pitch;
  p.xperm_pitch = pl.xperm_pitch;
  p.off_w = pl.off_w;
  p.off_xraw = pl.off_xraw;
  p.off_xperm = pl.off_xperm;
  p.off_const = pl.off_const;
  p.off_corr = pl.off_corr;
  p.off_sx = pl.off_sx;
  p.off_flag = pl.off_flag;
  p.stage_bytes = pl.stage_bytes;
  p.off_red = pl.off_red;
  p.off_bar = pl.off_bar;
  // Metadata bulk copies need 16-byte-aligned tensors; otherwise the aux
  // warps read scales/zeros from global memory.
  p.meta_direct = pl.meta_direct && reinterpret_cast<uintptr_t>(a.scales) % 16 == 0 &&
                  (a.zeros == nullptr || reinterpret_cast<uintptr_t>(a.zeros) % 16 == 0);
  p.off_meta = pl.off_meta;
  p.meta_stride = pl.meta_stride;

#define DQG_GEMV_CASE(B, S, I) \
  if (a.bits == B && a.symmetric == S && a.interleaved == I) \
    return dispatch_wpl<B, S, I>(pl.wpl, p, pl.grid, pl.smem, stream);
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
