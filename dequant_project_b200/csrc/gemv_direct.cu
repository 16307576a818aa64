// Host side of the direct GEMV kernel (gemv_direct.cuh): shared-memory plan
// and launch. Variants are instantiated per bit width in gemv_direct_b{2,4,8}.cu.
#include <cstdint>
#include <cuda_runtime.h>

#include "gemv.h"

namespace dqg {

cudaError_t launch_direct_b2(int wpl, int gs, bool sym, bool inter, const DirectParams& p,
                             int grid, int smem, cudaStream_t stream);
cudaError_t launch_direct_b4(int wpl, int gs, bool sym, bool inter, const DirectParams& p,
                             int grid, int smem, cudaStream_t stream);
cudaError_t launch_direct_b8(int wpl, int gs, bool sym, bool inter, const DirectParams& p,
                             int grid, int smem, cudaStream_t stream);

#ifndef DQG_DIRECT_MAX_K
#define DQG_DIRECT_MAX_K 6144
#endif
#ifndef DQG_DIRECT_MIN_BITS
#define DQG_DIRECT_MIN_BITS 4
#endif

namespace {
int round_up(int v, int m) { return (v + m - 1) / m * m; }
}  // namespace

bool plan_direct(int M, int N, int K, int bits, int group_size, int num_sms, DirectPlan* plan,
                 bool fused) {
  if (M < 1 || M > kMaxM || N < 1 || num_sms < 1 || group_size <= 0 || K % group_size) return false;
  const int wpl = gemv_words_per_lane(bits, group_size, K);
  if (wpl == 0) return false;
  const int sc = 4 * wpl * (32 / bits);
  const int G = K / group_size;
  // Group-wise formats whose group is exactly one MMA step of the lane
  // layout (INT4 up to g128, INT2 up to g256, INT8 up to g64).
  if (G < 2 || group_size != sc) return false;
  // Measured on B200 against the streaming kernel, inside the Llama-2-7B
  // decode step (INT4 g128): with one CTA per SM (below) the direct kernel
  // takes batch 1 from 2.305 to 2.229 ms/token and batch 8 from 4.54 to 4.16;
  // on rows longer than 6144 codes and for 2-bit codes (4-byte copies per
  // lane) it is slower than the streaming kernel.
  if (bits < DQG_DIRECT_MIN_BITS || K > DQG_DIRECT_MAX_K) return false;
  (void)fused;
  int mp = 1;
  while (mp < M) mp <<= 1;
  const int gs = 8 / mp;
  DirectPlan pl;
  pl.wpl = wpl;
  pl.mp = mp;
  pl.gs = gs;
  pl.Gp = (G + gs - 1) / gs * gs;
  // Activation rows: 32 bytes past a 128-byte multiple, so that the eight
  // rows an M = 8 fragment load touches fall on distinct bank groups.
  pl.xp = round_up(K * 2, 128) + 32;
  int off = 0;
  pl.off_x = off;
  off += round_up(M * pl.xp, 128);
  pl.off_sx = off;
  off += round_up(M * G * 4, 128);
  // Zero block (one step of activations, at most 512 bytes), 64 bytes off
  // the activation rows' bank phase.
  pl.off_zero = off + 64;
  off += 640;
  pl.off_red = off;
  off += kDirectNW * 2 * kTile * 8 * 4;
  pl.off_tiles = off;
  off += 128;
  pl.off_ring = off;
  off += kDirectNW * kDirectRingBytes;
  pl.smem = off;
  if (pl.smem > kDirectMaxSmem) return false;
  // One CTA per SM: a smaller request lets the block scheduler put two CTAs
  // of one launch on one SM (and none on another), which halves those CTAs'
  // share of the SM and measured 2.23 -> 2.55 ms/token in the decode step.
  if (pl.smem < kDirectMinSmem) pl.smem = kDirectMinSmem;
  const int tiles = (N + kTile - 1) / kTile;
  pl.grid = tiles < num_sms ? tiles : num_sms;
  *plan = pl;
  return true;
}

cudaError_t launch_direct(const GemvArgs& a, const DirectPlan& pl, cudaStream_t stream,
                          const PeerGemvArgs* ar, bool swiglu) {
  DirectParams p;
  p.x = a.x;
  p.qw = a.qweight;
  p.scales = a.scales;
  p.zeros = a.zeros;
  p.y = a.y;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.G = a.K / a.group_size;
  p.Gp = pl.Gp;
  p.xp = pl.xp;
  p.off_x = pl.off_x;
  p.off_sx = pl.off_sx;
  p.off_zero = pl.off_zero;
  p.off_red = pl.off_red;
  p.off_tiles = pl.off_tiles;
  p.off_ring = pl.off_ring;
  p.prefetch = weight_prefetch() ? 1 : 0;
  p.swiglu = swiglu ? 1 : 0;
  if (swiglu && (a.N % kTile != 0 || (ar != nullptr && ar->world > 1)))
    return cudaErrorInvalidValue;
  p.ar_rank = 0;
  p.ar_world = 1;
  p.ar_ctl = nullptr;
  p.ar_wait_ns = 0;
  p.ar_cap = 0;
  for (int r = 0; r < kArMaxRanks; ++r) p.ar_data[r] = p.ar_flags[r] = 0;
  if (ar != nullptr && ar->world > 1) {
    if (ar->world > kArMaxRanks || pl.grid > kArMaxCtas ||
        static_cast<long long>(a.M) * a.N > ar->cap)
      return cudaErrorInvalidValue;
    p.ar_rank = ar->rank;
    p.ar_world = ar->world;
    p.ar_ctl = ar->ctl;
    p.ar_wait_ns = ar->wait_ns;
    p.ar_cap = ar->cap;
    for (int r = 0; r < ar->world; ++r) {
      p.ar_data[r] = ar->data[r];
      p.ar_flags[r] = ar->flags[r];
    }
  }
  switch (a.bits) {
    case 2: return launch_direct_b2(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 4: return launch_direct_b4(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 8: return launch_direct_b8(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dqg
