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

namespace {
int round_up(int v, int m) { return (v + m - 1) / m * m; }
}  // namespace

bool plan_direct(int M, int N, int K, int bits, int group_size, int num_sms, DirectPlan* plan) {
  if (M < 1 || M > kMaxM || N < 1 || num_sms < 1 || group_size <= 0 || K % group_size) return false;
  const int wpl = gemv_words_per_lane(bits, group_size, K);
  if (wpl == 0) return false;
  const int sc = 4 * wpl * (32 / bits);
  const int G = K / group_size;
  // Group-wise formats whose group is exactly one MMA step of the lane
  // layout (INT4 up to g128, INT2 up to g256, INT8 up to g64).
  if (G < 2 || group_size != sc) return false;
  // Measured on B200 against the streaming kernel: the direct kernel is
  // faster for 4- and 8-bit codes on rows of up to 6144 codes (INT4 g128:
  // 4096x4096 6.85 -> 5.66 us, 128256x4096 108 -> 80 us, M = 8 11008x4096
  // 17.8 -> 15.6 us) and slower on longer rows (28672x8192 36.9 -> 39.7 us)
  // and for 2-bit codes (4-byte copies per lane); those stay streaming.
  if (bits < 4 || K > 6144) return false;
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
  const int tiles = (N + kTile - 1) / kTile;
  pl.grid = tiles < num_sms ? tiles : num_sms;
  *plan = pl;
  return true;
}

cudaError_t launch_direct(const GemvArgs& a, const DirectPlan& pl, cudaStream_t stream) {
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
  switch (a.bits) {
    case 2: return launch_direct_b2(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 4: return launch_direct_b4(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 8: return launch_direct_b8(pl.wpl, pl.gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dqg
