// Host side of the streaming GEMV kernel (gemv_stream.cuh): shared-memory
// plan and launch. The kernel variants are instantiated per bit width in
// gemv_stream_b{2,4,8}.cu so that they compile in parallel.
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "gemv.h"

namespace dqg {

cudaError_t launch_stream_b2(int wpl, int gs, bool sym, bool inter, const StreamParams& p,
                             int grid, int smem, cudaStream_t stream);
cudaError_t launch_stream_b4(int wpl, int gs, bool sym, bool inter, const StreamParams& p,
                             int grid, int smem, cudaStream_t stream);
cudaError_t launch_stream_b8(int wpl, int gs, bool sym, bool inter, const StreamParams& p,
                             int grid, int smem, cudaStream_t stream);

namespace {

int round_up(int v, int m) { return (v + m - 1) / m * m; }

std::atomic<int> g_weight_prefetch{1};

}  // namespace

void set_weight_prefetch(bool on) { g_weight_prefetch.store(on ? 1 : 0); }
bool weight_prefetch() { return g_weight_prefetch.load() != 0; }

bool plan_stream(int M, int N, int K, int bits, int group_size, int num_sms, StreamPlan* plan) {
  const int pp = 32 / bits;
  const int wpl = gemv_words_per_lane(bits, group_size, K);
  if (wpl == 0 || num_sms <= 0 || M < 1 || M > kMaxM || N < 1) return false;
  const int sc = 4 * wpl * pp;
  const int G = K / group_size;
  const bool grouped = G > 1;
  // Activation-row columns per group slot: M rounded up to a power of two
  // (M = 1: eight groups per unit); per-channel: all 8 columns are
  // activation rows.
  int mp = 1;
  while (mp < M) mp <<= 1;
  if (!grouped) mp = 8;
  const int gslots = 8 / mp;
  const int uc = grouped ? gslots * group_size : sc;  // codes per consumer unit
  StreamPlan pl;
  pl.wpl = wpl;
  pl.mp = mp;
  // Split K over a cluster of C CTAs when the activations do not fit one
  // CTA: each keeps a slice of KC codes (whole consumer units) resident.
  // Activation rows: 32 bytes of padding past a 128-byte multiple, so that the
  // eight rows an M=8 B-fragment load touches fall on distinct bank groups.
  // The smallest C whose slice's activations, sums, metadata ring (two
  // buffers), reduction buffers and two 16-row stages fit.
  const int meta_stride = 2 * round_up(kTile * G * 2 + 32, 128);
  // Bytes of one 16-row stage when a slice of kc codes is cut into slabs of
  // about kStreamStageBytes (whole units).
  auto slab_codes = [&](int kc) {
    const int64_t bytes = static_cast<int64_t>(kc) * bits / 8;
    int ns = static_cast<int>((kTile * bytes + kStreamStageBytes - 1) / kStreamStageBytes);
    if (ns < 1) ns = 1;
    int ks = round_up((kc + ns - 1) / ns, uc);
    return ks > kc ? kc : ks;
  };
  auto stage_bytes_for = [&](int kc) {
    return round_up(kTile * (round_up(slab_codes(kc) * bits / 8, 128) + 16 * wpl), 128);
  };
  const int red_bytes = round_up(kStreamNRB * kStreamNCW * kTile * M * 4, 128);
  int C = 1, KC = K;
  for (;;) {
    KC = round_up((K + C - 1) / C, uc);
    const int xb = round_up(M * (round_up(KC * 2, 128) + 32), 128);
    const int need = xb + round_up(M * (KC / sc) * 4, 128) +
                     round_up(M * (grouped ? KC / group_size : 1) * 4, 128) +
                     (C > 1 ? round_up(kStreamNRB * C * kTile * M * 4, 128) : 0) + red_bytes +
                     kStreamBarBytes + 640 + 2 * meta_stride + 2 * stage_bytes_for(KC);
    if ((C - 1) * KC < K && xb <= kStreamXMaxBytes && need <= kStreamSmemBytes) break;
    C *= 2;
    if (C > kStreamMaxCluster || C > num_sms) return false;
  }
  pl.C = C;
  pl.KC = KC;
  pl.xp = round_up(KC * 2, 128) + 32;
  const int x_bytes = round_up(M * pl.xp, 128);
  const int Gs = grouped ? KC / group_size : 1;
  int off = 0;
  pl.off_x = off;
  off += x_bytes;
  pl.off_sstep = off;
  off += round_up(M * (KC / sc) * 4, 128);
  pl.off_sx = off;
  off += round_up(M * Gs * 4, 128);
  // Zero block (one step of activations, 512 bytes at most) whose bank phase
  // is 64 bytes off the activation rows' (which start at 128-byte multiples).
  pl.off_zero = off + 64;
  off += 640;
  pl.off_xred = off;  // rank 0's slots for the peers' tile partials
  if (C > 1) off += round_up(kStreamNRB * C * kTile * M * 4, 128);
  // Metadata: a ring of tile buffers, each [scales span | zeros span] of 16
  // rows x G fp16 plus up to 16 bytes of alignment slack.
  pl.meta_half = round_up(kTile * G * 2 + 32, 128);
  pl.meta_stride = 2 * pl.meta_half;
  pl.off_red = off;
  off += round_up(kStreamNRB * kStreamNCW * kTile * M * 4, 128);
  pl.off_bar = off;
  off += kStreamBarBytes;
  pl.off_meta = off;  // NMB tile metadata buffers follow
  // Slabs: about kStreamStageBytes of packed weights per 16-row stage, in
  // whole consumer units.
  const int ks = slab_codes(KC);
  const int n_slabs = (KC + ks - 1) / ks;
  pl.ks = ks;
  pl.n_slabs = n_slabs;
  pl.w_pitch = round_up(ks * bits / 8, 128) + 16 * wpl;
  pl.stage_bytes = round_up(kTile * pl.w_pitch, 128);
  // Ring stages with two metadata buffers first; then more metadata buffers
  // (one per tile the ring can hold, plus one) while they fit.
  int stages = (kStreamSmemBytes - off - 2 * pl.meta_stride) / pl.stage_bytes;
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return false;
  int n_meta = (stages + n_slabs - 1) / n_slabs + 1;
  if (n_meta > kStreamMaxMeta) n_meta = kStreamMaxMeta;
  while (n_meta > 2 && off + n_meta * pl.meta_stride + stages * pl.stage_bytes > kStreamSmemBytes)
    --n_meta;
  if (n_meta < 2) n_meta = 2;
  pl.stages = stages;
  pl.n_meta = n_meta;
  off += n_meta * pl.meta_stride;
  // The ring sits at offset 0; everything else follows it.
  const int ring = stages * pl.stage_bytes;
  pl.off_x += ring;
  pl.off_sstep += ring;
  pl.off_sx += ring;
  pl.off_meta += ring;
  pl.off_red += ring;
  pl.off_bar += ring;
  pl.off_xred += ring;
  pl.off_zero += ring;
  pl.smem = ring + off;
  // Clusters (each a set of C CTAs on C SMs sharing rows); the launch caps
  // them at the number that can be resident at once.
  const int tiles = (N + kTile - 1) / kTile;
  const int clusters = num_sms / C;
  pl.grid = C * (tiles < clusters ? tiles : clusters);
  *plan = pl;
  return true;
}

cudaError_t launch_stream(const GemvArgs& a, const StreamPlan& pl, cudaStream_t stream,
                          unsigned long long wait_ns, bool starve) {
  StreamParams p;
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
  p.mp = pl.mp;
  p.KS = pl.ks;
  p.n_slabs = pl.n_slabs;
  p.stages = pl.stages;
  p.n_meta = pl.n_meta;
  p.w_pitch = pl.w_pitch;
  p.xp = pl.xp;
  p.stage_bytes = pl.stage_bytes;
  p.off_x = pl.off_x;
  p.off_sstep = pl.off_sstep;
  p.off_sx = pl.off_sx;
  p.off_meta = pl.off_meta;
  p.meta_half = pl.meta_half;
  p.meta_stride = pl.meta_stride;
  p.off_red = pl.off_red;
  p.off_bar = pl.off_bar;
  p.off_xred = pl.off_xred;
  p.off_zero = pl.off_zero;
  p.C = pl.C;
  p.KC = pl.KC;
  p.prefetch = weight_prefetch() ? 1 : 0;
  p.starve = starve ? 1 : 0;
  p.wait_ns = wait_ns ? wait_ns : 2000000000ull;  // 2 s: orders above any healthy wait
  const long long total = static_cast<long long>(a.N) * p.G;
  p.tail_first = total / 8 * 8;
  p.tail_n = static_cast<int>(total - p.tail_first);
  // Metadata spans are bulk-copied from 16-byte boundaries of the tensors.
  if (reinterpret_cast<uintptr_t>(a.scales) % 16 ||
      (a.zeros != nullptr && reinterpret_cast<uintptr_t>(a.zeros) % 16))
    return cudaErrorInvalidValue;
  const int gs = p.G > 1 ? 8 / pl.mp : 0;
  switch (a.bits) {
    case 2: return launch_stream_b2(pl.wpl, gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 4: return launch_stream_b4(pl.wpl, gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    case 8: return launch_stream_b8(pl.wpl, gs, a.symmetric, a.interleaved, p, pl.grid, pl.smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dqg
