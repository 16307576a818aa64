// Internal interface of the fused dequant + GEMV kernel (gemv.cu) and the
// materialising dequantize kernel (dequantize.cu). The public C ABI is in
// include/dequant_b200.h; capi.cu validates arguments and calls into here.
#pragma once

#include <cstdint>
#include <cuda.h>  // CUtensorMap (the encoder is fetched through the runtime)
#include <cuda_runtime.h>

namespace dqg {

constexpr int kTile = 16;         // rows per tile (one m16 MMA tile, one TMA box)
constexpr int kRowBlock = 32;     // output rows per row block (two tiles)
constexpr int kNCW = 8;           // consumer (tensor-core) warps
constexpr int kNAux = 4;          // constant/activation-permute warps
constexpr int kGemvThreads = 32 * (1 + kNAux + kNCW);
constexpr int kMaxStages = 8;
constexpr int kMaxM = 8;          // activation rows handled by the GEMV path
constexpr int kMaxEntPerLane = 17;  // (row, group) constants per aux lane per stage
constexpr int kMaxSmemBytes = 232448;  // 227 KB opt-in dynamic shared memory
constexpr int kRedBytes = 2 * kNCW * kRowBlock * kMaxM * 4;
constexpr int kBarBytes = 256;
constexpr int kAlignSlack = 1024;
constexpr int kMaxMetaBytes = 96 * 1024;  // cap on the two row-block metadata buffers   // dynamic smem is re-aligned to 1024 bytes

struct GemvParams {
  CUtensorMap tmap;         // packed words [N rows, K*bits/32 words], 32x16 boxes, 128B swizzle
  const uint16_t* x;        // fp16 [M, K]
  const uint32_t* qw;       // packed words [N, K*bits/32]
  const uint16_t* scales;   // fp16 [N, G]
  const uint16_t* zeros;    // fp16 [N, G] or null when symmetric
  uint16_t* y;              // fp16 [M, N]
  int M, N, K, G, gsize;
  int KS;                   // slab length in codes
  int n_slabs;
  int stages;
  uint32_t gq_magic;        // fast_div magic for group_size / step codes
  int gps_max;              // constant entries per row per stage
  int steps_max;            // steps per slab
  int xraw_pitch, xperm_pitch;
  int off_w, off_xraw, off_xperm, off_const, off_corr, off_sx, off_flag;
  int stage_bytes;
  int off_red, off_bar;
  int meta_direct;          // 1: row-block metadata arrives by bulk copy into off_meta
  int off_meta, meta_stride;  // two buffers, each [scales span | zeros span]
};

struct GemvArgs {
  const uint16_t* x;
  const uint32_t* qweight;
  const uint16_t* scales;
  const uint16_t* zeros;
  uint16_t* y;
  int M, N, K, bits, group_size;
  bool symmetric, interleaved;
};

struct GemvPlan {
  int wpl, ks, gps_max, steps_max, stages;
  int xraw_pitch, xperm_pitch;
  int off_w, off_xraw, off_xperm, off_const, off_corr, off_sx, off_flag;
  int stage_bytes, off_red, off_bar, smem, grid;
  int meta_direct, off_meta, meta_stride;
};

// Words of packed codes each lane loads per step (4, 2 or 1), or 0 when the
// group size does not allow one (group_size % (128 / bits) != 0).
int gemv_words_per_lane(int bits, int group_size, int K);

// Shared-memory layout, stage count and grid for one call shape.
bool plan_gemv(int M, int N, int K, int bits, int group_size, int num_sms, GemvPlan* plan);

cudaError_t launch_gemv(const GemvArgs& args, const GemvPlan& plan, cudaStream_t stream);

struct DequantArgs {
  const uint32_t* qweight;
  const uint16_t* scales;
  const uint16_t* zeros;
  uint16_t* out;            // fp16 [N, K]
  int N, K, bits, group_size;
  bool symmetric, interleaved;
};

cudaError_t launch_dequantize(const DequantArgs& args, cudaStream_t stream);

// Read (and optionally clear) the device status word g_status of `device`.
cudaError_t read_device_status(int device, uint32_t* status, bool reset);

cudaError_t launch_add_one(const float* x, float* out, int64_t n, cudaStream_t stream);

}  // namespace dqg
