// Internal interface of the fused dequant + GEMV kernel (gemv.cu) and the
// materialising dequantize kernel (dequantize.cu). The public C ABI is in
// include/dequant_b200.h; capi.cu validates arguments and calls into here.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace dqg {

constexpr int kTile = 16;         // rows per tile (one m16 MMA tile)
constexpr int kNCW = 8;           // consumer (tensor-core) warps
constexpr int kNAux = 4;          // constant/activation-permute warps
constexpr int kGemvThreads = 32 * (1 + kNAux + kNCW);
constexpr int kMaxStages = 8;
constexpr int kMaxM = 8;          // activation rows handled by the GEMV path
constexpr int kMaxSmemBytes = 232448;  // 227 KB opt-in dynamic shared memory
constexpr int kRedBytes = 2 * kNCW * kTile * kMaxM * 4;
constexpr int kStageBytes = 40 * 1024;     // target packed bytes per 16-row stage
constexpr int kMaxXresBytes = 100 * 1024;  // cap on resident permuted activations
constexpr int kXStageBytes = 48 * 1024;    // cap on per-stage raw + permuted activations
constexpr int kBarBytes = 256;
constexpr int kMaxMetaBytes = 64 * 1024;  // cap on the two tile metadata buffers

struct GemvParams {
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
  int ep;                   // constant entries per row (odd stride)
  int steps_max;            // steps per slab
  int w_pitch;              // padded bytes per packed row in a stage
  int xp_pitch;             // bytes per permuted activation row
  int off_w, off_xraw, off_xperm, off_ent, off_sx, off_flag;
  int stage_bytes;
  int off_xres;             // whole-K permuted activations (resident variant)
  int off_sxres;            // their per-step sums [M][K / step]
  int off_meta, meta_stride, meta_direct;
  int off_red, off_bar;
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
  int wpl, ks, n_slabs, ep, steps_max, xres, stages;
  int w_pitch, xp_pitch;
  int off_w, off_xraw, off_xperm, off_ent, off_sx, off_flag, stage_bytes;
  int off_xres, off_sxres, off_meta, meta_stride, meta_direct, off_red, off_bar, smem, grid;
};

// Words of packed codes each lane loads per step (4, 2 or 1), or 0 when the
// group size does not allow one (group_size % (128 / bits) != 0).
int gemv_words_per_lane(int bits, int group_size, int K);

// Shared-memory layout, stage count and grid for one call shape.
bool plan_gemv(int M, int N, int K, int bits, int group_size, int num_sms, GemvPlan* plan);

cudaError_t launch_gemv(const GemvArgs& args, const GemvPlan& plan, cudaStream_t stream);

// ---------------------------------------------------------------- streaming
// Streaming kernel (gemv_stream.cu): activations resident in shared memory,
// codes unpacked to fp16 subnormals, no preparation warps. Used whenever its
// plan fits; gemv_kernel above covers the rest (activations too large to keep
// resident, or very many groups per row).
#ifndef DQG_STREAM_NCW
#define DQG_STREAM_NCW 8
#endif
constexpr int kStreamNCW = DQG_STREAM_NCW;  // consumer (tensor-core) warps
#ifndef DQG_STREAM_SMEM
#define DQG_STREAM_SMEM 232448
#endif
#ifndef DQG_STREAM_MIN_BLOCKS
#define DQG_STREAM_MIN_BLOCKS 1
#endif
// Shared memory a streaming CTA may use, and CTAs per SM the register budget
// is sized for.
constexpr int kStreamSmemBytes = DQG_STREAM_SMEM;
constexpr int kStreamMinBlocks = DQG_STREAM_MIN_BLOCKS;
constexpr int kStreamThreads = 32 * (2 + kStreamNCW);  // + producer + reducer
constexpr int kStreamNRB = 4;     // tile reduction buffers
constexpr int kStreamXMaxBytes = 100 * 1024;   // cap on resident activations (per CTA)
constexpr int kStreamMaxCluster = 8;          // largest split-K cluster (portable size)
constexpr int kStreamStageBytes = 64 * 1024;   // target packed bytes per stage (long row runs)
constexpr int kStreamMaxMeta = 8;  // tile metadata buffers
constexpr int kStreamBarBytes = 512;

struct StreamParams {
  const uint16_t* x;
  const uint32_t* qw;
  const uint16_t* scales;
  const uint16_t* zeros;
  uint16_t* y;
  int M, N, K, G, gsize;
  int mp;                 // columns per group slot of the MMA's N=8 side (1,2,4,8)
  int KS, n_slabs, stages, n_meta;
  int C, KC;              // cluster size (split K) and codes per CTA's K slice
  int w_pitch, xp;        // bytes per packed row in a stage; per activation row
  int stage_bytes;
  int off_x, off_sstep, off_sx, off_meta, meta_half, meta_stride, off_red, off_bar, off_xred;
  int off_zero;           // zero block for non-live fragment columns
  int prefetch;           // 1: the first weight ring is issued before the dependent-launch wait
  int starve;             // diagnostic: 1 = the producer issues nothing (every wait gives up)
  unsigned long long wait_ns;  // limit of each bounded wait
  long long tail_first;   // first scales/zeros element past the last 16-byte boundary
  int tail_n;             // number of such elements (0..7)
};

struct StreamPlan {
  int wpl, mp, ks, n_slabs, stages, n_meta, w_pitch, xp, stage_bytes, C, KC;
  int off_x, off_sstep, off_sx, off_meta, meta_half, meta_stride, off_red, off_bar, off_xred;
  int off_zero;
  int smem, grid;
};

bool plan_stream(int M, int N, int K, int bits, int group_size, int num_sms, StreamPlan* plan);

// ------------------------------------------------------- peer all-reduce
// One-shot all-reduce of fp16 tensors over peer memory (peer_reduce.cu).
constexpr int kArMaxRanks = 8;
constexpr int kArNormMaxH = 8192;  // row length of the fused all-reduce + RMSNorm

struct PeerReduceParams {
  const __half* in;
  __half* out;
  long long n;                    // elements, a multiple of 8
  long long cap;                  // elements of one parity half (packets per slot: cap / 2)
  // Each rank's receive buffer: [parity 2][source rank world][cap / 2]
  // 8-byte packets (32-bit data word, 32-bit epoch flag).
  unsigned long long peer_data[kArMaxRanks];
  uint32_t* ctl;                  // this rank's [epoch, ticket]
  int rank, world;
  unsigned long long wait_ns;
};

cudaError_t launch_peer_allreduce(const PeerReduceParams& p, cudaStream_t stream);

// The all-reduce of a row-parallel layer's partial rows fused with the
// residual add + RMSNorm that follows it: in = this rank's partial [M, H]
// (n = M * H), h [M, H] updated in place, y = RMSNorm(h) * w.
struct PeerNormParams {
  PeerReduceParams ar;
  __half* h;
  const __half* w;
  __half* y;
  int M, H;
  float eps;
};
cudaError_t launch_peer_allreduce_add_rms_norm(const PeerNormParams& p, cudaStream_t stream);

// ------------------------------------------------------------------ direct
// Direct kernel (gemv_direct.cuh): group-wise formats with one MMA step per
// group, activations resident in one CTA; every warp streams its own range of
// work units from global memory into registers.
#ifndef DQG_DIRECT_NW
#define DQG_DIRECT_NW 8
#endif
#ifndef DQG_DIRECT_RING
#define DQG_DIRECT_RING 8192
#endif
constexpr int kDirectNW = DQG_DIRECT_NW;         // warps per CTA
constexpr int kDirectThreads = 32 * kDirectNW;
constexpr int kDirectRingBytes = DQG_DIRECT_RING;  // per-warp ring of packed words in flight
constexpr int kDirectMaxSmem = 232448;
constexpr int kDirectMinSmem = 120 * 1024;       // more than half an SM: one CTA per SM

struct DirectParams {
  const uint16_t* x;
  const uint32_t* qw;
  const uint16_t* scales;
  const uint16_t* zeros;
  uint16_t* y;
  int M, N, K, G;
  int Gp;                 // groups per tile padded to whole units
  int xp;                 // bytes per permuted activation row in shared memory
  int off_x, off_sx, off_zero, off_red, off_tiles, off_ring;
  int prefetch;           // 1: first ring issued before the dependent-launch wait
  // SwiGLU mode (N a multiple of 16, rows interleaved by 8: tile rows 0-7 the
  // gate rows, 8-15 the up rows of the same outputs): y is [M, N / 2],
  // y = silu(gate) * up.
  int swiglu;
  // Row-parallel mode (ar_world > 1): y = the sum over ranks of every rank's
  // x_r @ W_r^T, exchanged through peer memory (see PeerGemvArgs).
  int ar_rank, ar_world;
  unsigned long long ar_data[kArMaxRanks];   // each rank's fp32 exchange buffer [2][M * N]
  unsigned long long ar_flags[kArMaxRanks];  // each rank's flags [CTA][world] u32
  uint32_t* ar_ctl;                          // this rank's [epoch, ticket]
  long long ar_cap;                          // fp32 values per parity half
  unsigned long long ar_wait_ns;
};

// Peer memory of a row-parallel GEMV (dqg_gemv_allreduce).
struct PeerGemvArgs {
  int rank, world;
  const unsigned long long* data;    // [world] exchange buffers (fp32, 2 * cap values)
  const unsigned long long* flags;   // [world] flag arrays (kArMaxCtas * world u32)
  uint32_t* ctl;
  long long cap;
  unsigned long long wait_ns;
};
constexpr int kArMaxCtas = 1024;

struct DirectPlan {
  int wpl, mp, gs, Gp, xp, off_x, off_sx, off_zero, off_red, off_tiles, off_ring, smem, grid;
};

// fused: plan for the row-parallel GEMV + all-reduce (any M); otherwise only
// where the direct kernel measured faster than the streaming one.
bool plan_direct(int M, int N, int K, int bits, int group_size, int num_sms, DirectPlan* plan,
                 bool fused = false);
cudaError_t launch_direct(const GemvArgs& args, const DirectPlan& plan, cudaStream_t stream,
                          const PeerGemvArgs* ar = nullptr, bool swiglu = false);

// ------------------------------------------------------- decode attention
struct AttnParams {
  const __half* q;        // [M, Hq, 128]
  const __half* kc;       // [M, Hkv, cap, 128]
  const __half* vc;
  __half* o;              // [M, Hq, 128]
  float* part;            // workspace: [M * Hkv][S][g][128] partial outputs
  float* ml;              // workspace: [M * Hkv][S][g][2] running max and sum
  unsigned* tickets;      // workspace: [M * Hkv] split counters (zero between calls)
  int M, Hq, Hkv, g, cap, T, S, Ts;
  float scale_log2;       // log2(e) / sqrt(128)
};
int attention_splits(int M, int Hkv, int T, int num_sms, int* ts_out);
size_t attention_counter_bytes(int M, int Hkv);
size_t attention_workspace_bytes(int M, int Hq, int Hkv, int T, int num_sms);
cudaError_t launch_decode_attention(const AttnParams& p, cudaStream_t stream);
// The same kernel with its scratch in a static device array (no allocation).
size_t attention_noalloc_capacity();
cudaError_t launch_decode_attention_noalloc(AttnParams p, cudaStream_t stream);

// Process-wide switch (default on): the streaming kernel issues its first
// weight ring before waiting for the previous grid on the stream.
void set_weight_prefetch(bool on);
bool weight_prefetch();
// wait_ns: limit of each bounded wait in the kernel (0 = the default, 2 s);
// starve: diagnostic launch whose producer issues no copies, so that every
// wait of the kernel gives up after wait_ns and the status word records it.
cudaError_t launch_stream(const GemvArgs& args, const StreamPlan& plan, cudaStream_t stream,
                          unsigned long long wait_ns = 0, bool starve = false);

struct DequantArgs {
  const uint32_t* qweight;
  const uint16_t* scales;
  const uint16_t* zeros;
  uint16_t* out;            // fp16 [N, K]
  int N, K, bits, group_size;
  bool symmetric, interleaved;
};

cudaError_t launch_dequantize(const DequantArgs& args, cudaStream_t stream);

// Read (and optionally clear) the device status of `device`: the OR of the
// status words of every translation unit whose kernels wait.
cudaError_t read_device_status(int device, uint32_t* status, bool reset);
cudaError_t read_status_gemv(uint32_t* status, bool reset);
cudaError_t read_status_stream_b2(uint32_t* status, bool reset);
cudaError_t read_status_stream_b4(uint32_t* status, bool reset);
cudaError_t read_status_stream_b8(uint32_t* status, bool reset);
cudaError_t read_status_peer(uint32_t* status, bool reset);
cudaError_t read_status_direct_b2(uint32_t* status, bool reset);
cudaError_t read_status_direct_b4(uint32_t* status, bool reset);
cudaError_t read_status_direct_b8(uint32_t* status, bool reset);



cudaError_t launch_add_one(const float* x, float* out, int64_t n, cudaStream_t stream);

// Decoder-step element-wise kernels (decode_ops.cu).
// Bulk L2 prefetch ranges carried by the decode ops (16-byte aligned starts
// and sizes, normalised by the host).
struct L2Spans {
  const uint8_t* ptr[8];
  uint64_t bytes[8];
  int n;
};
cudaError_t launch_add_rms_norm(void* h, const void* delta, const void* w, void* y, int M, int H,
                                float eps, const L2Spans& pf, int num_sms, cudaStream_t stream);
cudaError_t launch_rope_kv_append(const void* qkv, const float* cosv, const float* sinv,
                                  void* q_out, void* kc, void* vc, int M, int hq, int hkv, int D,
                                  int pos, int cap, const L2Spans& pf, int num_sms,
                                  cudaStream_t stream);
cudaError_t launch_silu_mul(const void* gu, void* out, int M, int I, const L2Spans& pf,
                            int num_sms, cudaStream_t stream);

}  // namespace dqg
