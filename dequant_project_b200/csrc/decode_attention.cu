// Decode attention of the tensor-parallel decoder step: one query token per
// sequence attends over its fp16 KV cache, grouped KV heads (GQA) included.
// The reference has no attention code; it models the step's cache reads as
// bytes (dequant/byte_model.py:214-219): every position's key and value row is
// read once per step, so the kernel is bound by HBM bandwidth over the cache.
//
//   o[m, h] = softmax(q[m, h] . K[m, h / g, :T]^T / sqrt(D)) V[m, h / g, :T]
//
// with q [M, Hq, D], K/V caches [M, Hkv, cap, D] (positions 0..T-1 valid),
// g = Hq / Hkv query heads per KV head, D = 128.
//
// Split-KV ("flash decoding"): a CTA takes one (sequence, KV head) and a range
// of positions, so that M * Hkv * splits fills the GPU. Its four warps take
// 16-position slices of 64-position tiles that cp.async brings into shared
// memory (16-byte chunks XOR-swizzled by row, so the ldmatrix reads below are
// conflict-free; three tiles in flight). Per slice:
//   S^T = Q K^T on the tensor cores (mma.m16n8k16: the g query heads, padded
//   to 16, are the A rows, kept in registers for the whole kernel; K rows
//   arrive as B fragments by ldmatrix), online softmax in fp32 (base-2
//   exponent, running max and sum per head), then O += P V with P re-used
//   from the score registers as the A fragment and V as B by ldmatrix.trans.
// The warps' partial (max, sum, O) are merged in shared memory; with one split
// the CTA writes o, otherwise it writes its partial to the workspace and the
// last CTA of the (sequence, head) -- counted with an atomic ticket that it
// resets -- merges all splits in split order and writes o.
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {
namespace {

constexpr int kD = 128;            // head dimension
constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kTileT = 64;         // positions per shared-memory tile
constexpr int kStages = 3;
constexpr int kRowBytes = kD * 2;  // one cache row (256 bytes)
constexpr int kTileBytes = kTileT * kRowBytes;
constexpr int kAttnSmem = kStages * 2 * kTileBytes;  // K and V tiles
constexpr int kMaxSplits = 64;     // position splits per (sequence, KV head)

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_f16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kAttnThreads)
    decode_attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, c = lane & 3;
  const int g = p.g;
  const int t_begin = split * p.Ts;
  const int t_end = min(p.T, t_begin + p.Ts);
  const int n_tiles = (t_end - t_begin + kTileT - 1) / kTileT;
  const int64_t mh = static_cast<int64_t>(m) * p.Hkv + kvh;
  const __half* kbase = p.kc + mh * p.cap * kD;
  const __half* vbase = p.vc + mh * p.cap * kD;
  const uint32_t sbase = smem_u32(smem);

  // The query and the newest cache slot come from the previous kernels. The
  // next kernel may be scheduled at once: it waits for this grid before it
  // reads the output, and can stage its own inputs meanwhile.
  pdl_wait_prior_grid();
  if (threadIdx.x == 0) pdl_launch_dependents();

  // Q as A fragments for the eight 16-wide steps over D: rows are the g query
  // heads of this KV head (rows >= g are zero).
  uint32_t qa[kD / 16][4];
  const __half* qrow = p.q + (static_cast<int64_t>(m) * p.Hq + static_cast<int64_t>(kvh) * g) * kD;
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int j = gid + 8 * (r & 1);
      const int d = ks * 16 + 2 * c + 8 * (r >> 1);
      qa[ks][r] = j < g ? *reinterpret_cast<const uint32_t*>(qrow + j * kD + d) : 0u;
    }

  auto load_tile = [&](int tile, int stage) {
    const int t0 = t_begin + tile * kTileT;
    const uint32_t kdst = sbase + stage * 2 * kTileBytes;
    const uint32_t vdst = kdst + kTileBytes;
    for (int i = threadIdx.x; i < kTileT * 16; i += kAttnThreads) {
      const int row = i >> 4, chunk = i & 15;
      const int t = t0 + row;
      const bool ok = t < t_end;
      const int64_t off = static_cast<int64_t>(ok ? t : t_begin) * kD + chunk * 8;
      cp_async16(kdst + swz(row, chunk), kbase + off, ok ? 16u : 0u);
      cp_async16(vdst + swz(row, chunk), vbase + off, ok ? 16u : 0u);
    }
  };

  float o[kD / 8][4];
#pragma unroll
  for (int nb = 0; nb < kD / 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

#pragma unroll
  for (int st = 0; st < kStages - 1; ++st) {
    if (st < n_tiles) load_tile(st, st);
    cp_async_commit();
  }
  const int p0 = warp * 16;  // this warp's slice of every tile
  for (int tile = 0; tile < n_tiles; ++tile) {
    const int nxt = tile + kStages - 1;
    if (nxt < n_tiles) load_tile(nxt, nxt % kStages);
    cp_async_commit();
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const uint32_t kst = sbase + (tile % kStages) * 2 * kTileBytes;
    const uint32_t vst = kst + kTileBytes;
    const int ts = t_begin + tile * kTileT + p0;  // first position of the slice
    if (ts < t_end) {
      // Scores of 16 positions: two 8-position blocks.
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < kD / 16; ++ks) {
        uint32_t b[4];
        ldsm_x4(kst + swz(p0 + ((lane >> 4) & 1) * 8 + (lane & 7), ks * 2 + ((lane >> 3) & 1)), b);
        mma_f16(sc[0], qa[ks], b[0], b[1]);
        mma_f16(sc[1], qa[ks], b[2], b[3]);
      }
      // Online softmax per head row (gid: elements 0, 1; gid + 8: 2, 3).
      float pr[2][4];
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = ts + nb * 8 + 2 * c + (e & 1);
          sc[nb][e] = t < t_end ? sc[nb][e] * p.scale_log2 : -INFINITY;
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float mx = fmaxf(fmaxf(sc[0][2 * r], sc[0][2 * r + 1]), fmaxf(sc[1][2 * r], sc[1][2 * r + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[r], mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float corr = exp2f(m_run[r] - m_use);
        l_run[r] *= corr;
#pragma unroll
        for (int nb = 0; nb < kD / 8; ++nb) {
          o[nb][2 * r] *= corr;
          o[nb][2 * r + 1] *= corr;
        }
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          pr[nb][2 * r] = exp2f(sc[nb][2 * r] - m_use);
          pr[nb][2 * r + 1] = exp2f(sc[nb][2 * r + 1] - m_use);
          l_run[r] += pr[nb][2 * r] + pr[nb][2 * r + 1];
        }
        m_run[r] = m_new;
      }
      // P (fp16) as the A fragment of the 16 positions; V as B fragments.
      uint32_t pa[4];
      pa[0] = pack_half2(pr[0][0], pr[0][1]);
      pa[1] = pack_half2(pr[0][2], pr[0][3]);
      pa[2] = pack_half2(pr[1][0], pr[1][1]);
      pa[3] = pack_half2(pr[1][2], pr[1][3]);
#pragma unroll
      for (int dp = 0; dp < kD / 16; ++dp) {
        uint32_t b[4];
        ldsm_x4_trans(vst + swz(p0 + ((lane >> 3) & 1) * 8 + (lane & 7), dp * 2 + ((lane >> 4) & 1)), b);
        mma_f16(o[2 * dp], pa, b[0], b[1]);
        mma_f16(o[2 * dp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Merge the four warps' (max, sum, O) in shared memory (the tiles are free).
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  float* os = reinterpret_cast<float*>(smem);                  // [warp][16][kD]
  float* ms = os + kAttnWarps * 16 * kD;                        // [warp][16]
  float* ls = ms + kAttnWarps * 16;                             // [warp][16]
#pragma unroll
  for (int nb = 0; nb < kD / 8; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      os[(warp * 16 + gid + 8 * (e >> 1)) * kD + nb * 8 + 2 * c + (e & 1)] = o[nb][e];
  if (c == 0) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ms[warp * 16 + gid + 8 * r] = m_run[r];
      ls[warp * 16 + gid + 8 * r] = l_run[r];
    }
  }
  __syncthreads();
  const int S = p.S;
  float* part = p.part + mh * S * g * kD;
  float* pml = p.ml + mh * S * g * 2;
  __half* orow = p.o + (static_cast<int64_t>(m) * p.Hq + static_cast<int64_t>(kvh) * g) * kD;
  for (int idx = threadIdx.x; idx < g * kD; idx += kAttnThreads) {
    const int j = idx / kD, d = idx - (idx / kD) * kD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, ms[w * 16 + j]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = exp2f(ms[w * 16 + j] - mx);
      num += os[(w * 16 + j) * kD + d] * f;
      den += ls[w * 16 + j] * f;
    }
    if (S == 1) {
      orow[j * kD + d] = __float2half_rn(num / den);
    } else {
      part[(split * g + j) * kD + d] = num;
      if (d == 0) {
        pml[(split * g + j) * 2] = mx;
        pml[(split * g + j) * 2 + 1] = den;
      }
    }
  }
  if (S == 1) return;

  // The last CTA of this (sequence, KV head) merges the splits in order.
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(p.tickets + mh, 1u);
    last = t == static_cast<unsigned>(S - 1);
    if (last) p.tickets[mh] = 0u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Split weights first (max over splits, then exp2(m_s - max) / sum), staged
  // in shared memory; then every output element is one weighted sum over the
  // splits with independent loads.
  float* wsplit = reinterpret_cast<float*>(smem);            // [S][g]: max, then weight
  float* lsplit = wsplit + kMaxSplits * 16;                   // [S][g]: sum
  float* wmax = lsplit + kMaxSplits * 16;                     // [g]
  float* wden = wmax + 16;                                    // [g]
  for (int i = threadIdx.x; i < S * g; i += kAttnThreads) {
    wsplit[i] = __ldcg(pml + 2 * i);
    lsplit[i] = __ldcg(pml + 2 * i + 1);
  }
  __syncthreads();
  if (threadIdx.x < g) {
    const int j = threadIdx.x;
    float mx = -INFINITY;
    for (int sp = 0; sp < S; ++sp) mx = fmaxf(mx, wsplit[sp * g + j]);
    float den = 0.f;
    for (int sp = 0; sp < S; ++sp) den += lsplit[sp * g + j] * exp2f(wsplit[sp * g + j] - mx);
    wmax[j] = mx;
    wden[j] = den;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < S * g; i += kAttnThreads) {
    const int j = i % g;
    wsplit[i] = exp2f(wsplit[i] - wmax[j]) / wden[j];
  }
  __syncthreads();
  // Each thread owns four consecutive outputs and sums over the splits in
  // batches of 16 independent 16-byte loads (the partials were written by
  // other CTAs moments ago and sit in L2; a loop with one load in flight
  // at a time took 20 us for 33 splits of eight heads).
  const int nv = g * (kD / 4);
  const float4* part4 = reinterpret_cast<const float4*>(part);
  for (int v = threadIdx.x; v < nv; v += kAttnThreads) {
    const int j = v / (kD / 4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < S; sp += 16) {
      float4 w[16];
#pragma unroll
      for (int u = 0; u < 16; ++u)
        w[u] = sp + u < S ? __ldcg(part4 + static_cast<int64_t>(sp + u) * nv + v)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const float f = sp + u < S ? wsplit[(sp + u) * g + j] : 0.f;
        acc.x += w[u].x * f;
        acc.y += w[u].y * f;
        acc.z += w[u].z * f;
        acc.w += w[u].w * f;
      }
    }
    __half2* o2 = reinterpret_cast<__half2*>(orow + v * 4);
    o2[0] = __floats2half2_rn(acc.x, acc.y);
    o2[1] = __floats2half2_rn(acc.z, acc.w);
  }
}

}  // namespace

size_t attention_counter_bytes(int M, int Hkv) {
  return (static_cast<size_t>(M) * Hkv * 4 + 255) / 256 * 256;
}

#ifndef DQG_ATTN_CTAS_PER_SM
#define DQG_ATTN_CTAS_PER_SM 2
#endif

namespace {
// Splits of T positions when the target is `per_sm` CTAs per SM (positions
// per split rounded up to whole tiles; *ts_out: positions per split).
int splits_for(int mh, int T, int num_sms, int per_sm, int* ts_out) {
  int s = (per_sm * num_sms + mh - 1) / mh;
  int max_s = (T + kTileT - 1) / kTileT;
  if (max_s > kMaxSplits) max_s = kMaxSplits;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  const int ts = ((T + s - 1) / s + kTileT - 1) / kTileT * kTileT;
  *ts_out = ts;
  return (T + ts - 1) / ts;
}
}  // namespace

// Two CTAs fit on an SM. Of the splits that target one and two CTAs per SM,
// take the one whose busiest SM streams fewer tiles (CTAs per SM, rounded up,
// times tiles per CTA); on a tie the fewer splits (fewer CTAs, less merging).
// Measured on B200: 7B heads at batch 1 keep two per SM (11.8 us; one per SM
// leaves 12 SMs with two CTAs of 7 tiles, 12.8 us), batch 8 takes one split
// per (sequence, head) (50.0 -> 43.9 us), the 16- and 8-head shards of
// tensor-parallel ranks one per SM (9.7 -> 8.7 and 9.2 -> 7.8 us).
int attention_splits(int M, int Hkv, int T, int num_sms, int* ts_out) {
  const int mh = M * Hkv;
  const int sms = num_sms > 0 ? num_sms : 1;
  int ts1 = 0, ts2 = 0;
  const int s1 = splits_for(mh, T, sms, 1, &ts1);
  const int s2 = splits_for(mh, T, sms, DQG_ATTN_CTAS_PER_SM, &ts2);
  const long long c1 = static_cast<long long>(mh) * s1, c2 = static_cast<long long>(mh) * s2;
  const long long load1 = (c1 + sms - 1) / sms * ((ts1 + kTileT - 1) / kTileT);
  const long long load2 = (c2 + sms - 1) / sms * ((ts2 + kTileT - 1) / kTileT);
  const bool one = load1 <= load2;
  if (ts_out) *ts_out = one ? ts1 : ts2;
  return one ? s1 : s2;
}

size_t attention_workspace_bytes(int M, int Hq, int Hkv, int T, int num_sms) {
  // Split counters first (a fixed place for every T), then the partials,
  // sized for the most splits any T up to this one can take.
  const int mh = M * Hkv;
  int s_max = (DQG_ATTN_CTAS_PER_SM * num_sms + mh - 1) / mh;
  int t_tiles = (T + kTileT - 1) / kTileT;
  if (t_tiles > kMaxSplits) t_tiles = kMaxSplits;
  if (s_max > t_tiles) s_max = t_tiles;
  if (s_max < 1) s_max = 1;
  const size_t g = Hq / Hkv;
  return attention_counter_bytes(M, Hkv) + static_cast<size_t>(mh) * s_max * g * (kD + 2) * 4;
}

cudaError_t launch_decode_attention(const AttnParams& p, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(decode_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kAttnSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.S, p.Hkv, p.M);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = kAttnSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_attention_kernel, p);
}

namespace {

}  // namespace
}  // namespace dqg

// ---------------------------------------------------------------------------
// Decode attention for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: a host that binds the
// C ABI from a runtime whose device memory is all owned by another allocator
// (an inference server that reserves the GPU's memory for KV caches at start-up
// and hands each kernel only the step's tensors), or a plugin whose host gives
// it no allocator and no workspace. dqg_decode_attention_noalloc serves them:
// its scratch (split counters and per-split partials) is the file-scope array
// below, so the caller passes only inputs and outputs.
//
// The array is a device symbol: every GPU that loads this library holds its
// kNoAllocScratchBytes until the process exits. In host code its name is a
// host-side stand-in, not a device address, so the launcher looks up the device
// address once per device, with that device current, and passes it to the
// kernel. Every call shares the array and it keeps the last call's contents:
// the split counters are cleared on the stream before each launch, and calls
// that overlap on the GPU (other streams, other host threads) race on it.
namespace dqg {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB per GPU
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

}  // namespace

size_t attention_noalloc_capacity() { return kNoAllocScratchBytes; }

cudaError_t launch_decode_attention_noalloc(AttnParams p, cudaStream_t stream) {
  static void* scratch[64] = {nullptr};  // device address of the array, per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (scratch[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attn_scratch);
    if (e != cudaSuccess) return e;
    scratch[dev] = ptr;
  }
  uint8_t* ws = static_cast<uint8_t*>(scratch[dev]);
  const size_t mh = static_cast<size_t>(p.M) * p.Hkv;
  const size_t cnt = attention_counter_bytes(p.M, p.Hkv);
  if (cnt + mh * p.S * p.g * (kD + 2) * 4 > kNoAllocScratchBytes) return cudaErrorInvalidValue;
  e = cudaMemsetAsync(ws, 0, cnt, stream);  // split counters start at zero
  if (e != cudaSuccess) return e;
  p.tickets = reinterpret_cast<unsigned*>(ws);
  p.ml = reinterpret_cast<float*>(ws + cnt);
  p.part = reinterpret_cast<float*>(ws + cnt + mh * p.S * p.g * 2 * 4);
  return launch_decode_attention(p, stream);
}

}  // namespace dqg
