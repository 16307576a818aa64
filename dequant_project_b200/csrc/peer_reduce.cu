// One-shot all-reduce of small fp16 tensors over NVLink peer memory, for the
// row-parallel layers of the tensor-parallel decoder (two per layer, 8-128 KB
// each). The reference has no collective; it only models the decoder's bytes
// (dequant/byte_model.py:179-251). At these sizes a collective is bound by
// latency, not bandwidth, so the exchange takes one one-way trip over NVLink:
//
//   1. every rank stores its input into every peer's receive buffer as 8-byte
//      packets (one 32-bit data word and one 32-bit flag holding this call's
//      epoch), plain stores through IPC mappings of the peers' memory;
//   2. it polls its own receive buffer (local memory) until every peer's
//      packets carry this call's epoch (bounded: a wait that runs out sets
//      the device status bit and those outputs stay unwritten);
//   3. it sums the ranks' words in rank order in fp32 and rounds once to
//      fp16, so every rank gets bit-identical results.
//
// A packet's data and flag travel in one aligned 8-byte store (two packets
// per 16-byte store), so a reader that sees the flag sees the data: no
// fences, no separate flag round trip and no loads from peer memory.
//
// Receive buffers are double-buffered by the parity of a per-rank call
// counter ("epoch") that lives in device memory and is advanced by the last
// CTA of each call, so the kernel can be captured in a CUDA graph (nothing
// per call comes from the host). Call e writes parity e & 1 of every peer's
// buffer, which call e + 2 overwrites. A rank starts call e + 2 only after its
// call e + 1 received every peer's call e + 1 packets, which a peer sends only
// after it finished reading its call e packets.
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {
namespace {

constexpr int kArThreads = 256;

__device__ __forceinline__ void st_volatile_v4(void* p, uint32_t a, uint32_t b, uint32_t c,
                                               uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

// 16 bytes of this GPU's memory that a peer is writing during the call
// (volatile: never served from a stale L1 line).
__device__ __forceinline__ uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// The last CTA of a call advances the epoch for the next call.
__device__ __forceinline__ void advance_epoch(uint32_t* ctl, uint32_t ep) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(ctl + 1, 1u);
    if (t == gridDim.x - 1) {
      ctl[1] = 0u;
      __threadfence();
      atomicExch(ctl, ep);
    }
  }
}

// Each thread owns two consecutive 32-bit words of the input (four fp16
// values): one 16-byte pair of packets per source rank.
__global__ void __launch_bounds__(kArThreads)
    peer_allreduce_kernel(const __grid_constant__ PeerReduceParams p) {
  pdl_wait_prior_grid();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const uint32_t ep = *reinterpret_cast<volatile const uint32_t*>(p.ctl) + 1u;
  const int64_t slot = p.cap / 2;  // packets per (parity, source rank)
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * kArThreads + threadIdx.x;
  const bool mine = pair * 4 < p.n;
  const int64_t base = static_cast<int64_t>(ep & 1u) * p.world * slot;  // packets
  if (mine) {
    const uint2 d = reinterpret_cast<const uint2*>(p.in)[pair];
    // 1. This rank's words into slot `rank` of every peer's receive buffer.
    for (int r = 0; r < p.world; ++r) {
      if (r == p.rank) continue;
      uint8_t* dst = reinterpret_cast<uint8_t*>(p.peer_data[r]) +
                     (base + static_cast<int64_t>(p.rank) * slot + pair * 2) * 8;
      st_volatile_v4(dst, d.x, ep, d.y, ep);
    }
    // 2. + 3. Every peer's packets from this rank's own buffer, summed with
    // this rank's words in rank order.
    const uint8_t* own = reinterpret_cast<const uint8_t*>(p.peer_data[p.rank]);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    uint64_t t0 = 0;
    for (int r = 0; r < p.world && ok; ++r) {
      uint32_t w0 = d.x, w1 = d.y;
      if (r != p.rank) {
        const uint8_t* src = own + (base + static_cast<int64_t>(r) * slot + pair * 2) * 8;
        uint4 v = ld_volatile_v4(src);
        for (uint32_t spin = 1; v.y != ep || v.w != ep; ++spin) {
          if ((spin & 63u) == 0u) {
            const uint64_t now = globaltimer();
            if (t0 == 0) {
              t0 = now;
            } else if (now - t0 > p.wait_ns) {
              atomicOr(&g_status, kStatusWaitTimeout);
              ok = false;
              break;
            }
          }
          v = ld_volatile_v4(src);
        }
        w0 = v.x;
        w1 = v.z;
      }
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w0));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w1));
      acc[0] += a.x;
      acc[1] += a.y;
      acc[2] += b.x;
      acc[3] += b.y;
    }
    if (ok) {
      const __half2 o0 = __floats2half2_rn(acc[0], acc[1]);
      const __half2 o1 = __floats2half2_rn(acc[2], acc[3]);
      reinterpret_cast<uint2*>(p.out)[pair] = make_uint2(
          *reinterpret_cast<const uint32_t*>(&o0), *reinterpret_cast<const uint32_t*>(&o1));
    }
  }
  advance_epoch(p.ctl, ep);
}

constexpr int kNormVecs = kArNormMaxH / 8 / kArThreads;  // 8-value vectors per thread

// One CTA per row m: the packet exchange of the row's partial sums (the same
// packets, slots and epochs as peer_allreduce_kernel: elements m * H .. (m +
// 1) * H of the flat tensor), then the residual add and RMSNorm of
// add_rms_norm_kernel (decode_ops.cu) with the all-reduced row as delta:
//   delta = fp16(sum over ranks in rank order, fp32),
//   h[m] = fp16(h[m] + delta),
//   y[m] = fp16((h * rsqrt(mean(h^2) + eps)) * w),
// with the same thread layout (thread t takes the 8-value vectors t, t + 256,
// ...), the same order of the sum of squares and the same roundings, so the
// fused call and the two separate ones give the same bits. A row whose
// exchange ran out of time is left unwritten (h and y).
__global__ void __launch_bounds__(kArThreads)
    peer_allreduce_norm_kernel(const __grid_constant__ PeerNormParams q) {
  const PeerReduceParams& p = q.ar;
  pdl_wait_prior_grid();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const uint32_t ep = *reinterpret_cast<volatile const uint32_t*>(p.ctl) + 1u;
  const int64_t slot = p.cap / 2;
  const int64_t base = static_cast<int64_t>(ep & 1u) * p.world * slot;  // packets
  const int m = blockIdx.x;
  const int nv = q.H / 8;
  const int64_t e0 = static_cast<int64_t>(m) * q.H;  // first element of the row
  uint4 d[kNormVecs];
#pragma unroll
  for (int i = 0; i < kNormVecs; ++i) {
    const int v = threadIdx.x + i * kArThreads;
    d[i] = v < nv ? reinterpret_cast<const uint4*>(p.in + e0)[v] : make_uint4(0u, 0u, 0u, 0u);
  }
  // 1. This rank's words into slot `rank` of every peer's receive buffer
  // (vector v: words 4v .. 4v + 3 of the row, packets e0 / 2 + 4v ...).
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.peer_data[r]) +
                   (base + static_cast<int64_t>(p.rank) * slot + e0 / 2) * 8;
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
      const int v = threadIdx.x + i * kArThreads;
      if (v >= nv) continue;
      st_volatile_v4(dst + static_cast<int64_t>(v) * 32, d[i].x, ep, d[i].y, ep);
      st_volatile_v4(dst + static_cast<int64_t>(v) * 32 + 16, d[i].z, ep, d[i].w, ep);
    }
  }
  // 2. Every rank's words in rank order (polling this rank's own buffer).
  const uint8_t* own = reinterpret_cast<const uint8_t*>(p.peer_data[p.rank]);
  bool ok = true;
  uint64_t t0 = 0;
  float acc[kNormVecs][8];
#pragma unroll
  for (int i = 0; i < kNormVecs; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
  for (int r = 0; r < p.world; ++r) {
    const uint8_t* src = own + (base + static_cast<int64_t>(r) * slot + e0 / 2) * 8;
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
      const int v = threadIdx.x + i * kArThreads;
      if (v >= nv) continue;
      uint32_t w[4] = {d[i].x, d[i].y, d[i].z, d[i].w};
      if (r != p.rank) {
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
          const uint8_t* sp = src + static_cast<int64_t>(v) * 32 + hlf * 16;
          uint4 pk = ld_volatile_v4(sp);
          for (uint32_t spin = 1; ok && (pk.y != ep || pk.w != ep); ++spin) {
            if ((spin & 63u) == 0u) {
              const uint64_t now = globaltimer();
              if (t0 == 0) {
                t0 = now;
              } else if (now - t0 > p.wait_ns) {
                atomicOr(&g_status, kStatusWaitTimeout);
                ok = false;
              }
            }
            pk = ld_volatile_v4(sp);
          }
          w[2 * hlf] = pk.x;
          w[2 * hlf + 1] = pk.z;
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        acc[i][2 * k] += f.x;
        acc[i][2 * k + 1] += f.y;
      }
    }
  }
  ok = __syncthreads_and(ok);
  // 3. Residual add and the sum of squares, as add_rms_norm_kernel.
  __half* hr = q.h + e0;
  __half* yr = q.y + e0;
  float hv[kNormVecs][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormVecs; ++i) {
    const int v = threadIdx.x + i * kArThreads;
    if (v >= nv) continue;
    uint4 a = reinterpret_cast<const uint4*>(hr)[v];
    __half* ah = reinterpret_cast<__half*>(&a);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half delta = __float2half_rn(acc[i][e]);
      ah[e] = __float2half_rn(__fadd_rn(__half2float(ah[e]), __half2float(delta)));
      hv[i][e] = __half2float(ah[e]);
      ss = __fmaf_rn(hv[i][e], hv[i][e], ss);
    }
    if (ok) reinterpret_cast<uint4*>(hr)[v] = a;
  }
  __shared__ float red[kArThreads / 32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kArThreads / 32; ++i) tot += red[i];
  const float rs = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(q.H)), q.eps));
  if (ok) {
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
      const int v = threadIdx.x + i * kArThreads;
      if (v >= nv) continue;
      const uint4 b = reinterpret_cast<const uint4*>(q.w)[v];
      const __half* wh = reinterpret_cast<const __half*>(&b);
      uint4 o;
      __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        oh[e] = __float2half_rn(__fmul_rn(__fmul_rn(hv[i][e], rs), __half2float(wh[e])));
      reinterpret_cast<uint4*>(yr)[v] = o;
    }
  }
  advance_epoch(p.ctl, ep);
}

}  // namespace

cudaError_t launch_peer_allreduce_add_rms_norm(const PeerNormParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.M));
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer_allreduce_norm_kernel, p);
}

cudaError_t launch_peer_allreduce(const PeerReduceParams& p, cudaStream_t stream) {
  const int64_t pairs = p.n / 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((pairs + kArThreads - 1) / kArThreads));
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, p);
}

}  // namespace dqg

DQG_STATUS_READER(read_status_peer)
