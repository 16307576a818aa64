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
  // The last CTA of the call advances the epoch for the next call.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(p.ctl + 1, 1u);
    if (t == gridDim.x - 1) {
      p.ctl[1] = 0u;
      __threadfence();
      atomicExch(p.ctl, ep);
    }
  }
}

}  // namespace

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
