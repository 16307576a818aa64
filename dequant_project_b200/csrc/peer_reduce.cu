// One-shot all-reduce of small fp16 tensors over NVLink peer memory, for the
// row-parallel layers of the tensor-parallel decoder (two per layer, 8-128 KB
// each). The reference has no collective; it only models the decoder's bytes
// (dequant/byte_model.py:179-251). NCCL's ring/tree algorithms pay several
// link round trips per call; at these sizes the call is latency-bound, so a
// single exchange round is cheaper:
//
//   1. every rank copies its input chunk into its own exchange buffer;
//   2. it raises a flag in every peer's flag array (plain stores through an
//      IPC mapping of the peer's memory, ordered by a system-scope fence);
//   3. it waits until every peer's flag for the chunk has arrived in its own
//      flag array (bounded: a wait that runs out sets the device status bit
//      and the kernel returns);
//   4. it reads the chunk from every rank's buffer (plain loads from peer
//      memory, no bulk copies, no multicast) and sums in rank order in fp32,
//      rounding once to fp16, so every rank gets bit-identical results.
//
// Exchange buffers are double-buffered by the parity of a per-rank call
// counter ("epoch") that lives in device memory and is advanced by the last
// CTA of each call, so the kernel can be captured in a CUDA graph (nothing
// per call comes from the host). Flags hold the epoch of the last call that
// raised them and only grow, so a wait accepts any value >= its epoch.
//
// Buffer reuse: call e writes buffer e & 1, which call e + 2 overwrites. A
// rank starts call e + 2 only after its call e + 1 saw every peer's call e + 1
// flag, which a peer raises only after it finished call e (its reads of our
// buffer e & 1 included).
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {
namespace {

constexpr int kArThreads = 256;

__device__ __forceinline__ void fence_sys() { fence_acq_rel_sys(); }

// 16 bytes from a (possibly peer) address, bypassing L1: the data were written
// by another GPU during this call.
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads)
    peer_allreduce_kernel(const __grid_constant__ PeerReduceParams p) {
  pdl_wait_prior_grid();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int chunk = blockIdx.x;
  const int tid = threadIdx.x;
  const uint32_t ep = *reinterpret_cast<volatile const uint32_t*>(p.ctl) + 1u;
  const int64_t par_off = static_cast<int64_t>(ep & 1u) * p.cap;  // elements
  const int64_t e0 = static_cast<int64_t>(chunk) * kArChunk;
  const int64_t left = p.n - e0;
  const int n_here = static_cast<int>(left < kArChunk ? left : kArChunk);
  __half* mine = reinterpret_cast<__half*>(p.peer_data[p.rank]) + par_off + e0;

  // 1. This rank's chunk into its exchange buffer (n is a multiple of 8).
  for (int v = tid; v < n_here / 8; v += kArThreads)
    reinterpret_cast<uint4*>(mine)[v] = reinterpret_cast<const uint4*>(p.in + e0)[v];
  __syncthreads();
  // 2. Raise this chunk's flag in every rank's flag array (ours included).
  if (tid < p.world) {
    fence_sys();
    uint32_t* flags = reinterpret_cast<uint32_t*>(p.peer_flags[tid]);
    st_relaxed_sys(flags + chunk * p.world + p.rank, ep);
  }
  // 3. Wait for every rank's flag of this chunk in our own array.
  bool ok = true;
  if (tid < p.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(p.peer_flags[p.rank]) +
                        chunk * p.world + tid;
    ok = wait_flag_sys(f, ep, p.wait_ns);
    fence_sys();
  }
  ok = __syncthreads_and(ok);
  // 4. Sum the chunk over ranks in rank order, fp32, one rounding.
  if (ok) {
    for (int v = tid; v < n_here / 8; v += kArThreads) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < p.world; ++r) {
        const __half* src = reinterpret_cast<const __half*>(p.peer_data[r]) + par_off + e0;
        const uint4 w = ld_cg_v4(reinterpret_cast<const uint4*>(src) + v);
        const __half2* h2 = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          acc[2 * i] += f.x;
          acc[2 * i + 1] += f.y;
        }
      }
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) oh[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      reinterpret_cast<uint4*>(p.out + e0)[v] = o;
    }
  }
  // 5. The last CTA of the call advances the epoch for the next call.
  __syncthreads();
  if (tid == 0) {
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
  const int chunks = static_cast<int>((p.n + kArChunk - 1) / kArChunk);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(chunks);
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
