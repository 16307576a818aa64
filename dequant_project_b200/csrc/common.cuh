// Device-side building blocks shared by the sm_100a kernels of this library:
// mbarrier pipeline primitives, untiled bulk copies global->shared, named
// barriers, a bounded wait that reports instead of hanging, and small
// integer helpers. Hand-written inline PTX; no library code.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace dqg {

// Bits of the device status word g_status. A kernel that
// gives up a bounded wait ORs one of these in and returns instead of hanging;
// the host reads it with dqg_device_status().
enum : uint32_t {
  kStatusWaitTimeout = 1u << 0,   // an mbarrier wait ran past its time limit
};

// One status word per translation unit that includes this header (internal
// linkage; the library is built without relocatable device code). Every unit
// whose kernels wait exports a reader of its own word (DQG_STATUS_READER
// below), and the library's status query ORs all of them together.
static __device__ uint32_t g_status = 0;

// Upper bound on any single mbarrier wait (nanoseconds of %globaltimer). A
// healthy stage wait is microseconds; this is five orders of magnitude above.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make mbarrier.init visible to the async proxy (bulk copies) and other threads.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// Suspend-time hint for try_wait (ns): a waiting warp sleeps in hardware
// until the phase completes (or this much time passes) instead of spinning
// and taking issue slots from the warps that do the work.
constexpr uint32_t kSuspendHintNs = 1000000u;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Bounded: after
// limit_ns the wait gives up, flags kStatusWaitTimeout in g_status and
// returns false so that the caller can leave its loop and the kernel ends.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(&g_status, kStatusWaitTimeout);
      return false;
    }
  }
}

// mbar_wait taken by all 32 lanes of a warp with a warp-uniform outcome, so
// that a timed-out warp leaves its loop as a whole (no lane is left behind in
// a later __syncwarp or vote).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const bool ok = mbar_wait(bar, parity, limit_ns);
  return __all_sync(0xffffffffu, ok);
}

// ---- thread-block clusters (distributed shared memory) ----

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of all CTAs of the cluster; used once after barrier init so that
// no CTA touches a peer's barriers before they exist. (Hardware barrier: the
// CTAs of a cluster are always co-scheduled.)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// The same cluster barrier for threads that may arrive from different points
// of their code (not converged within a warp).
__device__ __forceinline__ void cluster_sync_all_unaligned() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (address from
// map_to_rank), releasing this thread's earlier writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_addr)
               : "memory");
}

// Bounded wait, acquiring at cluster scope (for barriers that peers arrive on).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool warp_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  bool ok = mbar_try_wait_cluster(bar, parity);
  if (!ok) {
    const uint64_t t0 = globaltimer();
    while (true) {
      if (mbar_try_wait_cluster(bar, parity)) {
        ok = true;
        break;
      }
      if (globaltimer() - t0 > limit_ns) {
        atomicOr(&g_status, kStatusWaitTimeout);
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// Untiled bulk copy global -> this CTA's shared memory, completing as
// transaction bytes on `bar`. dst, src and bytes must be multiples of 16.
// No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: let the next grid in the stream start its
// prologue (it still waits for this grid before reading our outputs), and wait
// for the previous grid before reading anything it may have produced.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// L2 policies for the bulk copies: packed weights are streamed exactly once
// per call (evict first); activations are re-read by every CTA (evict last).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- peer memory (other GPUs' buffers mapped through CUDA IPC) ----

// Store / acquire-load of a flag at system scope (visible across GPUs).
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Wait until *flag >= epoch (wrap-safe), bounded by limit_ns; false (and the
// timeout bit in g_status) when the limit ran out.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* flag, uint32_t epoch,
                                              uint64_t limit_ns) {
  if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const uint64_t t0 = globaltimer();
  while (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) < 0) {
    if (globaltimer() - t0 > limit_ns) {
      atomicOr(&g_status, kStatusWaitTimeout);
      return false;
    }
  }
  return true;
}

// Named barrier among a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// d = (a & b) | c, one LOP3.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Select two fp16 halves from {lo: a, hi: b} by byte selector (PRMT).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

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

// floor(n / d) for n < 2^16 and 1 <= d < 2^16, with magic = ceil(2^32 / d)
// (magic == 0 encodes d == 1). Exact in that range: the error of the
// reciprocal is below n / 2^32 < 1 / d.
__device__ __forceinline__ uint32_t fast_div(uint32_t n, uint32_t magic) {
  return magic ? __umulhi(n, magic) : n;
}

}  // namespace dqg

// Host-side reader of this translation unit's status word: defines
// `cudaError_t NAME(uint32_t* status, bool reset)` (current device).
#define DQG_STATUS_READER(NAME)                                                 \
  namespace dqg {                                                               \
  cudaError_t NAME(uint32_t* status, bool reset) {                              \
    cudaError_t e = cudaMemcpyFromSymbol(status, g_status, sizeof(uint32_t));   \
    if (e == cudaSuccess && reset) {                                            \
      const uint32_t zero = 0;                                                  \
      e = cudaMemcpyToSymbol(g_status, &zero, sizeof(uint32_t));                \
    }                                                                           \
    return e;                                                                   \
  }                                                                             \
  }
