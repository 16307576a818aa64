// Element-wise kernels of the decoder step around the packed GEMVs: residual
// add + RMSNorm, RoPE + KV-cache append, SwiGLU. Each replaces a chain of
// small torch kernels with one launch; all are tiny next to the GEMVs (a
// decode step moves kilobytes through them) and are bound by launch latency,
// so each is a single pass with one CTA per row or per head.
//
// All three are launched with programmatic dependent launch and wait for the
// previous grid (griddepcontrol.wait) before touching memory, then at once let
// the next grid launch: a GEMV that follows can be scheduled and run its own
// set-up while one of these runs, and one of these can be scheduled while a
// GEMV runs, so their launch latencies overlap instead of adding up.
//
// Each can also carry byte ranges of a later GEMV's packed weights to bring
// into L2 (bulk L2 prefetches issued before the dependency wait). The decoder
// step leaves HBM idle while these ops, the attention and each GEMV's start
// and end run; prefetching the next weights there lets that GEMV read them
// from L2. The grid is widened to the SM count so every SM's copy engine
// issues a share; the extra CTAs only prefetch and exit (the op's own CTAs
// still wait for the previous grid, so the chain of dependencies holds).
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv.h"

namespace dqg {
namespace {

constexpr int kNormThreads = 256;
constexpr uint64_t kPrefetchPiece = 16384;  // bytes per bulk L2 prefetch

// This CTA's share of the prefetch ranges: piece j of a range goes to CTA
// j % ncta (so that every SM's copy engine takes part), thread j / ncta.
// Fire and forget: nothing waits for these, and the op's own work does not
// depend on them.
__device__ __forceinline__ void l2_prefetch_share(const L2Spans& pf, int cta, int ncta) {
  const uint64_t rank = static_cast<uint64_t>(threadIdx.x) * ncta + cta;
  const uint64_t nt = static_cast<uint64_t>(ncta) * blockDim.x;
  for (int i = 0; i < pf.n; ++i) {
    const uint64_t n = pf.bytes[i];
    for (uint64_t off = rank * kPrefetchPiece; off < n; off += nt * kPrefetchPiece) {
      const uint32_t len = static_cast<uint32_t>(n - off < kPrefetchPiece ? n - off : kPrefetchPiece);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf.ptr[i] + off), "r"(len)
                   : "memory");
    }
  }
}

__device__ __forceinline__ float h2f(__half v) { return __half2float(v); }

// h[m] = fp16(h[m] + delta[m]) (when delta is given), then
// y[m] = fp16((h * rsqrt(mean(h^2) + eps)) * w), in fp32 with the two products
// rounded one at a time as torch evaluates them.
// CTAs m >= M only issue their share of the prefetch.
__global__ void __launch_bounds__(kNormThreads)
    add_rms_norm_kernel(__half* __restrict__ h, const __half* __restrict__ delta,
                        const __half* __restrict__ w, __half* __restrict__ y, int M, int H,
                        float eps, const __grid_constant__ L2Spans pf) {
  if (pf.n) l2_prefetch_share(pf, blockIdx.x, gridDim.x);
  const int m = blockIdx.x;
  if (m >= M) return;
  pdl_wait_prior_grid();
  pdl_launch_dependents();
  __half* hr = h + static_cast<int64_t>(m) * H;
  const __half* dr = delta ? delta + static_cast<int64_t>(m) * H : nullptr;
  __half* yr = y + static_cast<int64_t>(m) * H;
  const int nv = H / 8;
  float ss = 0.f;
  for (int v = threadIdx.x; v < nv; v += kNormThreads) {
    uint4 a = reinterpret_cast<const uint4*>(hr)[v];
    __half* ah = reinterpret_cast<__half*>(&a);
    if (dr) {
      const uint4 b = reinterpret_cast<const uint4*>(dr)[v];
      const __half* bh = reinterpret_cast<const __half*>(&b);
#pragma unroll
      for (int i = 0; i < 8; ++i) ah[i] = __float2half_rn(__fadd_rn(h2f(ah[i]), h2f(bh[i])));
      reinterpret_cast<uint4*>(hr)[v] = a;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float f = h2f(ah[i]);
      ss = __fmaf_rn(f, f, ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(H)), eps));
  // Each thread re-reads the vectors it wrote above (same indices).
  for (int v = threadIdx.x; v < nv; v += kNormThreads) {
    const uint4 a = reinterpret_cast<const uint4*>(hr)[v];
    const uint4 b = reinterpret_cast<const uint4*>(w)[v];
    const __half* ah = reinterpret_cast<const __half*>(&a);
    const __half* wh = reinterpret_cast<const __half*>(&b);
    uint4 o;
    __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = __float2half_rn(__fmul_rn(__fmul_rn(h2f(ah[i]), r), h2f(wh[i])));
    reinterpret_cast<uint4*>(yr)[v] = o;
  }
}

// One block per (sequence, head): query heads are rotated into q_out; key
// heads are rotated into the key cache at `pos`, and the matching value head
// is copied into the value cache at `pos`. Rotate-half RoPE:
//   out[i]     = x[i] * cos[i]         + (-x[i + D/2]) * sin[i]
//   out[i+D/2] = x[i + D/2] * cos[i+D/2] + x[i] * sin[i + D/2]
// each product and the sum rounded in fp32, then to fp16.
// Grid (M, hq + hkv, z): CTAs with blockIdx.z > 0 only prefetch.
__global__ void rope_kv_append_kernel(const __half* __restrict__ qkv, const float* __restrict__ cosv,
                                      const float* __restrict__ sinv, __half* __restrict__ q_out,
                                      __half* __restrict__ kc, __half* __restrict__ vc, int hq,
                                      int hkv, int D, int pos, int cap,
                                      const __grid_constant__ L2Spans pf) {
  if (pf.n)
    l2_prefetch_share(pf, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                      gridDim.x * gridDim.y * gridDim.z);
  if (blockIdx.z > 0) return;
  pdl_wait_prior_grid();
  pdl_launch_dependents();
  const int m = blockIdx.x;
  const int hd = blockIdx.y;
  const int half = D / 2;
  const __half* row = qkv + static_cast<int64_t>(m) * (hq + 2 * hkv) * D;
  const __half* src;
  __half* dst;
  if (hd < hq) {
    src = row + static_cast<int64_t>(hd) * D;
    dst = q_out + (static_cast<int64_t>(m) * hq + hd) * D;
  } else {
    const int k = hd - hq;
    const int64_t slot = ((static_cast<int64_t>(m) * hkv + k) * cap + pos) * D;
    src = row + static_cast<int64_t>(hq + k) * D;
    dst = kc + slot;
    const __half* vs = row + static_cast<int64_t>(hq + hkv + k) * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) vc[slot + i] = vs[i];
  }
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = h2f(src[i]);
    const float b = h2f(src[i + half]);
    const float lo = __fadd_rn(__fmul_rn(a, cosv[i]), __fmul_rn(-b, sinv[i]));
    const float hi = __fadd_rn(__fmul_rn(b, cosv[i + half]), __fmul_rn(a, sinv[i + half]));
    dst[i] = __float2half_rn(lo);
    dst[i + half] = __float2half_rn(hi);
  }
}

// out[m, i] = fp16(silu(g) * u), g = gu[m, i], u = gu[m, I + i],
// silu(g) = g / (1 + exp(-g)) in fp32.
__global__ void silu_mul_kernel(const __half* __restrict__ gu, __half* __restrict__ out, int I,
                                int64_t total, const __grid_constant__ L2Spans pf) {
  if (pf.n) l2_prefetch_share(pf, blockIdx.x, gridDim.x);
  pdl_wait_prior_grid();
  pdl_launch_dependents();
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = e / I;
    const int i = static_cast<int>(e - m * I);
    const float g = h2f(gu[m * 2 * I + i]);
    const float u = h2f(gu[m * 2 * I + I + i]);
    const float s = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
    out[e] = __float2half_rn(__fmul_rn(s, u));
  }
}

}  // namespace

// Launch with the programmatic-stream-serialization attribute (see top).
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, int threads, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

cudaError_t launch_add_rms_norm(void* h, const void* delta, const void* w, void* y, int M, int H,
                                float eps, const L2Spans& pf, int num_sms, cudaStream_t stream) {
  const int grid = pf.n && M < num_sms ? num_sms : M;
  return launch_pdl(add_rms_norm_kernel, dim3(grid), kNormThreads, stream, static_cast<__half*>(h),
                    static_cast<const __half*>(delta), static_cast<const __half*>(w),
                    static_cast<__half*>(y), M, H, eps, pf);
}

cudaError_t launch_rope_kv_append(const void* qkv, const float* cosv, const float* sinv,
                                  void* q_out, void* kc, void* vc, int M, int hq, int hkv, int D,
                                  int pos, int cap, const L2Spans& pf, int num_sms,
                                  cudaStream_t stream) {
  const int threads = D / 2 < 32 ? 32 : (D / 2 > 256 ? 256 : D / 2);
  const int base = M * (hq + hkv);
  const int z = pf.n && base < num_sms ? (num_sms + base - 1) / base : 1;
  return launch_pdl(rope_kv_append_kernel, dim3(M, hq + hkv, z), threads, stream,
                    static_cast<const __half*>(qkv), cosv, sinv, static_cast<__half*>(q_out),
                    static_cast<__half*>(kc), static_cast<__half*>(vc), hq, hkv, D, pos, cap, pf);
}

cudaError_t launch_silu_mul(const void* gu, void* out, int M, int I, const L2Spans& pf,
                            int num_sms, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(M) * I;
  const int threads = 256;
  const int sms = num_sms > 0 ? num_sms : 148;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 4 * sms) blocks = 4 * sms;
  if (pf.n && blocks < sms) blocks = sms;
  return launch_pdl(silu_mul_kernel, dim3(static_cast<unsigned>(blocks)), threads, stream,
                    static_cast<const __half*>(gu), static_cast<__half*>(out), I, total, pf);
}

}  // namespace dqg
