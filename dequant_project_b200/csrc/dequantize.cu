// Materialise a packed weight as fp16 [N, K], bit-exact with the reference
// packer's dequantize (KrishnaI2424/Dequant_Project dequant/packer.py:177-189):
// w = fp16((q - off) * scale) with the subtraction and the product each
// rounded in fp32 (round-to-nearest-even), then one rounding to fp16. It
// replaces dequantize_kernel (kernels/dequant_gemv.cu:113-140), the M > 8
// path of QuantLinear, and add_one (kernels/smoke.cu:9-13), the toolchain
// smoke kernel the reference binding also exports.
//
// One CTA per output row; its threads walk the row's packed words. Each
// thread turns one 32-bit word into 32/bits consecutive fp16 outputs and
// writes them with one 8/16/32-byte vector store, so the kernel is bound by
// the fp16 write stream (2 bytes per code).
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gemv.h"

namespace dqg {
namespace {

template <int BITS, bool INTER>
__device__ __forceinline__ int logical_of(int s) {
  if constexpr (!INTER) {
    return s;
  } else if constexpr (BITS == 4) {
    constexpr int o[8] = {0, 2, 4, 6, 1, 3, 5, 7};
    return o[s];
  } else if constexpr (BITS == 2) {
    constexpr int o[16] = {0, 4, 8, 12, 1, 5, 9, 13, 2, 6, 10, 14, 3, 7, 11, 15};
    return o[s];
  } else {
    constexpr int o[4] = {0, 2, 1, 3};
    return o[s];
  }
}

template <int BITS, bool SYM, bool INTER>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ qweight,
                                                         const __half* __restrict__ scales,
                                                         const __half* __restrict__ zeros,
                                                         __half* __restrict__ out, int N, int K,
                                                         int group_size) {
  constexpr int PP = 32 / BITS;
  constexpr uint32_t QMAX = (1u << BITS) - 1u;
  constexpr float BIAS = static_cast<float>(1 << (BITS - 1));
  const int words = K / PP;
  const int wpg = group_size / PP;  // words per group (group_size % PP == 0)
  const int G = K / group_size;
  for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
    const uint32_t* qrow = qweight + n * words;
    const __half* srow = scales + n * G;
    const __half* zrow = SYM ? nullptr : zeros + n * G;
    __half* orow = out + n * K;
    for (int w = threadIdx.x; w < words; w += blockDim.x) {
      const uint32_t word = __ldg(qrow + w);
      const int g = w / wpg;
      const float scale = __half2float(srow[g]);
      const float off = SYM ? BIAS : __half2float(zrow[g]);
      __align__(16) __half v[PP];
#pragma unroll
      for (int s = 0; s < PP; ++s) {
        const float q = static_cast<float>((word >> (BITS * s)) & QMAX);
        v[logical_of<BITS, INTER>(s)] = __float2half_rn(__fmul_rn(__fsub_rn(q, off), scale));
      }
      if constexpr (PP == 4) {
        *reinterpret_cast<uint2*>(orow + w * PP) = *reinterpret_cast<const uint2*>(v);
      } else {
#pragma unroll
        for (int i = 0; i < PP / 8; ++i)
          reinterpret_cast<uint4*>(orow + w * PP)[i] = reinterpret_cast<const uint4*>(v)[i];
      }
    }
  }
}

__global__ void add_one_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = in[i] + 1.0f;
}

template <int BITS, bool SYM, bool INTER>
cudaError_t launch(const DequantArgs& a, cudaStream_t stream) {
  const int grid = a.N < (1 << 30) ? a.N : (1 << 30);
  dequantize_kernel<BITS, SYM, INTER><<<grid, 256, 0, stream>>>(
      a.qweight, reinterpret_cast<const __half*>(a.scales),
      reinterpret_cast<const __half*>(a.zeros), reinterpret_cast<__half*>(a.out), a.N, a.K,
      a.group_size);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dequantize(const DequantArgs& a, cudaStream_t stream) {
#define DQG_DEQ_CASE(B, S, I) \
  if (a.bits == B && a.symmetric == S && a.interleaved == I) return launch<B, S, I>(a, stream);
  DQG_DEQ_CASE(2, false, false)
  DQG_DEQ_CASE(2, false, true)
  DQG_DEQ_CASE(2, true, false)
  DQG_DEQ_CASE(2, true, true)
  DQG_DEQ_CASE(4, false, false)
  DQG_DEQ_CASE(4, false, true)
  DQG_DEQ_CASE(4, true, false)
  DQG_DEQ_CASE(4, true, true)
  DQG_DEQ_CASE(8, false, false)
  DQG_DEQ_CASE(8, false, true)
  DQG_DEQ_CASE(8, true, false)
  DQG_DEQ_CASE(8, true, true)
#undef DQG_DEQ_CASE
  return cudaErrorInvalidValue;
}

cudaError_t launch_add_one(const float* x, float* out, int64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  add_one_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(x, out, n);
  return cudaGetLastError();
}

}  // namespace dqg
