// extern "C" entry points of libdequant_b200.so (declared in
// include/dequant_b200.h). Argument validation follows the reference
// extension's TORCH_CHECKs (kernels/dequant_gemv.cu:230-283 check_weight,
// :310-317 dequantize, :339-361 gemv, kernels/smoke.cu:15-25 add_one) with the
// same messages, adapted to raw pointers: dtype/contiguity checks become
// pointer-kind and alignment checks. Nothing here allocates or synchronises.
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dequant_b200.h"
#include "gemv.h"

namespace {

thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DQG_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int ok() {
  g_msg[0] = '\0';
  return DQG_OK;
}

// A pointer the kernels may dereference: device or managed memory of `dev`.
int check_device_ptr(const void* p, int dev, const char* name) {
  if (p == nullptr) return fail(DQG_ERR_INVALID, "%s must not be null", name);
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error this query may leave
    return fail(DQG_ERR_INVALID, "%s must be a CUDA tensor (%s)", name, cudaGetErrorString(e));
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(DQG_ERR_INVALID, "%s must be a CUDA tensor", name);
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev)
    return fail(DQG_ERR_INVALID, "%s and qweight must be on the same device", name);
  return DQG_OK;
}

// The driver's cuMemGetAddressRange, looked up at run time (the library does
// not link the driver library), or null where the driver does not offer it.
using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static const AddrRangeFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return static_cast<AddrRangeFn>(nullptr);
    }
    return reinterpret_cast<AddrRangeFn>(f);
  }();
  return fn;
}

// L2 prefetch ranges of a decode op, checked (each inside one device
// allocation of `dev`) and trimmed to 16-byte aligned starts and sizes.
int prepare_prefetch(const dqg_l2_spans* in, int dev, dqg::L2Spans* out) {
  std::memset(out, 0, sizeof(*out));
  if (in == nullptr || in->n == 0) return DQG_OK;
  if (in->n < 0 || in->n > 8)
    return fail(DQG_ERR_INVALID, "prefetch.n must be in [0, 8], got %d", static_cast<int>(in->n));
  const AddrRangeFn range = addr_range_fn();
  if (range == nullptr) return fail(DQG_ERR_UNSUPPORTED, "the driver has no cuMemGetAddressRange");
  for (int i = 0; i < in->n; ++i) {
    const uint64_t b = in->bytes[i];
    if (b == 0) continue;
    int rc = check_device_ptr(in->ptr[i], dev, "prefetch range");
    if (rc) return rc;
    CUdeviceptr base = 0;
    size_t size = 0;
    const uintptr_t p = reinterpret_cast<uintptr_t>(in->ptr[i]);
    if (range(&base, &size, static_cast<CUdeviceptr>(p)) != CUDA_SUCCESS)
      return fail(DQG_ERR_INVALID, "prefetch range %d is not inside a device allocation", i);
    if (p + b > static_cast<uintptr_t>(base) + size)
      return fail(DQG_ERR_INVALID, "prefetch range %d runs past the end of its allocation", i);
    const uintptr_t a = (p + 15) & ~static_cast<uintptr_t>(15);
    if (a - p >= b) continue;
    const uint64_t len = (b - (a - p)) & ~static_cast<uint64_t>(15);
    if (len == 0) continue;
    out->ptr[out->n] = reinterpret_cast<const uint8_t*>(a);
    out->bytes[out->n] = len;
    ++out->n;
  }
  return DQG_OK;
}

// Pointer-kind checks (cudaPointerGetAttributes on every operand) cost a few
// microseconds per call, which is comparable to a small GEMV; they run only
// when DQG_CHECK_POINTERS is set to a non-empty value other than "0". The
// Python binding checks tensor devices itself, and alignment and size checks
// always run.
bool pointer_checks() {
  static const bool on = [] {
    const char* v = std::getenv("DQG_CHECK_POINTERS");
    return v != nullptr && v[0] != '\0' && std::strcmp(v, "0") != 0;
  }();
  return on;
}

// Streaming-kernel plans of recent call shapes (direct-mapped, per thread):
// a decode step calls a handful of shapes over and over.
struct PlanEntry {
  int M, N, K, bits, group_size, sms;
  bool ok;
  dqg::StreamPlan plan;
  bool used;
};

bool cached_stream_plan(int M, int N, int K, int bits, int group_size, int sms,
                        dqg::StreamPlan* out) {
  thread_local PlanEntry cache[32] = {};
  const uint32_t h = (static_cast<uint32_t>(M) * 2654435761u) ^ (static_cast<uint32_t>(N) * 40503u) ^
                     (static_cast<uint32_t>(K) * 2246822519u) ^ static_cast<uint32_t>(bits << 3) ^
                     static_cast<uint32_t>(group_size) * 3266489917u ^ static_cast<uint32_t>(sms);
  PlanEntry& e = cache[(h ^ (h >> 15)) & 31];
  if (!(e.used && e.M == M && e.N == N && e.K == K && e.bits == bits &&
        e.group_size == group_size && e.sms == sms)) {
    e.ok = dqg::plan_stream(M, N, K, bits, group_size, sms, &e.plan);
    e.M = M; e.N = N; e.K = K; e.bits = bits; e.group_size = group_size; e.sms = sms;
    e.used = true;
  }
  if (e.ok) *out = e.plan;
  return e.ok;
}

// Direct-kernel plans of recent call shapes (same scheme as above).
struct DirectEntry {
  int M, N, K, bits, group_size, sms;
  bool ok;
  dqg::DirectPlan plan;
  bool used;
};

bool cached_direct_plan(int M, int N, int K, int bits, int group_size, int sms,
                        dqg::DirectPlan* out, bool fused = false) {
  thread_local DirectEntry cache_plain[32] = {};
  thread_local DirectEntry cache_fused[32] = {};
  DirectEntry* cache = fused ? cache_fused : cache_plain;
  const uint32_t h = (static_cast<uint32_t>(M) * 2654435761u) ^ (static_cast<uint32_t>(N) * 40503u) ^
                     (static_cast<uint32_t>(K) * 2246822519u) ^ static_cast<uint32_t>(bits << 3) ^
                     static_cast<uint32_t>(group_size) * 3266489917u ^ static_cast<uint32_t>(sms);
  DirectEntry& e = cache[(h ^ (h >> 15)) & 31];
  if (!(e.used && e.M == M && e.N == N && e.K == K && e.bits == bits &&
        e.group_size == group_size && e.sms == sms)) {
    e.ok = dqg::plan_direct(M, N, K, bits, group_size, sms, &e.plan, fused);
    e.M = M; e.N = N; e.K = K; e.bits = bits; e.group_size = group_size; e.sms = sms;
    e.used = true;
  }
  if (e.ok) *out = e.plan;
  return e.ok;
}

// 0: pick the kernel per shape (direct, else streaming, else general);
// 1: never the direct kernel; 2: the direct kernel wherever it has a plan
// (tests and comparisons).
std::atomic<int> g_gemv_path{0};

int sm_count(int dev) {
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cache[dev] = v;
  return v;
}

// check_weight (kernels/dequant_gemv.cu:230-283), scalar half: sizes, format
// and alignment. Runs before any CUDA call.
int check_weight_args(const int32_t* qweight, const void* scales, const void* zeros, int64_t N,
                      int64_t K, int64_t bits, int64_t group_size, int symmetric) {
  if (bits != 2 && bits != 4 && bits != 8)
    return fail(DQG_ERR_INVALID, "bits must be 2, 4 or 8, got %lld", (long long)bits);
  if (group_size <= 0)
    return fail(DQG_ERR_INVALID, "group_size must be positive, got %lld", (long long)group_size);
  if (K <= 0 || K % group_size != 0)
    return fail(DQG_ERR_INVALID, "K=%lld is not divisible by group_size=%lld", (long long)K,
                (long long)group_size);
  if (N <= 0)
    return fail(DQG_ERR_INVALID, "qweight must have at least one row, got N=%lld", (long long)N);
  if (K % (32 / bits) != 0)
    return fail(DQG_ERR_INVALID, "K=%lld is not a whole number of %lld-code words",
                (long long)K, (long long)(32 / bits));
  if (N > INT32_MAX || K > (1 << 24))
    return fail(DQG_ERR_UNSUPPORTED, "N=%lld, K=%lld exceed the supported sizes", (long long)N,
                (long long)K);
  if ((zeros != nullptr) == (symmetric != 0))
    return fail(DQG_ERR_INVALID, symmetric ? "symmetric=true takes no zeros"
                                           : "symmetric=false requires zeros");
  if (qweight == nullptr) return fail(DQG_ERR_INVALID, "qweight must not be null");
  if (scales == nullptr) return fail(DQG_ERR_INVALID, "scales must not be null");
  if (reinterpret_cast<uintptr_t>(qweight) % 4)
    return fail(DQG_ERR_INVALID, "qweight must be 4-byte aligned");
  if (reinterpret_cast<uintptr_t>(scales) % 2)
    return fail(DQG_ERR_INVALID, "scales must be 2-byte aligned");
  if (zeros && reinterpret_cast<uintptr_t>(zeros) % 2)
    return fail(DQG_ERR_INVALID, "zeros must be 2-byte aligned");
  return DQG_OK;
}

// check_weight, device half: every pointer is device (or managed) memory of
// the current device.
int check_weight_ptrs(const int32_t* qweight, const void* scales, const void* zeros, int dev) {
  int rc = check_device_ptr(qweight, dev, "qweight");
  if (rc) return rc;
  rc = check_device_ptr(scales, dev, "scales");
  if (rc) return rc;
  if (zeros) rc = check_device_ptr(zeros, dev, "zeros");
  return rc;
}

}  // namespace

extern "C" {

const char* dqg_last_error(void) { return g_msg; }

int dqg_version(void) { return 100; }

int dqg_add_one(const float* x, float* out, int64_t n, void* stream) {
  if (n < 0) return fail(DQG_ERR_INVALID, "n must be non-negative");
  if (n == 0) return ok();
  if (x == nullptr || out == nullptr) return fail(DQG_ERR_INVALID, "x and out must not be null");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int rc = check_device_ptr(x, dev, "x");
  if (rc) return rc;
  rc = check_device_ptr(out, dev, "out");
  if (rc) return rc;
  e = dqg::launch_add_one(x, out, n, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add_one launch");
  return ok();
}

int dqg_gemv(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
             void* y, int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
             int symmetric, int interleaved, void* stream) {
  if (M < 1 || M > dqg::kMaxM)
    return fail(DQG_ERR_INVALID,
                "gemv handles 1 <= M <= %d, got M=%lld; use the dequantize + F.linear fallback",
                dqg::kMaxM, (long long)M);
  int rc = check_weight_args(qweight, scales, zeros, N, K, bits, group_size, symmetric);
  if (rc) return rc;
  if (x == nullptr) return fail(DQG_ERR_INVALID, "x must not be null");
  if (y == nullptr) return fail(DQG_ERR_INVALID, "y must not be null");
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail(DQG_ERR_INVALID, "x must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(qweight) % 16)
    return fail(DQG_ERR_INVALID, "qweight must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(y) % 2) return fail(DQG_ERR_INVALID, "y must be 2-byte aligned");
  const int64_t cpl = 128 / bits;
  if (group_size % cpl != 0)
    return fail(DQG_ERR_INVALID,
                "group_size=%lld must be a multiple of %lld (the codes one lane loads per uint4) "
                "at %lld bits; this excludes INT2 with group_size 32",
                (long long)group_size, (long long)cpl, (long long)bits);
  const int wpl = dqg::gemv_words_per_lane(static_cast<int>(bits), static_cast<int>(group_size),
                                           static_cast<int>(K));
  if (wpl == 0 || K / (4 * wpl * (32 / bits)) >= 65536)
    return fail(DQG_ERR_UNSUPPORTED, "K=%lld is too large for the GEMV path", (long long)K);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (pointer_checks()) {
    rc = check_weight_ptrs(qweight, scales, zeros, dev);
    if (rc) return rc;
    rc = check_device_ptr(x, dev, "x");
    if (rc) return rc;
    rc = check_device_ptr(y, dev, "y");
    if (rc) return rc;
  }

  dqg::GemvArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.qweight = reinterpret_cast<const uint32_t*>(qweight);
  a.scales = static_cast<const uint16_t*>(scales);
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bits = static_cast<int>(bits);
  a.group_size = static_cast<int>(group_size);
  a.symmetric = symmetric != 0;
  a.interleaved = interleaved != 0;
  // The direct kernel for group-wise formats whose group is one MMA step and
  // whose activations fit one CTA; else the streaming kernel whenever its
  // plan fits (activations resident per CTA or per split-K cluster,
  // 16-byte-aligned scales/zeros); the general kernel otherwise.
  const int path = g_gemv_path.load();
  if (path != 1) {
    dqg::DirectPlan dplan;
    if (cached_direct_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                           static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev),
                           &dplan, path == 2)) {
      e = dqg::launch_direct(a, dplan, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
      return ok();
    }
  }
  dqg::StreamPlan splan;
  const bool meta_aligned = reinterpret_cast<uintptr_t>(scales) % 16 == 0 &&
                            (zeros == nullptr || reinterpret_cast<uintptr_t>(zeros) % 16 == 0);
  if (meta_aligned &&
      cached_stream_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                         static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev),
                         &splan)) {
    e = dqg::launch_stream(a, splan, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    return ok();
  }
  dqg::GemvPlan plan;
  if (!dqg::plan_gemv(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                      static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev), &plan))
    return fail(DQG_ERR_UNSUPPORTED, "no shared-memory plan for M=%lld K=%lld bits=%lld group=%lld",
                (long long)M, (long long)K, (long long)bits, (long long)group_size);
  e = dqg::launch_gemv(a, plan, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return ok();
}

int dqg_gemv_swiglu(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                    void* act, int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                    int symmetric, int interleaved, void* stream) {
  if (M < 1 || M > dqg::kMaxM)
    return fail(DQG_ERR_INVALID, "gemv handles 1 <= M <= %d, got M=%lld", dqg::kMaxM,
                (long long)M);
  int rc = check_weight_args(qweight, scales, zeros, N, K, bits, group_size, symmetric);
  if (rc) return rc;
  if (N % 16 != 0)
    return fail(DQG_ERR_INVALID, "N=%lld must be a multiple of 16 (8 gate rows, then 8 up rows)",
                (long long)N);
  if (x == nullptr || act == nullptr) return fail(DQG_ERR_INVALID, "x and act must not be null");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(qweight) % 16)
    return fail(DQG_ERR_INVALID, "x and qweight must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(act) % 2) return fail(DQG_ERR_INVALID, "act must be 2-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::DirectPlan dplan;
  if (!cached_direct_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                          static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev),
                          &dplan))
    return fail(DQG_ERR_UNSUPPORTED, "no direct-kernel plan for this shape and format");
  dqg::GemvArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.qweight = reinterpret_cast<const uint32_t*>(qweight);
  a.scales = static_cast<const uint16_t*>(scales);
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.y = static_cast<uint16_t*>(act);
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bits = static_cast<int>(bits);
  a.group_size = static_cast<int>(group_size);
  a.symmetric = symmetric != 0;
  a.interleaved = interleaved != 0;
  e = dqg::launch_direct(a, dplan, static_cast<cudaStream_t>(stream), nullptr, true);
  if (e != cudaSuccess) return cuda_fail(e, "gemv_swiglu launch");
  return ok();
}

int dqg_gemv_swiglu_supported(int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                              int* supported) {
  if (supported == nullptr) return fail(DQG_ERR_INVALID, "supported must not be null");
  *supported = 0;
  if (M < 1 || M > dqg::kMaxM || N < 16 || N % 16 != 0 || K < 1 || N > (1 << 30) ||
      K > (1 << 30) || (bits != 2 && bits != 4 && bits != 8) || group_size <= 0)
    return ok();
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::DirectPlan dplan;
  *supported = cached_direct_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                  static_cast<int>(bits), static_cast<int>(group_size),
                                  sm_count(dev), &dplan)
                   ? 1
                   : 0;
  return ok();
}

int dqg_dequantize(const int32_t* qweight, const void* scales, const void* zeros, void* out,
                   int64_t N, int64_t K, int64_t bits, int64_t group_size, int symmetric,
                   int interleaved, void* stream) {
  int rc = check_weight_args(qweight, scales, zeros, N, K, bits, group_size, symmetric);
  if (rc) return rc;
  const int64_t per_pack = 32 / bits;
  if (group_size % per_pack != 0)
    return fail(DQG_ERR_INVALID,
                "group_size=%lld must be a multiple of %lld values per uint32 word at %lld bits",
                (long long)group_size, (long long)per_pack, (long long)bits);
  if (out == nullptr) return fail(DQG_ERR_INVALID, "out must not be null");
  if (reinterpret_cast<uintptr_t>(out) % 16)
    return fail(DQG_ERR_INVALID, "out must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  rc = check_weight_ptrs(qweight, scales, zeros, dev);
  if (rc) return rc;
  rc = check_device_ptr(out, dev, "out");
  if (rc) return rc;
  dqg::DequantArgs a;
  a.qweight = reinterpret_cast<const uint32_t*>(qweight);
  a.scales = static_cast<const uint16_t*>(scales);
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.out = static_cast<uint16_t*>(out);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bits = static_cast<int>(bits);
  a.group_size = static_cast<int>(group_size);
  a.symmetric = symmetric != 0;
  a.interleaved = interleaved != 0;
  e = dqg::launch_dequantize(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequantize launch");
  return ok();
}

int dqg_add_rms_norm(void* h, const void* delta, const void* weight, void* y, int64_t M,
                     int64_t H, float eps, const dqg_l2_spans* prefetch, void* stream) {
  if (M < 1 || M > 65535) return fail(DQG_ERR_INVALID, "M must be in [1, 65535], got %lld", (long long)M);
  if (H < 8 || H % 8 != 0 || H > (1 << 24))
    return fail(DQG_ERR_INVALID, "H must be a positive multiple of 8, got %lld", (long long)H);
  if (!(eps >= 0.f)) return fail(DQG_ERR_INVALID, "eps must be non-negative");
  const void* ptrs[4] = {h, delta, weight, y};
  const char* names[4] = {"h", "delta", "weight", "y"};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  for (int i = 0; i < 4; ++i) {
    if (i == 1 && delta == nullptr) continue;
    int rc = check_device_ptr(ptrs[i], dev, names[i]);
    if (rc) return rc;
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16)
      return fail(DQG_ERR_INVALID, "%s must be 16-byte aligned", names[i]);
  }
  dqg::L2Spans pf;
  int rc = prepare_prefetch(prefetch, dev, &pf);
  if (rc) return rc;
  e = dqg::launch_add_rms_norm(h, delta, weight, y, static_cast<int>(M), static_cast<int>(H), eps,
                               pf, sm_count(dev), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "add_rms_norm launch");
  return ok();
}

int dqg_rope_kv_append(const void* qkv, const float* cos_row, const float* sin_row, void* q_out,
                       void* k_cache, void* v_cache, int64_t M, int64_t n_q_heads,
                       int64_t n_kv_heads, int64_t head_dim, int64_t pos, int64_t capacity,
                       const dqg_l2_spans* prefetch, void* stream) {
  if (M < 1 || M > 65535) return fail(DQG_ERR_INVALID, "M must be in [1, 65535], got %lld", (long long)M);
  if (n_q_heads < 1 || n_kv_heads < 1 || n_q_heads + n_kv_heads > 65535)
    return fail(DQG_ERR_INVALID, "head counts out of range (%lld query, %lld KV)",
                (long long)n_q_heads, (long long)n_kv_heads);
  if (head_dim < 2 || head_dim % 2 != 0 || head_dim > 1024)
    return fail(DQG_ERR_INVALID, "head_dim must be even and at most 1024, got %lld",
                (long long)head_dim);
  if (capacity < 1 || pos < 0 || pos >= capacity)
    return fail(DQG_ERR_INVALID, "position %lld outside the cache (capacity %lld)",
                (long long)pos, (long long)capacity);
  if (M * n_kv_heads * capacity * head_dim > (int64_t(1) << 40))
    return fail(DQG_ERR_INVALID, "cache too large");
  const void* ptrs[6] = {qkv, cos_row, sin_row, q_out, k_cache, v_cache};
  const char* names[6] = {"qkv", "cos", "sin", "q_out", "k_cache", "v_cache"};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  for (int i = 0; i < 6; ++i) {
    int rc = check_device_ptr(ptrs[i], dev, names[i]);
    if (rc) return rc;
  }
  dqg::L2Spans pf;
  int rc = prepare_prefetch(prefetch, dev, &pf);
  if (rc) return rc;
  e = dqg::launch_rope_kv_append(qkv, cos_row, sin_row, q_out, k_cache, v_cache,
                                 static_cast<int>(M), static_cast<int>(n_q_heads),
                                 static_cast<int>(n_kv_heads), static_cast<int>(head_dim),
                                 static_cast<int>(pos), static_cast<int>(capacity), pf,
                                 sm_count(dev), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_kv_append launch");
  return ok();
}

int dqg_silu_mul(const void* gate_up, void* out, int64_t M, int64_t I,
                 const dqg_l2_spans* prefetch, void* stream) {
  if (M < 1 || I < 1 || M * I > (int64_t(1) << 40))
    return fail(DQG_ERR_INVALID, "M and I must be positive (got %lld, %lld)", (long long)M,
                (long long)I);
  if (I > (int64_t(1) << 30)) return fail(DQG_ERR_INVALID, "I too large");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int rc = check_device_ptr(gate_up, dev, "gate_up");
  if (rc) return rc;
  rc = check_device_ptr(out, dev, "out");
  if (rc) return rc;
  dqg::L2Spans pf;
  rc = prepare_prefetch(prefetch, dev, &pf);
  if (rc) return rc;
  e = dqg::launch_silu_mul(gate_up, out, static_cast<int>(M), static_cast<int>(I), pf,
                           sm_count(dev), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "silu_mul launch");
  return ok();
}

int dqg_stream_plan(int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                    int num_sms, int32_t* out, int out_len) {
  if (out == nullptr || out_len < 23) return fail(DQG_ERR_INVALID, "out needs 23 entries");
  if (M < 1 || M > 8 || N < 1 || K < 1 || N > (1 << 30) || K > (1 << 30) || num_sms < 1)
    return fail(DQG_ERR_INVALID, "shape out of range");
  if (bits != 2 && bits != 4 && bits != 8) return fail(DQG_ERR_INVALID, "bits must be 2, 4 or 8");
  if (group_size <= 0 || K % group_size)
    return fail(DQG_ERR_INVALID, "K must be a multiple of group_size");
  dqg::StreamPlan pl;
  if (!dqg::plan_stream(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                        static_cast<int>(bits), static_cast<int>(group_size), num_sms, &pl))
    return fail(DQG_ERR_UNSUPPORTED, "no streaming plan for this shape");
  const int32_t v[23] = {pl.wpl, pl.mp, pl.ks, pl.n_slabs, pl.stages, pl.n_meta, pl.w_pitch,
                         pl.xp, pl.stage_bytes, pl.C, pl.KC, pl.off_x, pl.off_sstep, pl.off_sx,
                         pl.off_meta, pl.meta_half, pl.meta_stride, pl.off_red, pl.off_bar,
                         pl.off_xred, pl.off_zero, pl.smem, pl.grid};
  for (int i = 0; i < 23; ++i) out[i] = v[i];
  return ok();
}

int dqg_gemv_allreduce(const void* x, const int32_t* qweight, const void* scales,
                       const void* zeros, void* y, int64_t M, int64_t N, int64_t K, int64_t bits,
                       int64_t group_size, int symmetric, int interleaved,
                       const uint64_t* peer_data, const uint64_t* peer_flags, uint32_t* ctl,
                       int64_t cap, int rank, int world, uint64_t wait_ns, void* stream) {
  if (world < 2 || world > dqg::kArMaxRanks || rank < 0 || rank >= world)
    return fail(DQG_ERR_INVALID, "rank %d / world %d out of range (2 to %d ranks)", rank, world,
                dqg::kArMaxRanks);
  if (M < 1 || M > dqg::kMaxM)
    return fail(DQG_ERR_INVALID, "gemv handles 1 <= M <= %d, got M=%lld", dqg::kMaxM,
                (long long)M);
  int rc = check_weight_args(qweight, scales, zeros, N, K, bits, group_size, symmetric);
  if (rc) return rc;
  if (x == nullptr || y == nullptr || peer_data == nullptr || peer_flags == nullptr ||
      ctl == nullptr)
    return fail(DQG_ERR_INVALID, "pointers must not be null");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(qweight) % 16)
    return fail(DQG_ERR_INVALID, "x and qweight must be 16-byte aligned");
  if (M * N > cap)
    return fail(DQG_ERR_INVALID, "M * N = %lld exceeds the exchange capacity %lld",
                (long long)(M * N), (long long)cap);
  if (wait_ns != 0 && (wait_ns < 1000000ull || wait_ns > 10000000000ull))
    return fail(DQG_ERR_INVALID, "wait_ns must be 0 (default) or in [1 ms, 10 s]");
  for (int r = 0; r < world; ++r)
    if (peer_data[r] == 0 || peer_flags[r] == 0 || peer_data[r] % 16 || peer_flags[r] % 4)
      return fail(DQG_ERR_INVALID, "peer buffers of rank %d missing or misaligned", r);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::DirectPlan dplan;
  if (!cached_direct_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                          static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev),
                          &dplan, true) ||
      dplan.grid > dqg::kArMaxCtas)
    return fail(DQG_ERR_UNSUPPORTED, "no fused row-parallel plan for this shape");
  dqg::GemvArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.qweight = reinterpret_cast<const uint32_t*>(qweight);
  a.scales = static_cast<const uint16_t*>(scales);
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bits = static_cast<int>(bits);
  a.group_size = static_cast<int>(group_size);
  a.symmetric = symmetric != 0;
  a.interleaved = interleaved != 0;
  dqg::PeerGemvArgs ar;
  ar.rank = rank;
  ar.world = world;
  ar.data = reinterpret_cast<const unsigned long long*>(peer_data);
  ar.flags = reinterpret_cast<const unsigned long long*>(peer_flags);
  ar.ctl = ctl;
  ar.cap = cap;
  ar.wait_ns = wait_ns ? wait_ns : 2000000000ull;
  e = dqg::launch_direct(a, dplan, static_cast<cudaStream_t>(stream), &ar);
  if (e != cudaSuccess) return cuda_fail(e, "row-parallel gemv launch");
  return ok();
}

int dqg_decode_attention_workspace(int64_t M, int64_t n_q_heads, int64_t n_kv_heads,
                                   int64_t T, uint64_t* bytes) {
  if (bytes == nullptr) return fail(DQG_ERR_INVALID, "bytes must not be null");
  if (M < 1 || M > 65535 || n_kv_heads < 1 || n_q_heads < n_kv_heads ||
      n_q_heads % n_kv_heads != 0 || n_q_heads / n_kv_heads > 16 || n_q_heads > 65535)
    return fail(DQG_ERR_INVALID,
                "head counts (%lld query, %lld KV) must give 1..16 query heads per KV head",
                (long long)n_q_heads, (long long)n_kv_heads);
  if (T < 1 || T > (1 << 24)) return fail(DQG_ERR_INVALID, "T=%lld out of range", (long long)T);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  *bytes = dqg::attention_workspace_bytes(static_cast<int>(M), static_cast<int>(n_q_heads),
                                          static_cast<int>(n_kv_heads), static_cast<int>(T),
                                          sm_count(dev));
  return ok();
}

int dqg_decode_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                         void* workspace, uint64_t workspace_bytes, int64_t M, int64_t n_q_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t T, int64_t capacity,
                         void* stream) {
  if (head_dim != 128)
    return fail(DQG_ERR_UNSUPPORTED, "decode attention handles head_dim 128, got %lld",
                (long long)head_dim);
  uint64_t need = 0;
  int rc = dqg_decode_attention_workspace(M, n_q_heads, n_kv_heads, T, &need);
  if (rc) return rc;
  if (capacity < T)
    return fail(DQG_ERR_INVALID, "T=%lld positions exceed the cache capacity %lld", (long long)T,
                (long long)capacity);
  if (M * n_kv_heads * capacity * head_dim > (int64_t(1) << 40))
    return fail(DQG_ERR_INVALID, "cache too large");
  if (workspace == nullptr || workspace_bytes < need)
    return fail(DQG_ERR_INVALID, "workspace of %llu bytes needed, %llu given",
                (unsigned long long)need, (unsigned long long)workspace_bytes);
  const void* ptrs[5] = {q, k_cache, v_cache, out, workspace};
  const char* names[5] = {"q", "k_cache", "v_cache", "out", "workspace"};
  for (int i = 0; i < 5; ++i) {
    if (ptrs[i] == nullptr) return fail(DQG_ERR_INVALID, "%s must not be null", names[i]);
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16)
      return fail(DQG_ERR_INVALID, "%s must be 16-byte aligned", names[i]);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::AttnParams p;
  p.q = static_cast<const __half*>(q);
  p.kc = static_cast<const __half*>(k_cache);
  p.vc = static_cast<const __half*>(v_cache);
  p.o = static_cast<__half*>(out);
  p.M = static_cast<int>(M);
  p.Hq = static_cast<int>(n_q_heads);
  p.Hkv = static_cast<int>(n_kv_heads);
  p.g = p.Hq / p.Hkv;
  p.cap = static_cast<int>(capacity);
  p.T = static_cast<int>(T);
  p.S = dqg::attention_splits(p.M, p.Hkv, p.T, sm_count(dev), &p.Ts);
  const size_t mh = static_cast<size_t>(M) * n_kv_heads;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t cnt = dqg::attention_counter_bytes(p.M, p.Hkv);
  p.tickets = reinterpret_cast<unsigned*>(ws);
  p.ml = reinterpret_cast<float*>(ws + cnt);
  p.part = reinterpret_cast<float*>(ws + cnt + mh * p.S * p.g * 2 * 4);
  p.scale_log2 = static_cast<float>(1.4426950408889634 / 11.313708498984761);  // log2(e)/sqrt(128)
  e = dqg::launch_decode_attention(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode attention launch");
  return ok();
}

int dqg_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                 void* out, int64_t M, int64_t n_q_heads, int64_t n_kv_heads,
                                 int64_t head_dim, int64_t T, int64_t capacity, void* stream) {
  if (head_dim != 128)
    return fail(DQG_ERR_UNSUPPORTED, "decode attention handles head_dim 128, got %lld",
                (long long)head_dim);
  uint64_t need = 0;
  int rc = dqg_decode_attention_workspace(M, n_q_heads, n_kv_heads, T, &need);
  if (rc) return rc;
  if (need > dqg::attention_noalloc_capacity())
    return fail(DQG_ERR_UNSUPPORTED,
                "this call needs %llu bytes of scratch; the library's static scratch holds %llu "
                "(use dqg_decode_attention with a workspace)",
                (unsigned long long)need, (unsigned long long)dqg::attention_noalloc_capacity());
  if (capacity < T)
    return fail(DQG_ERR_INVALID, "T=%lld positions exceed the cache capacity %lld", (long long)T,
                (long long)capacity);
  if (M * n_kv_heads * capacity * head_dim > (int64_t(1) << 40))
    return fail(DQG_ERR_INVALID, "cache too large");
  const void* ptrs[4] = {q, k_cache, v_cache, out};
  const char* names[4] = {"q", "k_cache", "v_cache", "out"};
  for (int i = 0; i < 4; ++i) {
    if (ptrs[i] == nullptr) return fail(DQG_ERR_INVALID, "%s must not be null", names[i]);
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16)
      return fail(DQG_ERR_INVALID, "%s must be 16-byte aligned", names[i]);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::AttnParams p;
  p.q = static_cast<const __half*>(q);
  p.kc = static_cast<const __half*>(k_cache);
  p.vc = static_cast<const __half*>(v_cache);
  p.o = static_cast<__half*>(out);
  p.M = static_cast<int>(M);
  p.Hq = static_cast<int>(n_q_heads);
  p.Hkv = static_cast<int>(n_kv_heads);
  p.g = p.Hq / p.Hkv;
  p.cap = static_cast<int>(capacity);
  p.T = static_cast<int>(T);
  p.S = dqg::attention_splits(p.M, p.Hkv, p.T, sm_count(dev), &p.Ts);
  p.scale_log2 = static_cast<float>(1.4426950408889634 / 11.313708498984761);  // log2(e)/sqrt(128)
  e = dqg::launch_decode_attention_noalloc(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode attention (static scratch) launch");
  return ok();
}

int dqg_set_gemv_path(int path) {
  if (path < 0 || path > 2) return -1;
  return g_gemv_path.exchange(path);
}

int dqg_set_weight_prefetch(int enable) {
  const int prev = dqg::weight_prefetch() ? 1 : 0;
  dqg::set_weight_prefetch(enable != 0);
  return prev;
}

int dqg_debug_gemv_starved(const int32_t* qweight, const void* scales, const void* zeros,
                           void* y, const void* x, int64_t M, int64_t N, int64_t K, int64_t bits,
                           int64_t group_size, int symmetric, int interleaved,
                           uint64_t wait_ns, void* stream) {
  if (wait_ns < 1000000ull || wait_ns > 1000000000ull)
    return fail(DQG_ERR_INVALID, "wait_ns must be in [1 ms, 1 s], got %llu",
                (unsigned long long)wait_ns);
  if (M < 1 || M > dqg::kMaxM) return fail(DQG_ERR_INVALID, "M must be in [1, %d]", dqg::kMaxM);
  int rc = check_weight_args(qweight, scales, zeros, N, K, bits, group_size, symmetric);
  if (rc) return rc;
  if (x == nullptr || y == nullptr) return fail(DQG_ERR_INVALID, "x and y must not be null");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(qweight) % 16 ||
      reinterpret_cast<uintptr_t>(scales) % 16 ||
      (zeros != nullptr && reinterpret_cast<uintptr_t>(zeros) % 16))
    return fail(DQG_ERR_INVALID, "x, qweight, scales and zeros must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  dqg::StreamPlan splan;
  if (!dqg::plan_stream(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                        static_cast<int>(bits), static_cast<int>(group_size), sm_count(dev),
                        &splan))
    return fail(DQG_ERR_UNSUPPORTED, "no streaming plan for this shape");
  if (splan.C != 1)
    return fail(DQG_ERR_UNSUPPORTED, "the starved diagnostic runs single-CTA plans only");
  dqg::GemvArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.qweight = reinterpret_cast<const uint32_t*>(qweight);
  a.scales = static_cast<const uint16_t*>(scales);
  a.zeros = static_cast<const uint16_t*>(zeros);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.bits = static_cast<int>(bits);
  a.group_size = static_cast<int>(group_size);
  a.symmetric = symmetric != 0;
  a.interleaved = interleaved != 0;
  e = dqg::launch_stream(a, splan, static_cast<cudaStream_t>(stream), wait_ns, true);
  if (e != cudaSuccess) return cuda_fail(e, "starved gemv launch");
  return ok();
}

int dqg_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr)
    return fail(DQG_ERR_INVALID, "ptr, handle and offset must not be null");
  // Base of the allocation that holds ptr (the IPC handle names the whole
  // allocation); the driver function is looked up at run time so that the
  // library does not link the driver.
  using AddrRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddrRange range_fn = nullptr;
  if (range_fn == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(DQG_ERR_CUDA, "cuMemGetAddressRange is not available");
    range_fn = reinterpret_cast<AddrRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(DQG_ERR_INVALID, "ptr is not device memory of this process");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - base);
  return ok();
}

int dqg_ipc_open(const void* handle, void** base) {
  if (handle == nullptr || base == nullptr)
    return fail(DQG_ERR_INVALID, "handle and base must not be null");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return ok();
}

int dqg_ipc_close(void* base) {
  if (base == nullptr) return fail(DQG_ERR_INVALID, "base must not be null");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return ok();
}

int dqg_peer_allreduce(const void* in, void* out, int64_t n, const uint64_t* peer_bufs,
                       uint32_t* ctl, int64_t cap, int rank, int world, uint64_t wait_ns,
                       void* stream) {
  if (world < 1 || world > dqg::kArMaxRanks || rank < 0 || rank >= world)
    return fail(DQG_ERR_INVALID, "rank %d / world %d out of range (at most %d ranks)", rank, world,
                dqg::kArMaxRanks);
  if (n < 8 || n % 8 != 0 || n > cap)
    return fail(DQG_ERR_INVALID, "n=%lld must be a positive multiple of 8 and at most cap=%lld",
                (long long)n, (long long)cap);
  if (cap % 8 != 0) return fail(DQG_ERR_INVALID, "cap must be a multiple of 8");
  if (in == nullptr || out == nullptr || peer_bufs == nullptr || ctl == nullptr)
    return fail(DQG_ERR_INVALID, "pointers must not be null");
  if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    return fail(DQG_ERR_INVALID, "in and out must be 16-byte aligned");
  if (wait_ns != 0 && (wait_ns < 1000000ull || wait_ns > 10000000000ull))
    return fail(DQG_ERR_INVALID, "wait_ns must be 0 (default) or in [1 ms, 10 s]");
  dqg::PeerReduceParams p = {};
  p.in = static_cast<const __half*>(in);
  p.out = static_cast<__half*>(out);
  p.n = n;
  p.cap = cap;
  for (int r = 0; r < world; ++r) {
    if (peer_bufs[r] == 0 || peer_bufs[r] % 16)
      return fail(DQG_ERR_INVALID, "peer buffers of rank %d missing or misaligned", r);
    p.peer_data[r] = peer_bufs[r];
  }
  p.ctl = ctl;
  p.rank = rank;
  p.world = world;
  p.wait_ns = wait_ns ? wait_ns : 2000000000ull;
  cudaError_t e = dqg::launch_peer_allreduce(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "peer_allreduce launch");
  return ok();
}

int dqg_peer_allreduce_add_rms_norm(const void* partial, void* h, const void* weight, void* y,
                                    int64_t M, int64_t H, float eps, const uint64_t* peer_bufs,
                                    uint32_t* ctl, int64_t cap, int rank, int world,
                                    uint64_t wait_ns, void* stream) {
  if (world < 1 || world > dqg::kArMaxRanks || rank < 0 || rank >= world)
    return fail(DQG_ERR_INVALID, "rank %d / world %d out of range (at most %d ranks)", rank, world,
                dqg::kArMaxRanks);
  if (H < 8 || H % 8 != 0 || H > dqg::kArNormMaxH)
    return fail(DQG_ERR_INVALID, "H must be a multiple of 8 in [8, %d], got %lld", dqg::kArNormMaxH,
                (long long)H);
  if (M < 1 || M > 65535 || M * H > cap)
    return fail(DQG_ERR_INVALID, "M=%lld rows of H=%lld must be at least one and fit cap=%lld",
                (long long)M, (long long)H, (long long)cap);
  if (cap % 8 != 0) return fail(DQG_ERR_INVALID, "cap must be a multiple of 8");
  if (!(eps >= 0.f)) return fail(DQG_ERR_INVALID, "eps must be non-negative");
  if (partial == nullptr || h == nullptr || weight == nullptr || y == nullptr ||
      peer_bufs == nullptr || ctl == nullptr)
    return fail(DQG_ERR_INVALID, "pointers must not be null");
  const void* al[4] = {partial, h, weight, y};
  for (const void* q : al)
    if (reinterpret_cast<uintptr_t>(q) % 16)
      return fail(DQG_ERR_INVALID, "partial, h, weight and y must be 16-byte aligned");
  if (wait_ns != 0 && (wait_ns < 1000000ull || wait_ns > 10000000000ull))
    return fail(DQG_ERR_INVALID, "wait_ns must be 0 (default) or in [1 ms, 10 s]");
  dqg::PeerNormParams q = {};
  q.ar.in = static_cast<const __half*>(partial);
  q.ar.out = nullptr;
  q.ar.n = M * H;
  q.ar.cap = cap;
  for (int r = 0; r < world; ++r) {
    if (peer_bufs[r] == 0 || peer_bufs[r] % 16)
      return fail(DQG_ERR_INVALID, "peer buffers of rank %d missing or misaligned", r);
    q.ar.peer_data[r] = peer_bufs[r];
  }
  q.ar.ctl = ctl;
  q.ar.rank = rank;
  q.ar.world = world;
  q.ar.wait_ns = wait_ns ? wait_ns : 2000000000ull;
  q.h = static_cast<__half*>(h);
  q.w = static_cast<const __half*>(weight);
  q.y = static_cast<__half*>(y);
  q.M = static_cast<int>(M);
  q.H = static_cast<int>(H);
  q.eps = eps;
  cudaError_t e = dqg::launch_peer_allreduce_add_rms_norm(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "peer_allreduce_add_rms_norm launch");
  return ok();
}

int dqg_device_status(int device, uint32_t* status, int reset) {
  if (status == nullptr) return fail(DQG_ERR_INVALID, "status must not be null");
  cudaError_t e = dqg::read_device_status(device, status, reset != 0);
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  return ok();
}

}  // extern "C"
