/*
 * dequant_b200 -- C ABI of the B200 (sm_100a) packed low-bit dequant + GEMV
 * library, libdequant_b200.so.
 *
 * Drop-in boundary for the `dequant_cuda` torch extension of
 * KrishnaI2424/Dequant_Project (kernels/dequant_cuda.h, kernels/bindings.cpp):
 * the same three operations with the same argument meaning and the same
 * validation rules, expressed with plain device pointers, sizes and a CUDA
 * stream instead of torch tensors. No torch types cross this boundary.
 *
 * Conventions
 *   - All data pointers are CUDA device pointers on the stream's device. fp16
 *     tensors are passed as `const void *` (IEEE binary16, little endian).
 *   - The packed format is the reference packer's (dequant/packer.py:7-29):
 *     qweight is int32 [N, K * bits / 32] (uint32 bit patterns), scales are
 *     fp16 [N, K / group_size], zeros are fp16 [N, K / group_size] when
 *     asymmetric and NULL when symmetric; codes are unsigned and symmetric
 *     codes are biased by 2^(bits-1); `interleaved` selects the reference's
 *     _INTERLEAVE slot order (dequant/packer.py:37-41).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *     asynchronous on that stream, allocates nothing, never synchronises and
 *     never reads device data on the host, so it can be captured in a CUDA
 *     graph.
 *   - Return value: DQG_OK (0) or a non-zero dqg_status; the message of the
 *     most recent failure on the calling thread is dqg_last_error(). Invalid
 *     arguments are rejected before anything is launched.
 */
#ifndef DEQUANT_B200_H_
#define DEQUANT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dqg_status {
  DQG_OK = 0,
  DQG_ERR_INVALID = 1,     /* argument rejected (shape, format, alignment, pointer) */
  DQG_ERR_UNSUPPORTED = 2, /* valid but outside what this build handles */
  DQG_ERR_CUDA = 3         /* a CUDA runtime call failed */
} dqg_status;

/* Human-readable message of the last failure on this thread ("" if none). */
const char *dqg_last_error(void);

/* ABI version of this header/library pair (major * 100 + minor). */
int dqg_version(void);

/*
 * out[i] = x[i] + 1 for n fp32 values.
 * Replaces add_one (kernels/smoke.cu:15-25, bound at kernels/bindings.cpp:6),
 * the reference's toolchain smoke test.
 */
int dqg_add_one(const float *x, float *out, int64_t n, void *stream);

/*
 * y = x @ W^T for a packed W: x fp16 [M, K] row-major with 1 <= M <= 8,
 * y fp16 [M, N] row-major, fp32 accumulation.
 * Replaces gemv (kernels/dequant_cuda.h:12-15, kernels/dequant_gemv.cu:339-386,
 * bound at kernels/bindings.cpp:8-11) with the same checks:
 *   bits in {2, 4, 8}; group_size > 0; K % group_size == 0;
 *   group_size % (128 / bits) == 0 (so INT2 with group 32 is rejected);
 *   zeros != NULL exactly when symmetric == 0; x 16-byte aligned.
 * Additionally qweight must be 16-byte aligned (it is streamed with bulk
 * copies). group_size == K is per-channel quantisation. Whether each pointer
 * is device memory of the current device is checked only when the
 * environment variable DQG_CHECK_POINTERS is set (those queries cost about as
 * much as a small GEMV); see also dqg_set_weight_prefetch.
 */
int dqg_gemv(const void *x, const int32_t *qweight, const void *scales, const void *zeros,
             void *y, int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
             int symmetric, int interleaved, void *stream);

/*
 * out = dequantize(W) as fp16 [N, K], bit-exact with packer.dequantize.
 * Replaces dequantize (kernels/dequant_cuda.h:17-20,
 * kernels/dequant_gemv.cu:310-337, bound at kernels/bindings.cpp:13-16):
 *   bits in {2, 4, 8}; group_size > 0; K % group_size == 0;
 *   group_size % (32 / bits) == 0; zeros != NULL exactly when symmetric == 0.
 */
int dqg_dequantize(const int32_t *qweight, const void *scales, const void *zeros, void *out,
                   int64_t N, int64_t K, int64_t bits, int64_t group_size, int symmetric,
                   int interleaved, void *stream);

/*
 * Device-side status of `device` (bit 0: a kernel of this library gave up a
 * bounded wait), the OR of the status words of all its kernels. Synchronous;
 * for tests and diagnostics, not for the hot path.
 * If reset != 0 the word is cleared after reading. No reference counterpart:
 * the reference kernels have no waits.
 */
int dqg_device_status(int device, uint32_t *status, int reset);

/*
 * Process-wide switch, default on; returns the previous setting. When on,
 * dqg_gemv's streaming kernel issues its first ring of packed-weight copies
 * (qweight, scales, zeros) before it waits for the kernel that precedes it on
 * the stream, so those copies overlap that kernel's tail (programmatic
 * dependent launch; the activations are always read after the wait). The
 * packed weight must then not be written by the immediately preceding kernel
 * if that kernel lets dependent launches start early (griddepcontrol
 * launch_dependents); kernels that do not (every torch kernel) complete
 * before the GEMV starts. Turn it off for weights produced that way. No
 * reference counterpart: the reference kernel has no dependent launch.
 */
int dqg_set_weight_prefetch(int enable);

/*
 * Process-wide choice of dqg_gemv's kernel, for tests and comparisons; returns
 * the previous setting (or -1 for an invalid path). 0 (default): per shape,
 * the direct kernel (4/8-bit group-wise formats whose group is one
 * tensor-core step of a lane, rows of at most 6144 codes, M >= 5), else the
 * streaming kernel, else the general one. 1: never the direct kernel. 2: the
 * direct kernel wherever it applies, any M. Results agree within the GEMV
 * tolerance; each kernel is deterministic. No reference counterpart.
 */
int dqg_set_gemv_path(int path);

/*
 * Diagnostic for the bounded-wait path: launches the streaming GEMV kernel for
 * this shape with its copy-issuing warp doing nothing, so that every wait in
 * the kernel gives up after wait_ns (1 ms to 1 s) and the kernel returns with
 * bit 0 set in the device status word (dqg_device_status); y is left
 * unwritten. Only shapes whose plan is a single CTA per row block (no split-K
 * cluster) are accepted. For tests; no reference counterpart.
 */
int dqg_debug_gemv_starved(const int32_t *qweight, const void *scales, const void *zeros,
                           void *y, const void *x, int64_t M, int64_t N, int64_t K,
                           int64_t bits, int64_t group_size, int symmetric, int interleaved,
                           uint64_t wait_ns, void *stream);

/*
 * Tensor-parallel plumbing: CUDA IPC of device memory between the processes
 * of one node (no reference counterpart; the reference has no multi-GPU
 * code, dequant/byte_model.py:179-251 only models the decoder's bytes).
 * dqg_ipc_export writes the 64-byte IPC handle of the allocation holding ptr
 * and ptr's byte offset in it; dqg_ipc_open maps a peer's handle into this
 * process (base address of the peer allocation); dqg_ipc_close unmaps it.
 */
int dqg_ipc_export(const void *ptr, void *handle, uint64_t *offset);
int dqg_ipc_open(const void *handle, void **base);
int dqg_ipc_close(void *base);

/*
 * One-shot all-reduce (sum) of n fp16 values (n a multiple of 8, at most cap)
 * across `world` ranks of one node, out = sum over ranks of in (in == out is
 * allowed), summed in rank order in fp32 and rounded once, so every rank gets
 * the same bits. Replaces the NCCL all-reduce that follows each row-parallel
 * layer of the decoder step (the reference has none; it models the bytes in
 * dequant/byte_model.py:179-251). Each rank stores its values straight into
 * every peer's receive buffer as 8-byte packets (a 32-bit data word and a
 * 32-bit flag carrying the call's epoch, written together) and polls its own
 * buffer until every peer's packets of the call have arrived.
 *   peer_bufs[r] : rank r's receive buffer of 8 * world * cap bytes (two
 *                  parity halves of `world` slots of cap / 2 packets),
 *                  16-byte aligned (this rank's own buffer at r == rank, IPC
 *                  mappings of the others), zero-initialised once;
 *   ctl          : this rank's two uint32 call counters, zero-initialised once.
 * Every rank must make the same sequence of calls. Each wait for a peer is
 * bounded by wait_ns (0 = 2 s); a wait that runs out sets bit 0 of
 * dqg_device_status and leaves those values of out unwritten. Peer memory is
 * only written, with plain stores (no loads, bulk copies or multicast). The
 * host array peer_bufs is read during the call only; nothing is allocated.
 */
int dqg_peer_allreduce(const void *in, void *out, int64_t n, const uint64_t *peer_bufs,
                       uint32_t *ctl, int64_t cap, int rank, int world, uint64_t wait_ns,
                       void *stream);

/*
 * The all-reduce of a row-parallel layer's output fused with the residual add
 * + RMSNorm that follows it in the decoder step (no reference counterpart;
 * the reference only models these bytes, dequant/byte_model.py:179-251):
 * delta = the rank-order fp32 sum over ranks of `partial` [M, H] rounded to
 * fp16, exactly as dqg_peer_allreduce gives it, then, exactly as
 * dqg_add_rms_norm with that delta, h = fp16(h + delta) in place and
 * y = fp16((h * rsqrt(mean(h^2) + eps)) * weight). Same receive buffers,
 * call counters and rules as dqg_peer_allreduce (the two may be mixed in one
 * sequence of calls); M * H <= cap, H a multiple of 8 up to 8192, all tensors
 * fp16 and 16-byte aligned; partial is left unchanged. A row whose exchange
 * ran out of time (bit 0 of dqg_device_status) leaves h and y unwritten.
 * One launch instead of two, one CTA per row.
 */
int dqg_peer_allreduce_add_rms_norm(const void *partial, void *h, const void *weight, void *y,
                                    int64_t M, int64_t H, float eps, const uint64_t *peer_bufs,
                                    uint32_t *ctl, int64_t cap, int rank, int world,
                                    uint64_t wait_ns, void *stream);

/*
 * Row-parallel GEMV fused with its all-reduce: every rank passes its slice of
 * the input dimension (x [M, K_r], W_r [N, K_r] packed, as dqg_gemv) and gets
 * y = sum over ranks of x_r @ W_r^T, fp16 [M, N], the same bits on every rank.
 * One kernel: each CTA writes its rows' fp32 partial into this rank's
 * exchange buffer, raises its flag on every rank, waits (bounded by wait_ns,
 * 0 = 2 s) for the same CTA's flag of every rank and sums the ranks' partials
 * in rank order, reading peers with plain loads (no bulk copies, no
 * multicast); CTAs that finish early exchange while the others still stream.
 *   peer_data[r]  : rank r's exchange buffer, 2 * cap fp32 values, 16-byte
 *                   aligned (IPC mappings for the peers); M * N <= cap;
 *   peer_flags[r] : rank r's flag array, 1024 * world uint32, zeroed once;
 *   ctl           : this rank's two uint32 call counters, zeroed once (not
 *                   shared with dqg_peer_allreduce).
 * Every rank must make the same sequence of calls. Returns
 * DQG_ERR_UNSUPPORTED for shapes without a fused plan (then call dqg_gemv and
 * dqg_peer_allreduce). Replaces gemv + the NCCL all-reduce that follows each
 * row-parallel layer; the reference has neither (it models the bytes in
 * dequant/byte_model.py:179-251).
 */
int dqg_gemv_allreduce(const void *x, const int32_t *qweight, const void *scales,
                       const void *zeros, void *y, int64_t M, int64_t N, int64_t K, int64_t bits,
                       int64_t group_size, int symmetric, int interleaved,
                       const uint64_t *peer_data, const uint64_t *peer_flags, uint32_t *ctl,
                       int64_t cap, int rank, int world, uint64_t wait_ns, void *stream);

/*
 * The streaming GEMV kernel's launch plan for a shape (host arithmetic only,
 * no device access): out[0..22] = wpl, mp, ks, n_slabs, stages, n_meta,
 * w_pitch, xp, stage_bytes, C (cluster size), KC (codes per cluster rank),
 * off_x, off_sstep, off_sx, off_meta, meta_half, meta_stride, off_red, off_bar,
 * off_xred, off_zero, smem (bytes), grid. Returns DQG_ERR_UNSUPPORTED when the
 * shape takes the fallback kernel. For tests and diagnostics; no reference
 * counterpart.
 */
int dqg_stream_plan(int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                    int num_sms, int32_t *out, int out_len);

/*
 * Element-wise steps of the tensor-parallel decoder around the GEMVs
 * (dequant_project_b200/decoder.py). No reference counterpart: the reference
 * only models the decode step as bytes (dequant/byte_model.py:179-251). fp16
 * tensors, row-major, on the current device.
 */

/*
 * Byte ranges that a decode op brings into L2 while it runs, for the packed
 * weights of a GEMV that follows it (every CTA of the op issues its share of
 * bulk L2 prefetches before it waits for the previous kernel; the op's grid
 * is widened to the SM count so that the prefetches are spread over every
 * SM). A range whose start is not 16-byte aligned is trimmed to the aligned
 * part; sizes are rounded down to 16 bytes. Up to 8 ranges, n of them used;
 * NULL or n == 0 prefetches nothing. The ranges must be device memory of the
 * current device that stays allocated while the op may run.
 */
typedef struct dqg_l2_spans {
  const void *ptr[8];
  uint64_t bytes[8];
  int32_t n;
} dqg_l2_spans;

/*
 * Residual add + RMSNorm over rows of H values (H % 8 == 0, all pointers
 * 16-byte aligned): if delta != NULL, h[m] = fp16(h[m] + delta[m]) in place;
 * then y[m] = fp16((h[m] * rsqrt(mean(h[m]^2) + eps)) * weight), fp32 math.
 * This op, dqg_rope_kv_append and dqg_silu_mul take an optional prefetch
 * (dqg_l2_spans above).
 */
int dqg_add_rms_norm(void *h, const void *delta, const void *weight, void *y, int64_t M,
                     int64_t H, float eps, const dqg_l2_spans *prefetch, void *stream);

/*
 * Rotate-half RoPE at one position and KV-cache append. qkv is [M, (Hq +
 * 2 Hkv) * D] (query heads, then key heads, then value heads); cos_row and
 * sin_row are fp32 [D] for the position. Rotated queries go to q_out
 * [M, Hq, D]; rotated keys and the values go to slot `pos` of k_cache and
 * v_cache [M, Hkv, capacity, D].
 */
int dqg_rope_kv_append(const void *qkv, const float *cos_row, const float *sin_row, void *q_out,
                       void *k_cache, void *v_cache, int64_t M, int64_t n_q_heads,
                       int64_t n_kv_heads, int64_t head_dim, int64_t pos, int64_t capacity,
                       const dqg_l2_spans *prefetch, void *stream);

/*
 * Decode attention: one query token per sequence over its KV cache.
 * q is [M, Hq, 128] (rotated), k_cache/v_cache are [M, Hkv, capacity, 128]
 * with positions 0..T-1 valid, Hq a multiple of Hkv (at most 16 query heads
 * per KV head, grouped consecutively); out[m, h] = softmax(q[m, h] .
 * K[m, h / (Hq / Hkv), :T]^T / sqrt(128)) V[...], fp32 softmax, fp16 out.
 * workspace: dqg_decode_attention_workspace(M, Hq, Hkv, T) bytes or more,
 * 16-byte aligned, zeroed once before its first use and then left to the
 * library (it keeps its split counters at zero between calls); calls that
 * share a workspace must not overlap on the GPU. The split of positions over
 * CTAs depends on T and the device's SM count; a workspace sized for some T
 * serves every call with fewer positions (size it for the cache capacity).
 */
int dqg_decode_attention_workspace(int64_t M, int64_t n_q_heads, int64_t n_kv_heads, int64_t T,
                                   uint64_t *bytes);
int dqg_decode_attention(const void *q, const void *k_cache, const void *v_cache, void *out,
                         void *workspace, uint64_t workspace_bytes, int64_t M, int64_t n_q_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t T, int64_t capacity,
                         void *stream);

/*
 * Decode attention exactly as dqg_decode_attention, for callers that cannot
 * allocate device memory (for example a host whose GPU memory is all owned by
 * another allocator, such as a server that reserves it for KV caches at
 * start-up and gives each kernel only the step's tensors): no workspace
 * argument. No counterpart in the reference; it exists for such callers only.
 * The scratch is a static array of 2 MiB inside the library, held by every GPU
 * that loads the library until the process exits; a call whose split partials
 * need more (dqg_decode_attention_workspace reports the size) is rejected with
 * DQG_ERR_UNSUPPORTED. The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture. Every call shares the array: its split counters are cleared on the
 * stream before each launch, and calls that overlap on the GPU race on it.
 * Nothing is allocated (no cudaMalloc, no cudaFree).
 */
int dqg_decode_attention_noalloc(const void *q, const void *k_cache, const void *v_cache,
                                 void *out, int64_t M, int64_t n_q_heads, int64_t n_kv_heads,
                                 int64_t head_dim, int64_t T, int64_t capacity, void *stream);

/*
 * The decoder's gate/up GEMV fused with its SwiGLU (no reference counterpart:
 * the reference only models these bytes, dequant/byte_model.py:221-242). The
 * packed weight [N, K] (format as dqg_gemv) holds the gate and up rows
 * interleaved by eights: rows 16b .. 16b + 7 are gate rows 8b .. 8b + 7 and rows
 * 16b + 8 .. 16b + 15 the matching up rows (N a multiple of 16).
 * act[m, 8b + i] = fp16(silu(g) * u) with g and u the fp16-rounded GEMV
 * outputs of those two rows, in dqg_silu_mul's arithmetic, so the result
 * equals dqg_gemv on the interleaved weight followed by dqg_silu_mul on the
 * de-interleaved halves. act is [M, N / 2]. One launch of the direct kernel;
 * formats and shapes without a direct-kernel plan (4/8-bit group-wise
 * formats whose group is one step, K up to 6144) return DQG_ERR_UNSUPPORTED.
 */
int dqg_gemv_swiglu(const void *x, const int32_t *qweight, const void *scales, const void *zeros,
                    void *act, int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                    int symmetric, int interleaved, void *stream);
/* *supported = 1 when dqg_gemv_swiglu has a plan for this shape and format on
 * the current device, else 0 (host only, no launch). */
int dqg_gemv_swiglu_supported(int64_t M, int64_t N, int64_t K, int64_t bits, int64_t group_size,
                              int *supported);

/*
 * SwiGLU: gate_up is [M, 2 I] (gate columns, then up columns);
 * out[m, i] = fp16(silu(gate) * up), silu(g) = g / (1 + exp(-g)) in fp32.
 */
int dqg_silu_mul(const void *gate_up, void *out, int64_t M, int64_t I,
                 const dqg_l2_spans *prefetch, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* DEQUANT_B200_H_ */
