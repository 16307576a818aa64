"""One-shot all-reduce over NVLink peer memory for the tensor-parallel decoder.

The decoder's row-parallel layers (O and down projections) end in an
all-reduce of a few KB to a few hundred KB of fp16 partial outputs, two per
layer (the reference's ``dequant/byte_model.py:179-251`` counts these bytes;
the reference itself has no multi-GPU code). At these
sizes a collective is bound by latency, not bandwidth, so this replaces NCCL's
algorithms with one exchange round through memory every rank can address:

* at set-up, each rank allocates one buffer (the all-reduce's receive
  packets, the fused GEMV's fp32 exchange and its flags) and call counters,
  zeroed; the buffers' CUDA IPC handles are swapped over the process group
  (``all_gather_object``) and every peer's buffer is mapped into this process;
* each call (``dqg_peer_allreduce`` in libdequant_b200.so) stores the input
  into every peer's receive buffer as packets that carry the call's epoch
  beside each data word, waits (bounded) until every peer's packets have
  arrived in this rank's buffer and sums all ranks' values in rank order in
  fp32 with one rounding, so every rank gets the same bits;
* ``gemv`` runs a row-parallel layer as ONE kernel (``dqg_gemv_allreduce``):
  the GEMV's CTAs write their rows' fp32 partials into this buffer and
  exchange them through the same peer mappings while other CTAs still stream
  weights; shapes without a fused plan take the GEMV, then the all-reduce.

The call counter lives on the device, so calls can be captured in a CUDA graph
and replayed. All ranks must make the same sequence of calls, as with any
collective. ``close()`` unmaps the peers' buffers; call it (or let the decoder
call it) before the process group is destroyed.
"""

from __future__ import annotations

import ctypes

import torch

from dequant_project_b200 import _native

MAX_RANKS = 8
MAX_GEMV_CTAS = 1024  # flags of the fused row-parallel GEMV: one per CTA and rank
HANDLE_BYTES = 64     # sizeof(cudaIpcMemHandle_t)


class CudaIpc:
    """CUDA IPC of device memory through the library's C ABI."""

    def export(self, ptr: int) -> tuple[bytes, int]:
        buf = ctypes.create_string_buffer(HANDLE_BYTES)
        off = ctypes.c_uint64(0)
        _native.check(_native.lib().dqg_ipc_export(ptr, buf, ctypes.byref(off)))
        return buf.raw, off.value

    def open(self, handle: bytes) -> int:
        base = ctypes.c_void_p(0)
        _native.check(_native.lib().dqg_ipc_open(handle, ctypes.byref(base)))
        return base.value

    def close(self, base: int) -> None:
        _native.check(_native.lib().dqg_ipc_close(base))


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


class PeerAllReduce:
    """Sum-all-reduce of fp16 tensors of at most ``max_elems`` values across
    the ranks of ``group`` (one process per GPU of one node, at most 8).

    ``ipc`` maps buffers between processes (``CudaIpc`` by default; the CPU
    tests pass a stand-in to check the exchange). ``wait_ns`` bounds each wait
    for a peer (0: the library's 2 s)."""

    def __init__(self, group, device, max_elems: int, wait_ns: int = 0, ipc=None):
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= MAX_RANKS:
            raise ValueError(f"peer all-reduce takes 1..{MAX_RANKS} ranks, got {self.world}")
        if max_elems < 8:
            raise ValueError("max_elems must be at least 8")
        self.device = torch.device(device)
        self.cap = _round_up(max_elems, 8)
        self.wait_ns = int(wait_ns)
        self._ipc = ipc if ipc is not None else CudaIpc()
        # One allocation, so one handle per rank: [all-reduce receive packets
        # (two parity halves of `world` slots of cap / 2 eight-byte packets) |
        # fused-GEMV exchange (fp32, two parity halves of cap values) |
        # fused-GEMV flags].
        packet_bytes = 8 * self.world * self.cap
        data_bytes = 2 * self.cap * 4
        gemv_flag_bytes = MAX_GEMV_CTAS * self.world * 4
        self.buffer = torch.zeros(packet_bytes + data_bytes + gemv_flag_bytes,
                                  dtype=torch.uint8, device=self.device)
        # Call counters: [all-reduce epoch, ticket, fused-GEMV epoch, ticket].
        self.ctl = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._data_off = packet_bytes
        self._gemv_flag_off = packet_bytes + data_bytes
        handle, offset = self._ipc.export(self.buffer.data_ptr())
        infos = [None] * self.world
        dist.all_gather_object(infos, (self.rank, handle, offset), group=group)
        self._opened: list[int] = []
        data_ptrs = []
        for r, (rr, h, off) in enumerate(infos):
            if rr != r:
                raise RuntimeError(f"peer exchange out of order: slot {r} holds rank {rr}")
            if r == self.rank:
                data_ptrs.append(self.buffer.data_ptr())
            else:
                base = self._ipc.open(h)
                self._opened.append(base)
                data_ptrs.append(base + off)
        self.peer_bufs = (ctypes.c_uint64 * self.world)(*data_ptrs)
        self.peer_data = (ctypes.c_uint64 * self.world)(*[p + self._data_off for p in data_ptrs])
        self.peer_gemv_flags = (ctypes.c_uint64 * self.world)(
            *[p + self._gemv_flag_off for p in data_ptrs])
        # No rank may write into a buffer its peer has not mapped yet.
        dist.barrier(group=group)

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over ranks of the contiguous fp16 tensor ``t``."""
        if self._opened is None:
            raise RuntimeError("peer all-reduce used after close()")
        if t.dtype != torch.float16 or not t.is_contiguous() or t.device != self.device:
            raise RuntimeError("peer all-reduce takes a contiguous float16 tensor on its device")
        n = t.numel()
        if n % 8 or n > self.cap or n == 0:
            raise RuntimeError(f"{n} values: need a positive multiple of 8 up to {self.cap}")
        _native.check(_native.lib().dqg_peer_allreduce(
            t.data_ptr(), t.data_ptr(), n, self.peer_bufs, self.ctl.data_ptr(),
            self.cap, self.rank, self.world, self.wait_ns,
            torch.cuda.current_stream(self.device).cuda_stream))
        return t

    def add_rms_norm(self, partial: torch.Tensor, h: torch.Tensor, weight: torch.Tensor,
                     eps: float) -> torch.Tensor:
        """The all-reduce of ``partial`` [M, H] fused with the residual add +
        RMSNorm after it (one kernel): ``h += sum over ranks of partial`` in
        place and the returned fp16 ``RMSNorm(h) * weight``, the same bits as
        this all-reduce followed by ``decode_ops.add_rms_norm``. ``partial`` is
        left unchanged."""
        if self._opened is None:
            raise RuntimeError("peer all-reduce used after close()")
        for t in (partial, h, weight):
            if t.dtype != torch.float16 or not t.is_contiguous() or t.device != self.device:
                raise RuntimeError("fused all-reduce + RMSNorm takes contiguous float16 tensors "
                                   "on its device")
        m, hd = h.shape
        if tuple(partial.shape) != (m, hd) or weight.numel() != hd:
            raise RuntimeError(f"shapes differ: partial {tuple(partial.shape)}, h {(m, hd)}, "
                               f"weight {weight.numel()}")
        y = torch.empty_like(h)
        _native.check(_native.lib().dqg_peer_allreduce_add_rms_norm(
            partial.data_ptr(), h.data_ptr(), weight.data_ptr(), y.data_ptr(), m, hd, float(eps),
            self.peer_bufs, self.ctl.data_ptr(), self.cap, self.rank, self.world, self.wait_ns,
            torch.cuda.current_stream(self.device).cuda_stream))
        return y

    def gemv(self, x: torch.Tensor, pw) -> torch.Tensor:
        """Row-parallel layer: the sum over ranks of ``x_r @ W_r^T`` for this
        rank's slice ``x`` [M, K_r] and packed ``pw`` [N, K_r]; fp16 [M, N],
        the same on every rank."""
        from dequant_project_b200 import quant_linear as ql
        if self._opened is None:
            raise RuntimeError("peer all-reduce used after close()")
        n, k = pw.shape
        x2 = x.reshape(-1, k).contiguous()
        m = x2.shape[0]
        bits, gs, sym, inter = ql._format_args(pw.config, k)
        if m <= ql.MAX_M and m * n <= self.cap:
            y = torch.empty((m, n), dtype=torch.float16, device=self.device)
            rc = _native.lib().dqg_gemv_allreduce(
                x2.data_ptr(), pw.qweight.data_ptr(), pw.scales.data_ptr(),
                None if pw.zeros is None else pw.zeros.data_ptr(), y.data_ptr(), m, n, k, bits,
                gs, int(sym), int(inter), self.peer_data, self.peer_gemv_flags,
                self.ctl.data_ptr() + 8, self.cap, self.rank, self.world, self.wait_ns,
                torch.cuda.current_stream(self.device).cuda_stream)
            if rc == 0:
                return y.view(*x.shape[:-1], n)
            if rc != 2:                       # anything but "no fused plan" is an error
                _native.check(rc)
        return self(ql.gemv(x2, pw)).view(*x.shape[:-1], n)

    def close(self) -> None:
        """Unmap the peers' buffers (idempotent)."""
        if self._opened is None:
            return
        for base in self._opened:
            self._ipc.close(base)
        self._opened = None
