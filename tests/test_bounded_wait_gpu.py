"""Bounded device waits end in an error status, not a hang.

``dqg_debug_gemv_starved`` launches the streaming GEMV kernel with its
copy-issuing warp doing nothing, so every mbarrier wait in the kernel runs
out after a short limit (20 ms here). The kernel must return on its own, set
bit 0 of the device status word (read through ``dqg_device_status``, which
ORs the words of every kernel file: this one lives in the 4-bit streaming
unit), leave y unwritten, and leave the CUDA context usable: a normal GEMV
right after it is correct and sets no status bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bench_inputs
from dequant_project_b200 import _native, dequant_cuda
from oracle import native
from oracle import packer_np as P

pytestmark = pytest.mark.gpu

WAIT_NS = 20_000_000


def _packed(n, k):
    w, x = bench_inputs(n, k)
    qw, s, z = P.quantize_tensor(w.numpy(), 4, 128, False, "sequential")
    return x.numpy(), qw, s, z


def test_starved_gemv_gives_up_and_reports(cuda_device):
    n, k = 4096, 4096
    x, qw, s, z = _packed(n, k)
    xd, qd, sd, zd = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
                      for a in (x, qw, s, z))
    torch.cuda.synchronize()
    _native.device_status(cuda_device.index, reset=True)
    sentinel = torch.full((1, n), 7.0, dtype=torch.float16, device=cuda_device)
    lib = _native.lib()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    _native.check(lib.dqg_debug_gemv_starved(
        qd.data_ptr(), sd.data_ptr(), zd.data_ptr(), sentinel.data_ptr(), xd.data_ptr(),
        1, n, k, 4, 128, 0, 0, WAIT_NS, stream))
    torch.cuda.synchronize()  # returns: every wait gave up after WAIT_NS
    status = _native.device_status(cuda_device.index, reset=True)
    assert status & 1, f"status {status:#x}: no wait reported giving up"
    assert bool((sentinel == 7.0).all()), "a starved kernel wrote y"
    assert _native.device_status(cuda_device.index) == 0, "reset did not clear the status"

    # The context is still usable and the next call is correct.
    y = dequant_cuda.gemv(xd, qd, sd, zd, 4, 128, False, False).cpu().numpy()
    yref = native.gemv(x, qw, s, z, 4, 128, False, False)
    assert P.max_rel_err(y, yref) <= 2e-3
    torch.cuda.synchronize()
    assert _native.device_status(cuda_device.index) == 0


def test_prefetch_switch_gives_identical_results(cuda_device):
    """The weight ring issued before or after the dependent-launch wait: the
    same kernel arithmetic, bit-identical outputs."""
    lib = _native.lib()
    n, k = 11008, 4096
    x, qw, s, z = _packed(n, k)
    xd, qd, sd, zd = (torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)
                      for a in (x, qw, s, z))
    prev = lib.dqg_set_weight_prefetch(1)
    try:
        y_on = dequant_cuda.gemv(xd, qd, sd, zd, 4, 128, False, False)
        assert lib.dqg_set_weight_prefetch(0) == 1
        y_off = dequant_cuda.gemv(xd, qd, sd, zd, 4, 128, False, False)
    finally:
        lib.dqg_set_weight_prefetch(prev)
    assert torch.equal(y_on, y_off)
