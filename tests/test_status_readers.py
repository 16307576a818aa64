"""Every kernel file whose kernels can give up a bounded wait exports a reader
of its own status word, and dqg_device_status ORs all of them (each
translation unit has its own copy of the word; a file left out would make its
timeouts invisible). Checked on the sources, no GPU needed."""

from __future__ import annotations

import re

from conftest import ROOT

CSRC = ROOT / "dequant_project_b200" / "csrc"
# A bounded wait through the shared helpers, or a kernel's own poll that sets
# the timeout bit itself.
WAITS = re.compile(r"\b(warp_wait|mbar_wait|warp_wait_cluster|wait_flag_sys)\s*\(|"
                   r"atomicOr\(&g_status, kStatusWaitTimeout\)")


def _text_with_includes(path):
    text = path.read_text()
    for inc in re.findall(r'#include "([^"]+\.cuh)"', text):
        p = CSRC / inc
        if p.exists() and p.name != "common.cuh":
            text += _text_with_includes(p)
    return text


def test_every_waiting_file_is_read_by_device_status():
    readers = set()
    for cu in sorted(CSRC.glob("*.cu")):
        text = _text_with_includes(cu)
        if WAITS.search(text):
            m = re.search(r"DQG_STATUS_READER\((\w+)\)", cu.read_text())
            assert m, f"{cu.name} waits but exports no status reader"
            readers.add(m.group(1))
    src = (CSRC / "gemv.cu").read_text()
    block = src[src.index("cudaError_t read_device_status("):]
    block = block[:block.index("}")]
    listed = set(re.findall(r"read_status_\w+", block))
    assert readers <= listed, f"not read by dqg_device_status: {sorted(readers - listed)}"
    assert len(readers) >= 8
