"""Host side of the peer all-reduce, on gloo CPU ranks (no GPU): every rank
maps every other rank's exchange buffer exactly once, builds its pointer
tables in rank order (its own buffer in its own slot, peers at their handle's
offset), lays the buffer out as the all-reduce's receive packets (both
parity halves, one slot per rank), the fused GEMV's exchange and its flags,
releases each mapping once, and refuses calls after close()."""

from __future__ import annotations

import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", (2, 4))
def test_gloo_ranks_exchange_and_map_every_peer(world):
    import tp_workers
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_workers.peer_exchange, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    out, t0 = {}, time.time()
    while len(out) < world and time.time() - t0 < 120:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert set(out) == set(range(world)), out
    for r, (status, info) in out.items():
        assert status == "ok", info
        others = [s for s in range(world) if s != r]
        opened_ranks = [int(h.split(":")[0][4:]) for h in info["opened"]]
        assert opened_ranks == others                     # each peer once, in rank order
        for s in others:                                  # the handle a peer exported
            assert f"rank{s}:{out[s][1]['own']}" in info["opened"]
        assert info["bufs"][r] == info["own"]
        assert len(info["bufs"]) == world and len(set(info["bufs"])) == world
        packet_bytes = 8 * world * info["cap"]            # all-reduce receive packets first
        assert [d - b for d, b in zip(info["data"], info["bufs"])] == [packet_bytes] * world
        gemv_off = packet_bytes + 2 * info["cap"] * 4     # then the fused GEMV's fp32 exchange
        assert [f - b for f, b in zip(info["gemv_flags"], info["bufs"])] == [gemv_off] * world
        assert info["cap"] == 5000
        assert info["nbytes"] == gemv_off + 1024 * world * 4
        assert info["closed"] == world - 1                # close() is idempotent
        assert "after close" in info["after_close"]
