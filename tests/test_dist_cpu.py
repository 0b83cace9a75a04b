"""World-size-2 gloo tests of the multi-rank host logic (CPU, no GPU): bench.py's rank
helpers, the relay-plan exchange between ranks, and failure detection when a rank dies."""
import json
import socket
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent))
import _dist_workers as W  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(fn, world, tmp_path, timeout=120):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process did not finish within {timeout}s")
    return procs


def test_dist_helpers_gloo_world2(tmp_path):
    procs = _run(W.helpers, 2, tmp_path)
    assert [p.exitcode for p in procs] == [0, 0]
    for r in range(2):
        res = json.loads((tmp_path / f"r{r}.json").read_text())
        assert res["max"] == 1.5                                  # max over ranks
        assert res["gather"] == ["handle-0", "handle-1"]          # rank order
        assert res["bcast"] == "nccl-unique-id"                   # rank 0's bytes


def test_relay_plans_exchanged_between_ranks(krlib, tmp_path):
    procs = _run(W.relay_plans, 2, tmp_path)
    assert [p.exitcode for p in procs] == [0, 0]
    p0 = json.loads((tmp_path / "r0.json").read_text())
    p1 = json.loads((tmp_path / "r1.json").read_text())
    assert p0 == p1                                               # both ranks hold both plans
    a, b = p0
    for key in ("R", "Rk", "bn", "bn2", "p1", "total", "tiles", "band_tiles", "nseg"):
        assert a[key] == b[key]                                   # ranks agree on the tiling
    assert a["R"] == 2048 // 4 and a["Rk"] == a["R"] // 2


def test_dead_rank_fails_the_peer_collective(tmp_path):
    """Host-side failure detection: a rank that leaves without joining the barrier makes the
    peer's collective end with an error within the process-group timeout, not hang."""
    procs = _run(W.dead_peer, 2, tmp_path, timeout=90)
    assert procs[1].exitcode == 3
    res = json.loads((tmp_path / "r0.json").read_text())
    assert res["error"], res
    assert res["seconds"] < 60
