"""Worker functions for the gloo multi-process tests (spawned children import this module)."""
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _setup(rank, world, port):
    if str(REPO) not in sys.path:
        sys.path.insert(0, str(REPO))
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import bench
    return bench


def helpers(rank, world, port, out_dir):
    """bench.Dist over gloo: max over ranks, byte gather / broadcast, barrier."""
    bench = _setup(rank, world, port)
    d = bench.Dist()
    d.init("gloo", timeout_s=60)
    res = {"max": d.max(float(rank) + 0.5),
           "gather": [b.decode() for b in d.gather_bytes(f"handle-{rank}".encode())],
           "bcast": d.bcast_bytes(b"nccl-unique-id" if rank == 0 else None).decode()}
    d.barrier()
    d.close()
    Path(out_dir, f"r{rank}.json").write_text(json.dumps(res))


def relay_plans(rank, world, port, out_dir):
    """Every rank builds its relay plan through the C ABI and the ranks exchange them."""
    bench = _setup(rank, world, port)
    from kernrelay_b200 import _lib
    d = bench.Dist()
    d.init("gloo", timeout_s=60)
    mine = _lib.relay_plan(2048, 3584, 4, world, rank, 224)
    plans = [json.loads(b) for b in d.gather_bytes(json.dumps(mine).encode())]
    d.close()
    Path(out_dir, f"r{rank}.json").write_text(json.dumps(plans))


def dead_peer(rank, world, port, out_dir):
    """Rank 1 dies before the barrier; rank 0's barrier must end with an error."""
    bench = _setup(rank, world, port)
    d = bench.Dist()
    d.init("gloo", timeout_s=5)
    if rank == 1:
        os._exit(3)  # leaves without joining any collective
    import time
    t0 = time.time()
    try:
        d.barrier()
        res = {"error": None}
    except Exception as e:  # noqa: BLE001 - any failure of the collective is the signal
        res = {"error": type(e).__name__ + ": " + str(e)[:200]}
    res["seconds"] = time.time() - t0
    Path(out_dir, f"r{rank}.json").write_text(json.dumps(res))
    os._exit(0)
