"""Multi-rank host logic on CPU (gloo, world size 2): replica timing and stream assignment,
plus a rank that fails before joining a collective (host-side fault, no GPU involved)."""
import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from pocketinfer import replicas


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, fail_rank):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected host failure before the timing collective")
        local_ms = 100.0 * (rank + 1)
        value, ms = replicas.replica_throughput(50, local_ms, world, dist)
        q.put((rank, value, ms, replicas.assign_streams(64, rank, world)))
    except Exception as e:  # report, then leave without joining further collectives
        q.put((rank, "error", str(e)[:200], None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(out, key=lambda t: t[0])


def test_replica_throughput_uses_slowest_rank():
    out = _run(2)
    for rank, value, ms, streams in out:
        assert ms == 200.0
        assert value == pytest.approx(2 * 50 / 0.2)
        assert streams == list(range(rank, 64, 2))


def test_failed_rank_surfaces_as_error_on_peer():
    out = _run(2, fail_rank=1)
    assert out[1][1] == "error" and "injected" in out[1][2]
    assert out[0][1] == "error"  # the peer's collective ends with an error instead of hanging


def test_single_process_paths():
    assert replicas.max_over_ranks(3.5) == 3.5
    assert replicas.replica_throughput(10, 500.0, 1) == (20.0, 500.0)
    with pytest.raises(ValueError):
        replicas.replica_throughput(10, 0.0, 1)
    assert replicas.assign_streams(5, 0, 1) == [0, 1, 2, 3, 4]
    with pytest.raises(ValueError):
        replicas.assign_streams(5, 2, 2)
