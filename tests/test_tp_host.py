"""Tensor-parallel host logic on CPU: the shard of each rank, the token pick
over the vocabulary shards (against a restatement of the one-device argmax
over the whole vocabulary), and the peer-handle exchange over gloo with
world size 2 (no GPU involved)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from pocketinfer import PkError, tp


def test_split_m70_covers_every_row_once():
    m = tp.M70
    for world in (1, 2, 4, 8):
        seen = []
        for rank in range(world):
            s = tp.split(m["n_head"], m["n_head_kv"], m["head_dim"], m["n_ff"], m["n_vocab"], rank, world)
            assert s["local_heads"] * world == m["n_head"]
            assert s["local_kv_heads"] * world == m["n_head_kv"]
            assert s["local_ff"] * world == m["n_ff"]
            assert (s["local_heads"] * m["head_dim"]) % 256 == 0 and s["local_ff"] % 256 == 0
            seen.append((s["vocab0"], s["local_vocab"]))
        assert seen[0][0] == 0
        for (a0, an), (b0, _) in zip(seen, seen[1:]):
            assert a0 + an == b0
        assert seen[-1][0] + seen[-1][1] == m["n_vocab"]


@pytest.mark.parametrize("args", [
    (64, 8, 128, 28672, 128256, 0, 16),   # world above 8
    (36, 36, 64, 5760, 73448, 0, 8),      # 36 heads do not split 8 ways
    (36, 36, 64, 5760, 73448, 0, 2),      # down slice 2880 is not a multiple of 256
    (8, 2, 64, 1024, 1, 1, 2),            # vocabulary smaller than the world (rank 1 gets none)
])
def test_split_refuses_models_that_do_not_split(args):
    with pytest.raises(PkError):
        tp.split(*args)


def first_max(x):
    """k_argmax over one array: strict '>', NaN never wins, -inf never wins, 0 if nothing is above -inf."""
    best, bi = -np.inf, None
    for i, v in enumerate(x):
        if v > best:
            best, bi = v, i
    return best, bi


def shard_pick(x, world):
    per = -(-len(x) // world)
    vals, idx = [], []
    for r in range(world):
        lo, hi = min(len(x), r * per), min(len(x), (r + 1) * per)
        v, i = first_max(x[lo:hi])
        vals.append(float(v))
        idx.append(-1 if i is None else lo + i)
    return tp.pick(vals, idx)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_pick_equals_argmax_over_whole_vocabulary(world):
    rng = np.random.default_rng(world)
    cases = [rng.standard_normal(1000).astype(np.float32)]
    ties = np.zeros(1000, np.float32)
    ties[[10, 400, 900]] = 5.0                     # first maximum wins across shards
    cases.append(ties)
    nans = rng.standard_normal(1000).astype(np.float32)
    nans[[0, 3, 700]] = np.nan                     # NaN never wins, index 0 included
    cases.append(nans)
    cases.append(np.full(1000, -np.inf, np.float32))  # nothing above -inf: token 0
    late = np.full(1000, -np.inf, np.float32)
    late[999] = -1e30
    cases.append(late)
    for x in cases:
        _, want = first_max(x)
        assert shard_pick(x, world) == (0 if want is None else want)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        got = tp.allgather_bytes(bytes([rank]) * 64)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_handle_exchange_is_rank_ordered_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=120) for _ in range(2)])
    for p in procs:
        p.join(timeout=60)
    for _, got in out:
        assert got == [bytes([0]) * 64, bytes([1]) * 64]


class _FakeLib:
    """The C entry points TpEngine.connect calls, with pk_tp_nccl_id failing."""

    def __init__(self):
        self.used_nccl = False

    def pk_tp_handle_bytes(self):
        return 4

    def pk_tp_ipc_handle(self, h, out):
        return 0

    def pk_tp_open_peers(self, h, handles):
        return 0

    def pk_tp_nccl_id_bytes(self):
        return 8

    def pk_tp_nccl_id(self, out):
        return 2  # PK_ERR_UNSUPPORTED: no NCCL here

    def pk_tp_use_nccl(self, h, ident):
        self.used_nccl = True
        return 0

    def pk_last_error(self):
        return b"NCCL is not available"


@pytest.mark.parametrize("rank", [0, 1])
def test_nccl_connect_failure_reaches_every_rank(monkeypatch, rank):
    """When rank 0 cannot make an NCCL id it still takes part in the id
    exchange (an empty id), so every rank raises instead of the others
    waiting in the exchange until the process group times out; no rank
    joins a communicator."""
    import pocketinfer

    fake = _FakeLib()
    monkeypatch.setattr(tp, "lib", lambda: fake)
    monkeypatch.setattr(pocketinfer, "lib", lambda: fake)
    eng = tp.TpEngine.__new__(tp.TpEngine)
    eng.rank, eng.world, eng.h, eng.connected = rank, 2, None, False
    sent = []

    def exchange(blob):  # rank 0's blob first, as an all-gather in rank order
        sent.append(blob)
        if len(blob) == 4:  # the peer handles
            return [b"\0" * 4, b"\0" * 4]
        return [blob if rank == 0 else b"", b""]

    with pytest.raises(PkError, match="rank 0 could not make an NCCL id"):
        eng.connect(exchange=exchange, collective="nccl")
    assert len(sent) == 2 and not fake.used_nccl
    eng.h = None
