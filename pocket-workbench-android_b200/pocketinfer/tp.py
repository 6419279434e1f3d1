"""Tensor-parallel decode over T GPUs, one process per GPU (include/pk.h pk_tp_*).

Each rank holds a shard of every matrix: q/k/v rows of whole heads, o and
down k ranges, gate/up rows, output vocabulary rows.  After o and after down
the ranks' partial row sums go through peer memory (the ranks exchange
cudaIpc handles once, through ``torch.distributed``) and are added in rank
order, so every rank keeps the same residual.  Every rank makes the same
calls in the same order.
"""
from __future__ import annotations

import ctypes as C

from . import PkError, TpInfo, TpModel, _check, lib

# the 70B-shaped stack (80 layers, d 8192, 64 / 8 heads x 128, FFN 28672, vocab 128256).
M70 = dict(n_layer=80, n_embd=8192, n_head=64, n_head_kv=8, head_dim=128, n_ff=28672, n_vocab=128256, n_rot=128,
           rope_theta=10000.0, rms_eps=1e-5)


def split(n_head: int, n_head_kv: int, head_dim: int, n_ff: int, n_vocab: int, rank: int, world: int,
          o_block: int = 256, down_block: int = 256) -> dict:
    """The shard of rank ``rank`` of ``world`` (raises PkError when the model does not split)."""
    out = (C.c_int * 5)()
    _check(lib().pk_tp_split(n_head, n_head_kv, head_dim, n_ff, n_vocab, rank, world, o_block, down_block,
                             C.cast(out, C.c_void_p)))
    return dict(zip(("local_heads", "local_kv_heads", "local_ff", "vocab0", "local_vocab"), list(out)))


def pick(vals, idx) -> int:
    """The token from the shards' {first-maximum value, global index or -1}, in rank order."""
    n = len(vals)
    v = (C.c_float * n)(*[float(x) for x in vals])
    i = (C.c_int * n)(*[int(x) for x in idx])
    return int(lib().pk_tp_pick(C.cast(v, C.c_void_p), C.cast(i, C.c_void_p), n))


def allgather_bytes(blob: bytes, group=None) -> list:
    """Every rank's ``blob`` in rank order, through torch.distributed."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, blob, group=group)
    return out


class TpEngine:
    """One rank of a tensor-parallel engine on CUDA device ``device``."""

    def __init__(self, rank: int, world: int, device: int | None = None, n_ctx: int = 512):
        self.rank, self.world = rank, world
        self.h = C.c_void_p()
        _check(lib().pk_tp_create(rank if device is None else device, n_ctx, rank, world, C.byref(self.h)))
        self.connected = False

    def close(self):
        if self.h:
            lib().pk_tp_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, path: str):
        _check(lib().pk_tp_load_gguf(self.h, path.encode()))

    def load_synthetic(self, model: dict, seed: int = 0):
        m = TpModel(**model)
        _check(lib().pk_tp_load_synthetic(self.h, C.byref(m), seed))

    def handle(self) -> bytes:
        n = lib().pk_tp_handle_bytes()
        buf = (C.c_uint8 * n)()
        _check(lib().pk_tp_ipc_handle(self.h, C.cast(buf, C.c_void_p)))
        return bytes(buf)

    def connect(self, exchange=allgather_bytes, collective: str = "peer"):
        """Exchange peer-memory handles (``exchange(bytes) -> [bytes] * world`` in rank order) and open them.

        ``collective="nccl"`` then moves the o / down exchange onto an NCCL
        all-reduce: rank 0's NCCL id goes to every rank through ``exchange``
        and every rank joins the communicator (pk_tp_use_nccl)."""
        if collective not in ("peer", "nccl"):
            raise PkError(1, "collective must be 'peer' or 'nccl'")
        mine = self.handle()
        allh = exchange(mine)
        if len(allh) != self.world or allh[self.rank] != mine:
            raise PkError(1, "handle exchange returned the wrong number or order of handles")
        blob = b"".join(allh)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(lib().pk_tp_open_peers(self.h, C.cast(buf, C.c_void_p)))
        self.connected = True
        if collective == "nccl":
            # rank 0 always takes part in the id exchange (an empty id when it
            # could not make one), so every rank fails together, not only rank 0
            n = lib().pk_tp_nccl_id_bytes()
            mine_id, why = b"", ""
            if self.rank == 0:
                idb = (C.c_uint8 * n)()
                try:
                    _check(lib().pk_tp_nccl_id(C.cast(idb, C.c_void_p)))
                    mine_id = bytes(idb)
                except PkError as e:
                    why = str(e)
            ids = exchange(mine_id)
            if len(ids[0]) != n:
                raise PkError(2, "rank 0 could not make an NCCL id" + (f": {why}" if why else ""))
            root = (C.c_uint8 * n).from_buffer_copy(ids[0])
            _check(lib().pk_tp_use_nccl(self.h, C.cast(root, C.c_void_p)))
        self.collective = collective

    def prefill(self, prompt):
        import numpy as np

        p = np.ascontiguousarray(prompt, np.uint32)
        _check(lib().pk_tp_prefill(self.h, p.ctypes.data_as(C.c_void_p), len(p)))

    def decode(self, n_steps: int, return_ms: bool = False):
        import numpy as np

        out = np.zeros(max(n_steps, 1), np.uint32)
        ms = C.c_float()
        _check(lib().pk_tp_decode(self.h, n_steps, out.ctypes.data_as(C.c_void_p), C.byref(ms)))
        ids = out[:n_steps].tolist()
        return (ids, ms.value) if return_ms else ids

    def logits(self):
        """This rank's logits of the last step with the head, and the first vocabulary row they cover."""
        import numpy as np

        info = self.info
        out = np.zeros(info["local_vocab"], np.float32)
        n, v0 = C.c_int(), C.c_int()
        _check(lib().pk_tp_logits(self.h, out.ctypes.data_as(C.c_void_p), len(out), C.byref(n), C.byref(v0)))
        return out, v0.value

    @property
    def info(self) -> dict:
        i = TpInfo()
        _check(lib().pk_tp_info_get(self.h, C.byref(i)))
        return {f: getattr(i, f) for f, _ in TpInfo._fields_}
