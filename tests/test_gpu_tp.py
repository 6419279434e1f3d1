"""Tensor-parallel decode on the GPU.

* T = 1 is the single-GPU b = 1 op sequence bit for bit (prefill logits and
  greedy tokens against pk.Engine stepping the same prompt one token at a
  time).
* T = 2 (two GPUs, one process each, handles exchanged over gloo): the
  vocabulary shards' logits within 1e-3 of T = 1 (the partial row sums of o
  and down are added across ranks, a different rounding order) and the same
  greedy tokens.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from pocketinfer import synth, tp

pytestmark = pytest.mark.gpu

MODELS = {"tiny": synth.TINY, "q40": synth.SMALL_Q40}


@pytest.fixture(scope="module")
def paths(tmp_path_factory):
    d = tmp_path_factory.mktemp("tpmodels")
    out = {}
    for name, spec in MODELS.items():
        out[name] = str(d / f"{name}.gguf")
        synth.write_gguf(out[name], spec, seed=33)
    return out


@pytest.mark.parametrize("name", list(MODELS))
def test_tp1_equals_single_gpu_b1(pk, paths, name):
    spec = MODELS[name]
    prompt = synth.prompt_ids(41, 20, spec.n_vocab)
    e = pk.Engine(paths[name], n_ctx=256)
    for i in range(len(prompt)):
        e.forward(prompt[i:i + 1], [i], i == len(prompt) - 1)
    want_logits = e.logits()
    want = e.decode_steps_device(16)
    t = tp.TpEngine(0, 1, device=0, n_ctx=256)
    t.load(paths[name])
    info = t.info
    assert info["local_heads"] == spec.n_head and info["collectives_per_token"] == 2 * spec.n_layer + 1
    t.prefill(prompt)
    lg, v0 = t.logits()
    assert v0 == 0 and np.array_equal(lg.view(np.uint32), want_logits.view(np.uint32))
    assert t.decode(16) == want
    assert t.decode(5) == e.decode_steps_device(5)  # a second call continues from the last token


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp2_worker(rank, world, port, path, prompt, n, q, collective="peer"):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        t = tp.TpEngine(rank, world, device=rank, n_ctx=256)
        t.load(path)
        t.connect(collective=collective)
        t.prefill(prompt)
        lg, v0 = t.logits()
        ids = t.decode(n)
        q.put((rank, ids, v0, lg))
        t.close()
    except Exception as e:
        q.put((rank, "error", str(e)[:300], None))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("collective", ["peer", "nccl"])
def test_tp2_matches_tp1(pk, paths, collective):
    """T = 2 (two GPUs, two processes) against T = 1: logits within 1e-3 of
    their spread and the same greedy tokens, with the o / down exchange on
    the peer-memory push or on an NCCL all-reduce."""
    spec = MODELS["q40"]
    prompt = synth.prompt_ids(43, 24, spec.n_vocab)
    n = 24
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp2_worker, args=(r, 2, port, paths["q40"], prompt, n, q, collective))
             for r in range(2)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in range(2)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    for r in out:
        assert r[1] != "error", r[2]
    t = tp.TpEngine(0, 1, device=0, n_ctx=256)
    t.load(paths["q40"])
    t.prefill(prompt)
    ref, _ = t.logits()
    ref_ids = t.decode(n)
    lg = np.concatenate([out[0][3], out[1][3]])
    assert out[0][2] == 0 and out[1][2] == len(out[0][3])
    assert float(np.max(np.abs(lg - ref))) <= 1e-3 * float(np.std(ref))
    assert out[0][1] == out[1][1] == ref_ids
