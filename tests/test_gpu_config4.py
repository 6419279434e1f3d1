"""BASELINE config 4 against the CPU oracle: long prefill in 32-token chunks
and the prefix-reuse extension (model.rs:1251-1295; the reference checks
the extension with its `prefixcheck` mode, pocketinfer-cli.rs:24-46, at a
max logit difference below 1e-3).

* M26 itself: a fresh 323-token prompt, then a 379-token prompt that extends
  it.  Engine::generate reuses the full 32-token chunks of the common prefix,
  min(323, 323, 378) // 32 * 32 = 320 tokens, and prefills the other 59.
  Reuse counts, the greedy token and the final logits equal the oracle's bit
  for bit.
* The 4096-token prefill (128 chunks of 32) on an M26-shaped stack with the
  full layer shapes and fewer layers: the final-token logits equal the
  oracle's bit for bit.  The oracle's attention over 4096 positions at all
  40 layers takes minutes on the host; PK_CONFIG4_LAYERS=40 runs that case.
"""
import os
import tempfile

import numpy as np
import pytest

from pocketinfer import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
THREADS = max(1, os.cpu_count() or 1)
MODEL_DIR = os.environ.get("PK_MODEL_DIR", tempfile.gettempdir())


def test_m26_323_then_379_reuses_320_and_matches_oracle(pk, oracle):
    path = synth.m26_path(MODEL_DIR)
    V = synth.M26.n_vocab
    first = synth.prompt_ids(323, 323, V).tolist()
    ext = first + synth.prompt_ids(379, 56, V).tolist()
    assert len(ext) == 379
    g = pk.Engine(path, n_ctx=512, max_batch=32)
    o = oracle.Engine(path, 512, THREADS)
    for p, reused in ((first, 0), (ext, 320)):
        rg, ro = g.generate(p, 1, stop_at_eog=False), o.generate(p, 1)
        assert rg["prefill_cached_tokens"] == ro["prefill_cached_tokens"] == reused
        assert rg["prefill_tokens"] == ro["prefill_tokens"] == len(p) - reused
        assert rg["gen_ids"] == ro["gen_ids"]
        lg, lo = g.logits(), o.logits()
        assert np.array_equal(lg.view(np.uint32), lo.view(np.uint32)), float(np.max(np.abs(lg - lo)))


def test_4096_token_prefill_matches_oracle(pk, oracle):
    layers = int(os.environ.get("PK_CONFIG4_LAYERS", "3"))
    spec = synth.m26_spec(None if layers == 40 else layers, None if layers == 40 else 8192)
    path = synth.m26_path(MODEL_DIR, spec=spec)
    prompt = synth.prompt_ids(4096, 4096, spec.n_vocab).tolist()
    g = pk.Engine(path, n_ctx=4096 + 64, max_batch=32)
    o = oracle.Engine(path, 4096 + 64, THREADS)
    rg, ro = g.generate(prompt, 1, stop_at_eog=False), o.generate(prompt, 1)
    assert rg["prefill_tokens"] == ro["prefill_tokens"] == 4096
    assert rg["gen_ids"] == ro["gen_ids"]
    lg, lo = g.logits(), o.logits()
    assert np.array_equal(lg.view(np.uint32), lo.view(np.uint32)), float(np.max(np.abs(lg - lo)))
