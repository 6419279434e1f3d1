"""Full-size BASELINE config 3 ("M26", 40 x 2304, vocab 73448, Q4_K_M mix):
323-token seeded prompt, then 128 greedy tokens, device engine vs CPU oracle.

This is the north-star parity check: identical greedy token ids for 128
steps.  The final top-1/top-2 logit gap is printed so a near tie is visible if
it ever decides a mismatch.
"""
import os
import tempfile

import numpy as np
import pytest

from pocketinfer import synth

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
THREADS = max(1, os.cpu_count() or 1)


def test_m26_323_prompt_then_128_greedy_tokens(pk, oracle):
    path = synth.m26_path(os.environ.get("PK_MODEL_DIR", tempfile.gettempdir()))
    prompt = synth.prompt_ids(323, 323, synth.M26.n_vocab)
    g = pk.Engine(path, n_ctx=512, max_batch=32)
    o = oracle.Engine(path, 512, THREADS)
    rg = g.generate(prompt, 128, stop_at_eog=False)
    ro = o.generate(prompt, 128)
    assert rg["prefill_tokens"] == ro["prefill_tokens"] == 323
    lg, lo = g.logits(), o.logits()
    rel = float(np.max(np.abs(lg - lo)) / np.std(lo))
    top2 = np.sort(lo)[-2:]
    print(f"M26 logits max|diff|/std = {rel:.2e}; final top-2 gap {top2[1] - top2[0]:.4f}")
    mism = [i for i, (a, b) in enumerate(zip(rg["gen_ids"], ro["gen_ids"])) if a != b]
    assert not mism, f"first mismatch at step {mism[0]}"
    assert len(rg["gen_ids"]) == 128
    assert rel < 1e-3
