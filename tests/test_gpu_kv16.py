"""The f16 K/V cache option (pk_set_kv_type(PK_KV_F16)) against the CPU
oracle with the same option (pko_engine_set_kv_f16): every K and V value is
rounded to f16 (nearest even) when stored and converted back exactly when
read, and all other arithmetic is the reference's, so logits and greedy
tokens are the oracle's bits.  The reference itself keeps an f32 cache
(model.rs:352-387); this is a B200 option, checked against the reference's
arithmetic over f16-rounded cache entries."""
import os

import numpy as np
import pytest

from pocketinfer import synth

pytestmark = pytest.mark.gpu
THREADS = max(1, min(32, os.cpu_count() or 1))
MODELS = {"tiny": synth.TINY, "q8down": synth.SMALL_Q8DOWN, "q40": synth.SMALL_Q40}
# head_dim 128: the split value pass runs two 64-dim parts per head
DH128 = synth.ModelSpec("tiny-dh128", n_layer=2, n_embd=256, n_head=2, n_head_kv=1, head_dim=128, n_ff=512,
                        n_vocab=1000)


@pytest.fixture(scope="module")
def paths(tmp_path_factory):
    d = tmp_path_factory.mktemp("kv16")
    out = {}
    for name, spec in list(MODELS.items()) + [("dh128", DH128)]:
        out[name] = str(d / f"{name}.gguf")
        synth.write_gguf(out[name], spec, seed=33)
    return out


def oracle_f16(oracle, path, n_ctx=256):
    o = oracle.Engine(path, n_ctx, THREADS)
    o.set_kv_f16(True)
    return o


@pytest.mark.parametrize("name", list(MODELS))
def test_kv16_prefill_and_decode_match_oracle(pk, oracle, paths, name):
    """A 77-token prompt (three chunks), then greedy tokens: the same logits
    and token ids as the oracle's f16-cache engine, bit for bit."""
    spec = MODELS[name]
    prompt = synth.prompt_ids(19, 77, spec.n_vocab)
    g = pk.Engine(paths[name], n_ctx=256, kv="f16")
    o = oracle_f16(oracle, paths[name])
    rg = g.generate(prompt, 40, stop_at_eog=False)
    ro = o.generate(prompt, 40)
    assert rg["gen_ids"] == ro["gen_ids"]
    assert np.array_equal(g.logits().view(np.uint32), o.logits().view(np.uint32))
    # the f16 cache is half the f32 one
    f32 = pk.Engine(paths[name], n_ctx=256)
    assert g.model_info()["kv_bytes"] * 2 == f32.model_info()["kv_bytes"]


@pytest.mark.parametrize("name", ["tiny", "q8down"])
def test_kv16_streams_match_oracle(pk, oracle, paths, name):
    """Independent streams over f16 caches, decoded in one batched step per
    token: each stream's tokens are the oracle's f16-cache tokens for it."""
    spec = MODELS[name]
    prompts = [synth.prompt_ids(51 + i, n, spec.n_vocab) for i, n in enumerate((1, 20, 45))]
    want = [oracle_f16(oracle, paths[name]).generate(p, 24)["gen_ids"] for p in prompts]
    e = pk.Engine(paths[name], n_ctx=256, kv="f16")
    e.streams_begin(len(prompts))
    for s, p in enumerate(prompts):
        e.stream_prefill(s, p)
    got = e.streams_decode(24)
    for s in range(len(prompts)):
        assert got[s] == want[s]


def test_kv16_set_after_load_is_rejected(pk, paths):
    """The caches are sized at load, so the entry type can only change before it."""
    g = pk.Engine(paths["tiny"], n_ctx=128)
    assert pk.lib().pk_set_kv_type(g.h, pk.KV_F16) != 0
    assert pk.lib().pk_set_kv_type(None, pk.KV_F16) != 0


@pytest.mark.parametrize("name", ["tiny", "q8down"])
def test_kv16_chunk_attention_equals_per_token_kernel(pk, paths, name):
    """f16 entries through the shared-memory tile kernels (n_ctx = 256, whole
    16-byte pieces of eight entries) give the same bits as the one-CTA-per-
    token kernel (n_ctx = 252 is not a multiple of eight, so it takes that
    path), across prefill chunks and the decode step."""
    spec = MODELS[name]
    prompt = synth.prompt_ids(13, 200, spec.n_vocab)
    a, b = pk.Engine(paths[name], n_ctx=256, kv="f16"), pk.Engine(paths[name], n_ctx=252, kv="f16")
    ra, rb = a.generate(prompt, 24, stop_at_eog=False), b.generate(prompt, 24, stop_at_eog=False)
    assert ra["gen_ids"] == rb["gen_ids"]
    assert np.array_equal(a.logits().view(np.uint32), b.logits().view(np.uint32))


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("name", ["tiny", "dh128"])
def test_streams_long_history_match_oracle(pk, oracle, paths, kv, name):
    """Above 1024 positions the streams' attention is split (scores over
    512-position chunks on many CTAs, then the value chains of 64 dims per
    CTA over 64-position tiles); each stream's greedy tokens equal the
    oracle's for that prompt alone, with an f32 or an f16 cache, across chunk
    and tile edges, at head_dim 64 and 128."""
    spec = DH128 if name == "dh128" else MODELS[name]
    prompts = [synth.prompt_ids(41 + i, n, spec.n_vocab) for i, n in enumerate((3, 530, 1100))]
    want = []
    for p in prompts:
        o = oracle.Engine(paths[name], 1536, THREADS)
        o.set_kv_f16(kv == "f16")
        want.append(o.generate(p, 24)["gen_ids"])
    e = pk.Engine(paths[name], n_ctx=1536, kv=kv)
    e.streams_begin(len(prompts))
    for s, p in enumerate(prompts):
        e.stream_prefill(s, p)
    first, rest = e.streams_decode(9), e.streams_decode(15)
    for s in range(len(prompts)):
        assert first[s] + rest[s] == want[s]
