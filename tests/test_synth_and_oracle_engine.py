"""Synthetic GGUF models and the oracle's Engine::generate semantics.

The prefix-reuse checks restate rust/pocketinfer/tests/prefix_cache.rs:5-89
(of the reference) on seeded token ids instead of tokenizer text.
"""
import numpy as np
import pytest

from pocketinfer import synth


@pytest.fixture(scope="module")
def tiny_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / "tiny.gguf")
    synth.write_gguf(p, synth.TINY, seed=3)
    return p


@pytest.fixture(scope="module")
def q8down_path(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("m") / "q8down.gguf")
    synth.write_gguf(p, synth.SMALL_Q8DOWN, seed=4)
    return p


def test_splitmix_matches_reference_rng(oracle):
    r = oracle.Rng(0xC0FFEE)
    assert [r.next_u64() for _ in range(6)] == synth.splitmix_u64(0xC0FFEE, 0, 6).tolist()
    r = oracle.Rng(5)
    got = np.array([r.next_f32() for _ in range(8)], np.float32)
    assert np.array_equal(got, synth.splitmix_f32(5, 0, 8))


def test_m26_tensor_mix_and_bytes():
    specs = {n: s for n, s, k, r in synth.M26.tensor_specs()}
    assert specs["blk.0.attn_q.weight"].ttype == synth.Q4_K
    assert specs["blk.0.attn_v.weight"].ttype == synth.Q6_K
    assert specs["output.weight"].ttype == synth.Q6_K
    # 5760 is not a multiple of 256, so ffn_down falls back to Q8_0
    assert specs["blk.0.ffn_down.weight"].ttype == synth.Q8_0
    assert synth.M26.streamed_bytes_per_token() == 1_833_280_992
    assert synth.M26.kv_bytes_per_position() == 737_280


@pytest.mark.parametrize("spec", [synth.SPEC_Q4K, synth.SPEC_Q6K, synth.SPEC_Q8_0, synth.SPEC_Q4_0])
def test_synthetic_blocks_have_target_std(oracle, spec):
    k = 2304 if spec.ttype != synth.Q8_0 else 5760
    w = synth.quant_blocks(spec, 77, 32, k)
    rb = oracle.row_bytes(spec.ttype, k)
    vals = np.concatenate([oracle.dequant_row(spec.ttype, w[i * rb:(i + 1) * rb], k) for i in range(32)])
    assert abs(float(vals.std()) - 0.02) < 0.003
    assert abs(float(vals.mean())) < 0.004


def test_q6k_scale_is_f16_subnormal():
    w = synth.quant_blocks(synth.SPEC_Q6K, 1, 4, 256).reshape(4, 210)
    d = w[:, 208:210].copy().view(np.float16).astype(np.float32)
    assert np.all(d < 6.1e-5) and np.all(d > 0)


def test_oracle_loads_synthetic_models(oracle, tiny_path, q8down_path):
    assert oracle.Engine(tiny_path, 128, 2).vocab == synth.TINY.n_vocab
    assert oracle.Engine(q8down_path, 128, 2).vocab == synth.SMALL_Q8DOWN.n_vocab


def test_oracle_rejects_bad_files(oracle, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOTGGUF" + b"\0" * 64)
    with pytest.raises(RuntimeError, match="not a GGUF"):
        oracle.Engine(str(p), 64, 1)
    good = tmp_path / "t.gguf"
    synth.write_gguf(str(good), synth.TINY, seed=1)
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(good.read_bytes()[:200])
    with pytest.raises(RuntimeError):
        oracle.Engine(str(trunc), 64, 1)


def test_batched_prefill_equals_token_by_token_logits(oracle, tiny_path):
    """lanes::* is bit-identical per lane, so b=32 and b=1 agree to float noise."""
    ids = synth.prompt_ids(11, 32, synth.TINY.n_vocab)
    a = oracle.Engine(tiny_path, 128, 2)
    a.forward(ids, np.arange(32), True)
    b = oracle.Engine(tiny_path, 128, 2)
    for i in range(32):
        b.forward(ids[i:i + 1], [i], i == 31)
    assert np.max(np.abs(a.logits() - b.logits())) < 1e-4


def test_prefix_reuse_matches_fresh(oracle, tiny_path):
    """prefix_cache.rs:17-63 on seeded ids."""
    V = synth.TINY.n_vocab
    base = synth.prompt_ids(1, 12 * 8, V).tolist()
    extended = base + synth.prompt_ids(2, 9, V).tolist()
    divergent = synth.prompt_ids(3, 7, V).tolist()
    eng = oracle.Engine(tiny_path, 512, 2)
    eng.generate(base, 2)
    cached = eng.generate(extended, 2)
    assert cached["prefill_cached_tokens"] > 0
    assert cached["prefill_cached_tokens"] + cached["prefill_tokens"] == len(extended)
    uncached = oracle.Engine(tiny_path, 512, 2).generate(extended, 2)
    assert cached["gen_ids"] == uncached["gen_ids"]
    rep = eng.generate(extended, 2, temp=0.7, top_p=0.95, seed=1)
    rep_fresh = oracle.Engine(tiny_path, 512, 2).generate(extended, 2, temp=0.7, top_p=0.95, seed=1)
    assert rep["prefill_cached_tokens"] == (len(extended) - 1) // 32 * 32
    assert rep["gen_ids"] == rep_fresh["gen_ids"]
    changed = eng.generate(divergent, 2)
    assert changed["gen_ids"] == oracle.Engine(tiny_path, 512, 2).generate(divergent, 2)["gen_ids"]
    eng.forward([divergent[0]], [0], False)  # a public forward invalidates the cache
    after = eng.generate(extended, 2)
    assert after["prefill_cached_tokens"] == 0
    assert after["gen_ids"] == uncached["gen_ids"]
    oracle.request_stop()
    try:
        stopped = eng.generate(extended, 2)
    finally:
        oracle.clear_stop()
    assert stopped["stop"] == "user_stop"
    again = eng.generate(extended, 2)
    assert again["prefill_cached_tokens"] == 0
    assert again["gen_ids"] == uncached["gen_ids"]


def test_generate_edge_cases(oracle, tiny_path):
    eng = oracle.Engine(tiny_path, 40, 1)
    with pytest.raises(RuntimeError, match="empty prompt"):
        eng.generate([], 2)
    r = eng.generate(synth.prompt_ids(5, 38, synth.TINY.n_vocab), 8)
    assert r["stop"] == "context_full" and r["gen_tokens"] == 3
    with pytest.raises(RuntimeError, match="out of vocab"):
        eng.forward([synth.TINY.n_vocab], [0])
    with pytest.raises(RuntimeError, match="context full"):
        eng.forward([1], [40])


def test_eog_stops_generation(oracle, tmp_path):
    spec = synth.ModelSpec(**{**synth.TINY.__dict__, "name": "tiny-eos"})
    p = str(tmp_path / "eos.gguf")
    prompt = synth.prompt_ids(9, 20, spec.n_vocab)
    synth.write_gguf(p, spec, seed=3)
    first = oracle.Engine(p, 128, 1).generate(prompt, 4)["gen_ids"]
    spec.eos_token_id = first[2]
    synth.write_gguf(p, spec, seed=3)
    e = oracle.Engine(p, 128, 1)
    r = e.generate(prompt, 8)
    assert r["stop"] == "eog" and r["gen_ids"] == first[:2]
    e.set_eog(False)
    assert e.generate(prompt, 4)["gen_ids"] == first
