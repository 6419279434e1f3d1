"""Seeded synthetic GGUF models and inputs for pocketinfer's decode path.

There is no network and no MiniCPM5 checkpoint on this machine, so the
benchmarks and parity tests use random-block models of the shapes the
reference is measured on.  Everything is derived from splitmix64 (the
reference's ``Rng``, rust/pocketinfer/src/sampler.rs:1-19), evaluated as a
counter-based stream so gigabytes of blocks can be produced with numpy.

Block layouts follow rust/pocketinfer/src/quant.rs:19-37 / 102-359:
  Q4_K 144 B = f16 d | f16 dmin | 12 B scales | 128 B qs
  Q6_K 210 B = 128 B ql | 64 B qh | 16 B i8 scales | f16 d
  Q8_0  34 B = f16 d | 32 B i8
  Q4_0  18 B = f16 d | 16 B nibbles
The GGUF container follows rust/pocketinfer/src/gguf.rs:113-192 (v3, 32-byte
alignment), the same format rust/pocketinfer/tools/make_tiny_model.py writes.
"""
from __future__ import annotations

import dataclasses
import struct
import zlib

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
C1 = np.uint64(0xBF58476D1CE4E5B9)
C2 = np.uint64(0x94D049BB133111EB)

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
TYPE_NAME = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def splitmix_u64(seed: int, start: int, n: int) -> np.ndarray:
    """Outputs start..start+n-1 of ``Rng::new(seed).next_u64()``.

    Rng::new sets s = seed + G and every call first adds G, so output i mixes
    seed + (i + 2) * G.
    """
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (np.arange(start + 2, start + 2 + n, dtype=np.uint64) * GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * C1
        z = (z ^ (z >> np.uint64(27))) * C2
        return z ^ (z >> np.uint64(31))


def splitmix_f32(seed: int, start: int, n: int) -> np.ndarray:
    """``Rng::next_f32``: (u64 >> 40) / 2^24, in [0, 1)."""
    return ((splitmix_u64(seed, start, n) >> np.uint64(40)).astype(np.float32) / np.float32(1 << 24))


def random_bytes(seed: int, n: int) -> np.ndarray:
    return splitmix_u64(seed, 0, (n + 7) // 8).view(np.uint8)[:n].copy()


def normal_f32(seed: int, n: int) -> np.ndarray:
    """N(0,1) by Box-Muller on consecutive next_f32 pairs (u1, u2)."""
    u = splitmix_f32(seed, 0, 2 * n).astype(np.float64)
    u1, u2 = u[0::2], u[1::2]
    return (np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)).astype(np.float32)


def uniform_f32(seed: int, n: int, lo: float, hi: float) -> np.ndarray:
    return (lo + (hi - lo) * splitmix_f32(seed, 0, n).astype(np.float64)).astype(np.float32)


def f16_bytes(v: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(v.astype(np.float16)).view(np.uint8).reshape(-1, 2)


def tensor_seed(base: int, name: str) -> int:
    return ((base & 0xFFFFFFFF) << 32) ^ zlib.crc32(name.encode())


@dataclasses.dataclass
class QuantSpec:
    """How to draw one tensor's blocks.

    ``d`` is the nominal f16 super-block scale; each block's scale is drawn
    uniformly in d * [1 - jitter, 1 + jitter].  For Q4_K, dmin = dmin_ratio * d.
    """
    ttype: int
    d: float = 0.0
    jitter: float = 0.25
    dmin_ratio: float = 7.5
    d_range: tuple | None = None      # (lo, hi): uniform draw, overrides d/jitter
    dmin_range: tuple | None = None


def quant_blocks(spec: QuantSpec, seed: int, rows: int, k: int) -> np.ndarray:
    """Raw GGUF bytes for a rows x k tensor (row-major rows of blocks)."""
    t = spec.ttype
    be, bb = BLOCK[t]
    assert k % be == 0, (k, be)
    nblk = rows * (k // be)
    raw = random_bytes(seed, nblk * bb).reshape(nblk, bb)

    def scales(sub_seed, rng=None, base=None):
        if rng is not None:
            return uniform_f32(seed ^ sub_seed, nblk, rng[0], rng[1])
        j = uniform_f32(seed ^ sub_seed, nblk, 1.0 - spec.jitter, 1.0 + spec.jitter)
        return (np.float32(base) * j).astype(np.float32)

    if t == Q4_K:
        d = scales(0x51, spec.d_range, spec.d)
        if spec.dmin_range is not None:
            dmin = uniform_f32(seed ^ 0x52, nblk, *spec.dmin_range)
        else:
            dmin = (d * np.float32(spec.dmin_ratio)).astype(np.float32)
        raw[:, 0:2] = f16_bytes(d)
        raw[:, 2:4] = f16_bytes(dmin)
    elif t == Q6_K:
        raw[:, 208:210] = f16_bytes(scales(0x61, spec.d_range, spec.d))
    elif t in (Q8_0, Q4_0):
        raw[:, 0:2] = f16_bytes(scales(0x81, spec.d_range, spec.d))
    else:
        raise ValueError(f"unsupported synthetic type {t}")
    return raw.reshape(-1)


# Scales from the measurement plan: dequantised weights with std ~0.02.
SPEC_Q4K = QuantSpec(Q4_K, d=7.75e-5, dmin_ratio=7.5)
SPEC_Q6K = QuantSpec(Q6_K, d=1.5e-5)           # full-range i8 scales: an f16 subnormal d
SPEC_Q8_0 = QuantSpec(Q8_0, d=0.02 / 73.9)
SPEC_Q4_0 = QuantSpec(Q4_0, d=0.02 / 4.61)
SPEC_CONFIG1 = QuantSpec(Q4_K, d_range=(1e-3, 4e-3), dmin_range=(1e-3, 4e-3))


@dataclasses.dataclass
class ModelSpec:
    name: str
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_ff: int
    n_vocab: int
    n_rot: int | None = None
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    n_ctx_train: int = 4096
    # tensor role -> QuantSpec; a role whose k is not block-divisible falls back to Q8_0
    mix: dict | None = None
    eos_token_id: int | None = None

    def tensor_specs(self):
        mix = {"attn_q": SPEC_Q4K, "attn_k": SPEC_Q4K, "attn_v": SPEC_Q6K, "attn_output": SPEC_Q4K,
               "ffn_gate": SPEC_Q4K, "ffn_up": SPEC_Q4K, "ffn_down": SPEC_Q6K,
               "output": SPEC_Q6K, "token_embd": SPEC_Q4K}
        if self.mix:
            mix.update(self.mix)
        qdim, kdim = self.n_head * self.head_dim, self.n_head_kv * self.head_dim

        def fit(spec, k):
            be = BLOCK[spec.ttype][0]
            if k % be == 0:
                return spec
            return SPEC_Q8_0 if k % 32 == 0 else None

        out = [("token_embd.weight", fit(mix["token_embd"], self.n_embd), self.n_embd, self.n_vocab),
               ("output.weight", fit(mix["output"], self.n_embd), self.n_embd, self.n_vocab),
               ("output_norm.weight", "norm", self.n_embd, 1)]
        for i in range(self.n_layer):
            p = f"blk.{i}."
            out += [(p + "attn_norm.weight", "norm", self.n_embd, 1),
                    (p + "ffn_norm.weight", "norm", self.n_embd, 1),
                    (p + "attn_q.weight", fit(mix["attn_q"], self.n_embd), self.n_embd, qdim),
                    (p + "attn_k.weight", fit(mix["attn_k"], self.n_embd), self.n_embd, kdim),
                    (p + "attn_v.weight", fit(mix["attn_v"], self.n_embd), self.n_embd, kdim),
                    (p + "attn_output.weight", fit(mix["attn_output"], qdim), qdim, self.n_embd),
                    (p + "ffn_gate.weight", fit(mix["ffn_gate"], self.n_embd), self.n_embd, self.n_ff),
                    (p + "ffn_up.weight", fit(mix["ffn_up"], self.n_embd), self.n_embd, self.n_ff),
                    (p + "ffn_down.weight", fit(mix["ffn_down"], self.n_ff), self.n_ff, self.n_embd)]
        return out

    def streamed_bytes_per_token(self) -> int:
        """Weight + norm bytes one decode token reads, including its one embedding row."""
        total = 0
        for name, spec, k, rows in self.tensor_specs():
            if name == "token_embd.weight":
                be, bb = BLOCK[spec.ttype]
                total += (k // be) * bb
                continue
            if spec == "norm":
                total += k * 4
            else:
                be, bb = BLOCK[spec.ttype]
                total += rows * (k // be) * bb
        return total

    def kv_bytes_per_position(self) -> int:
        return 2 * self.n_layer * self.n_head_kv * self.head_dim * 4


# the 2.6B-class Q4_K_M decoder ("M26").
M26 = ModelSpec("synthetic-2.6B-q4km", n_layer=40, n_embd=2304, n_head=36, n_head_kv=36, head_dim=64,
                n_ff=5760, n_vocab=73448)
# the 70B-shaped stack ("M70").
M70 = ModelSpec("synthetic-70B-q4km", n_layer=80, n_embd=8192, n_head=64, n_head_kv=8, head_dim=128,
                n_ff=28672, n_vocab=128256)
# Small models for parity tests (GQA, partial rotary, Q8_0 down, Q4_0 mix).
TINY = ModelSpec("tiny-gqa", n_layer=2, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, n_ff=512, n_vocab=1000)
SMALL_Q8DOWN = ModelSpec("small-q8down", n_layer=3, n_embd=512, n_head=8, n_head_kv=8, head_dim=64, n_ff=800,
                         n_vocab=3000, n_rot=32)
SMALL_Q40 = ModelSpec("small-q40", n_layer=2, n_embd=512, n_head=8, n_head_kv=2, head_dim=64, n_ff=1024,
                      n_vocab=2048, mix={"attn_q": SPEC_Q4_0, "ffn_up": SPEC_Q4_0, "attn_output": SPEC_Q8_0,
                                         "ffn_down": SPEC_Q4K})


def _s(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_str(key, val):
    b = val.encode()
    return _s(key) + struct.pack("<I", 8) + struct.pack("<Q", len(b)) + b


def _kv_u32(key, val):
    return _s(key) + struct.pack("<I", 4) + struct.pack("<I", val)


def _kv_f32(key, val):
    return _s(key) + struct.pack("<I", 6) + struct.pack("<f", val)


def _kv_arr_str(key, vals):
    body = b"".join(struct.pack("<Q", len(v)) + v for v in (x if isinstance(x, bytes) else x.encode() for x in vals))
    return _s(key) + struct.pack("<IIQ", 9, 8, len(vals)) + body


def _kv_arr_i32(key, vals):
    return _s(key) + struct.pack("<IIQ", 9, 5, len(vals)) + b"".join(struct.pack("<i", int(v)) for v in vals)


def write_tokenizer_gguf(path: str, tokens, token_types=None, merges=None, pre=None, bos=None, eos=None,
                         name="synthetic-tokenizer") -> None:
    """A GGUF v3 file holding only tokenizer metadata (tokenizer.ggml.*) and no tensors."""
    kvs = [_kv_str("general.architecture", "llama"), _kv_str("general.name", name),
           _kv_arr_str("tokenizer.ggml.tokens", tokens)]
    if token_types is not None:
        kvs.append(_kv_arr_i32("tokenizer.ggml.token_type", token_types))
    if merges is not None:
        kvs.append(_kv_arr_str("tokenizer.ggml.merges", merges))
    if pre is not None:
        kvs.append(_kv_str("tokenizer.ggml.pre", pre))
    if bos is not None:
        kvs.append(_kv_u32("tokenizer.ggml.bos_token_id", bos))
    if eos is not None:
        kvs.append(_kv_u32("tokenizer.ggml.eos_token_id", eos))
    header = struct.pack("<IIQQ", 0x46554747, 3, 0, len(kvs)) + b"".join(kvs)
    with open(path, "wb") as f:
        f.write(header + b"\x00" * ((-len(header)) % 32))


def write_gguf(path: str, spec: ModelSpec, seed: int = 0, alignment: int = 32) -> dict:
    """Writes ``spec`` as a GGUF v3 file; returns a summary dict."""
    tensors = spec.tensor_specs()
    arch = "llama"
    kvs = [_kv_str("general.architecture", arch), _kv_str("general.name", spec.name),
           _kv_u32("general.alignment", alignment),
           _kv_u32(f"{arch}.block_count", spec.n_layer),
           _kv_u32(f"{arch}.context_length", spec.n_ctx_train),
           _kv_u32(f"{arch}.embedding_length", spec.n_embd),
           _kv_u32(f"{arch}.feed_forward_length", spec.n_ff),
           _kv_u32(f"{arch}.attention.head_count", spec.n_head),
           _kv_u32(f"{arch}.attention.head_count_kv", spec.n_head_kv),
           _kv_u32(f"{arch}.attention.key_length", spec.head_dim),
           _kv_u32(f"{arch}.attention.value_length", spec.head_dim),
           _kv_u32(f"{arch}.rope.dimension_count", spec.n_rot or spec.head_dim),
           _kv_f32(f"{arch}.rope.freq_base", spec.rope_theta),
           _kv_f32(f"{arch}.attention.layer_norm_rms_epsilon", spec.rms_eps),
           _kv_u32(f"{arch}.vocab_size", spec.n_vocab)]
    if spec.eos_token_id is not None:
        kvs.append(_kv_u32("tokenizer.ggml.eos_token_id", spec.eos_token_id))
    info = b""
    sizes = []
    offset = 0
    for name, qs, k, rows in tensors:
        ttype = F32 if qs == "norm" else qs.ttype
        be, bb = BLOCK[ttype]
        nbytes = rows * (k // be) * bb
        dims = [k] if qs == "norm" else [k, rows]
        info += _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        info += struct.pack("<I", ttype) + struct.pack("<Q", offset)
        sizes.append(nbytes)
        offset += nbytes + ((-nbytes) % alignment)
    header = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(kvs)) + b"".join(kvs) + info
    with open(path, "wb") as f:
        f.write(header + b"\x00" * ((-len(header)) % alignment))
        for (name, qs, k, rows), nbytes in zip(tensors, sizes):
            ts = tensor_seed(seed, name)
            if qs == "norm":
                data = (np.float32(1.0) + np.float32(0.01) * normal_f32(ts, k)).astype(np.float32).tobytes()
            else:
                data = quant_blocks(qs, ts, rows, k).tobytes()
            assert len(data) == nbytes
            f.write(data)
            f.write(b"\x00" * ((-nbytes) % alignment))
    return {"path": path, "tensors": len(tensors), "data_bytes": offset}


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """n token ids uniform in [0, vocab)."""
    return (splitmix_u64(seed, 0, n) % np.uint64(vocab)).astype(np.uint32)


def config1_inputs(seed: int = 0):
    """Q4_K 6144 x 2048 weights and x ~ N(0,1) of length 2048."""
    w = quant_blocks(SPEC_CONFIG1, tensor_seed(seed, "config1.weight"), 6144, 2048)
    x = normal_f32(tensor_seed(seed, "config1.x"), 2048)
    return w, x


CONFIG2_SHAPES = [(2048, 2048), (2048, 6144), (6144, 2048), (2048, 65536)]  # (k, rows)


def config2_inputs(ttype: int, k: int, rows: int, seed: int = 0):
    spec = {Q6_K: SPEC_Q6K, Q4_0: SPEC_Q4_0, Q8_0: SPEC_Q8_0, Q4_K: SPEC_Q4K}[ttype]
    w = quant_blocks(spec, tensor_seed(seed, f"config2.{ttype}.{k}.{rows}"), rows, k)
    x = normal_f32(tensor_seed(seed, f"config2.x.{k}"), k)
    return w, x


def m26_spec(n_layer: int | None = None, n_vocab: int | None = None) -> ModelSpec:
    """M26, or an M26-shaped model with fewer layers / a smaller vocabulary
    (same per-layer matrices: the small case used for detailed profiles)."""
    import dataclasses

    if n_layer is None and n_vocab is None:
        return M26
    return dataclasses.replace(M26, name=f"m26-{n_layer or M26.n_layer}l-{n_vocab or M26.n_vocab}v",
                               n_layer=n_layer or M26.n_layer, n_vocab=n_vocab or M26.n_vocab)


def m26_path(directory: str, seed: int = 0, spec: ModelSpec | None = None) -> str:
    """Path of the cached M26 (or ``spec``) GGUF in ``directory``, written on first use."""
    import os

    spec = spec or M26
    tag = "m26" if spec is M26 else spec.name
    os.makedirs(directory, exist_ok=True)
    p = os.path.join(directory, f"pk_{tag}_seed{seed}.gguf")
    if not os.path.exists(p):
        tmp = f"{p}.{os.getpid()}.tmp"
        write_gguf(tmp, spec, seed=seed)
        os.replace(tmp, p)
    return p
