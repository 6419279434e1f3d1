"""ctypes binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/_build/libpk_oracle.so`` (the C++ restatement of pocketinfer's
CPU kernels, see pk_oracle.h for the reference line ranges it follows).  Only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this module;
the product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libpk_oracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        sz = C.c_size_t
        L.pko_f16_to_f32.argtypes = [C.c_uint16]
        L.pko_f16_to_f32.restype = C.c_float
        L.pko_f32_to_f16.argtypes = [C.c_float]
        L.pko_f32_to_f16.restype = C.c_uint16
        L.pko_type_block.argtypes = [C.c_uint32, C.POINTER(sz), C.POINTER(sz)]
        L.pko_tensor_nbytes.argtypes = [C.c_uint32, C.c_uint64, C.c_uint64]
        L.pko_tensor_nbytes.restype = C.c_int64
        L.pko_dequant_row.argtypes = [C.c_uint32, P, sz, P]
        L.pko_dot_row_scalar.argtypes = [C.c_uint32, P, sz, P]
        L.pko_dot_row_scalar.restype = C.c_float
        L.pko_row_dot_multi.argtypes = [C.c_uint32, P, sz, P, sz, P]
        L.pko_q8_prepare.argtypes = [P, sz, sz, P, P, P]
        L.pko_dot_row_q8.argtypes = [C.c_uint32, P, sz, P, P, P, sz]
        L.pko_dot_row_q8.restype = C.c_float
        L.pko_dot_row_q8_lanes.argtypes = [C.c_uint32, P, sz, P, P, P, sz, P]
        L.pko_row_int_dots.argtypes = [C.c_uint32, P, sz, P, sz, P]
        L.pko_row_int_dots.restype = sz
        L.pko_matmul.argtypes = [C.c_uint32, P, sz, sz, P, sz, P, sz, C.c_int, P, P, P, sz]
        L.pko_pool_new.argtypes = [sz]
        L.pko_pool_new.restype = P
        L.pko_pool_free.argtypes = [P]
        L.pko_pool_matmul.argtypes = [P, C.c_uint32, P, sz, sz, P, sz, P, sz, C.c_int, P, P, P]
        L.pko_engine_load.argtypes = [C.c_char_p, sz, sz, C.c_char_p, sz]
        L.pko_engine_load.restype = P
        L.pko_engine_free.argtypes = [P]
        L.pko_engine_set_int8.argtypes = [P, C.c_int]
        L.pko_engine_set_eog.argtypes = [P, C.c_int]
        L.pko_engine_set_kv_f16.argtypes = [P, C.c_int]
        L.pko_engine_vocab.argtypes = [P]
        L.pko_engine_vocab.restype = sz
        L.pko_forward.argtypes = [P, P, P, sz, C.c_int, C.c_char_p, sz]
        L.pko_logits.argtypes = [P, P, sz]
        L.pko_logits.restype = sz
        L.pko_generate.argtypes = [P, P, sz, sz, C.c_float, C.c_float, C.c_uint64, P, sz,
                                   C.POINTER(sz), P, C.c_char_p, sz]
        L.pko_engine_set_debug.argtypes = [P, C.c_int]
        L.pko_engine_dump.argtypes = [P, C.c_char_p, P, sz]
        L.pko_engine_dump.restype = sz
        L.pko_expf_batch.argtypes = [P, P, sz]
        L.pko_sample.argtypes = [P, sz, C.c_float, C.c_float, C.POINTER(C.c_uint64)]
        L.pko_sample.restype = C.c_uint32
        L.pko_rng_new.argtypes = [C.c_uint64]
        L.pko_rng_new.restype = C.c_uint64
        L.pko_rng_next_u64.argtypes = [C.POINTER(C.c_uint64)]
        L.pko_rng_next_u64.restype = C.c_uint64
        L.pko_rng_next_f32.argtypes = [C.POINTER(C.c_uint64)]
        L.pko_rng_next_f32.restype = C.c_float
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def type_block(t: int):
    be, bb = C.c_size_t(), C.c_size_t()
    if not lib().pko_type_block(t, C.byref(be), C.byref(bb)):
        return None
    return be.value, bb.value


def row_bytes(t: int, k: int) -> int:
    be, bb = type_block(t)
    return k // be * bb


def f16_to_f32(h: int) -> float:
    return lib().pko_f16_to_f32(h)


def f32_to_f16(v: float) -> int:
    return lib().pko_f32_to_f16(v)


def dequant_row(t: int, data: np.ndarray, k: int) -> np.ndarray:
    out = np.zeros(k, np.float32)
    lib().pko_dequant_row(t, _p(np.ascontiguousarray(data, np.uint8)), k, _p(out))
    return out


def dot_row(t: int, data: np.ndarray, k: int, x: np.ndarray) -> float:
    return lib().pko_dot_row_scalar(t, _p(np.ascontiguousarray(data, np.uint8)), k,
                                    _p(np.ascontiguousarray(x, np.float32)))


def row_dot_multi(t, row, k, xt, b):
    out = np.zeros(b, np.float32)
    lib().pko_row_dot_multi(t, _p(np.ascontiguousarray(row, np.uint8)), k,
                            _p(np.ascontiguousarray(xt, np.float32)), b, _p(out))
    return out


class Q8Act:
    """Q8Act (quant_int.rs:3-10): q [b][k] i8, d [b][k/32] f32, sum [b][k/32] i32."""

    def __init__(self, x: np.ndarray, k: int, b: int):
        x = np.ascontiguousarray(x, np.float32)
        assert x.size == k * b
        self.k, self.b, self.nb = k, b, k // 32
        self.q = np.zeros(k * b, np.int8)
        self.d = np.zeros(self.nb * b, np.float32)
        self.sum = np.zeros(self.nb * b, np.int32)
        lib().pko_q8_prepare(_p(x), k, b, _p(self.q), _p(self.d), _p(self.sum))


def dot_row_q8(t, row, k, act: Q8Act, lane: int) -> float:
    return lib().pko_dot_row_q8(t, _p(np.ascontiguousarray(row, np.uint8)), k, _p(act.q), _p(act.d),
                                _p(act.sum), lane)


def dot_row_q8_lanes(t, row, k, act: Q8Act, b: int) -> np.ndarray:
    out = np.zeros(b, np.float32)
    lib().pko_dot_row_q8_lanes(t, _p(np.ascontiguousarray(row, np.uint8)), k, _p(act.q), _p(act.d),
                               _p(act.sum), b, _p(out))
    return out


def row_int_dots(t, row, k, act: Q8Act, lane: int) -> np.ndarray:
    dots = np.zeros(k // 16 + 16, np.int32)
    n = lib().pko_row_int_dots(t, _p(np.ascontiguousarray(row, np.uint8)), k, _p(act.q), lane, _p(dots))
    return dots[:n].copy()


def matmul(t, w: np.ndarray, rb: int, k: int, xt: np.ndarray, b: int, n_rows: int,
           act: Q8Act | None, threads: int = 1) -> np.ndarray:
    """Pool::matmul: out [n_rows][b]."""
    out = np.zeros(n_rows * b, np.float32)
    xt = np.ascontiguousarray(xt, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    if act is None:
        lib().pko_matmul(t, _p(w), rb, k, _p(xt), b, _p(out), n_rows, 0, None, None, None, threads)
    else:
        lib().pko_matmul(t, _p(w), rb, k, _p(xt), b, _p(out), n_rows, 1, _p(act.q), _p(act.d),
                         _p(act.sum), threads)
    return out


class Pool:
    def __init__(self, threads: int):
        self.h = lib().pko_pool_new(threads)

    def matmul(self, t, w, rb, k, xt, b, n_rows, act: Q8Act | None, out=None):
        if out is None:
            out = np.zeros(n_rows * b, np.float32)
        if act is None:
            lib().pko_pool_matmul(self.h, t, _p(w), rb, k, _p(xt), b, _p(out), n_rows, 0, None, None, None)
        else:
            lib().pko_pool_matmul(self.h, t, _p(w), rb, k, _p(xt), b, _p(out), n_rows, 1, _p(act.q),
                                  _p(act.d), _p(act.sum))
        return out

    def close(self):
        if self.h:
            lib().pko_pool_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Stats(C.Structure):
    _fields_ = [("prefill_tokens", C.c_size_t), ("prefill_cached_tokens", C.c_size_t),
                ("prefill_ms", C.c_double), ("gen_tokens", C.c_size_t), ("gen_ms", C.c_double),
                ("stop", C.c_char * 32)]


class Engine:
    """Engine::load / forward / generate of the CPU oracle."""

    def __init__(self, path: str, n_ctx: int, threads: int = 1):
        err = C.create_string_buffer(512)
        self.h = lib().pko_engine_load(path.encode(), n_ctx, threads, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self.vocab = lib().pko_engine_vocab(self.h)
        self.n_ctx = n_ctx

    def close(self):
        if getattr(self, "h", None):
            lib().pko_engine_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def set_int8(self, on: bool):
        lib().pko_engine_set_int8(self.h, int(on))

    def set_eog(self, on: bool):
        lib().pko_engine_set_eog(self.h, int(on))

    def set_kv_f16(self, on: bool):
        """Cache entries rounded to f16 at store (the library's f16 KV mode)."""
        lib().pko_engine_set_kv_f16(self.h, int(on))

    def set_debug(self, on: bool):
        lib().pko_engine_set_debug(self.h, int(on))

    def dump(self, name: str) -> np.ndarray | None:
        n = lib().pko_engine_dump(self.h, name.encode(), None, 0)
        if n == 0:
            return None
        out = np.zeros(n, np.float32)
        lib().pko_engine_dump(self.h, name.encode(), _p(out), n)
        return out

    def forward(self, ids, positions, want_logits=True):
        ids = np.ascontiguousarray(ids, np.uint32)
        pos = np.ascontiguousarray(positions, np.uint64)
        err = C.create_string_buffer(512)
        rc = lib().pko_forward(self.h, _p(ids), _p(pos), len(ids), int(want_logits), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())

    def logits(self) -> np.ndarray:
        out = np.zeros(self.vocab, np.float32)
        lib().pko_logits(self.h, _p(out), self.vocab)
        return out

    def generate(self, prompt, max_tokens, temp=0.0, top_p=1.0, seed=1):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        n_out = C.c_size_t()
        st = Stats()
        err = C.create_string_buffer(512)
        rc = lib().pko_generate(self.h, _p(prompt), len(prompt), max_tokens, temp, top_p, seed, _p(out),
                                len(out), C.byref(n_out), C.byref(st), err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return {
            "gen_ids": out[: n_out.value].tolist(),
            "prefill_tokens": st.prefill_tokens,
            "prefill_cached_tokens": st.prefill_cached_tokens,
            "prefill_ms": st.prefill_ms,
            "gen_tokens": st.gen_tokens,
            "gen_ms": st.gen_ms,
            "stop": st.stop.decode(),
        }


def expf_batch(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().pko_expf_batch(_p(x), _p(out), x.size)
    return out


def request_stop():
    lib().pko_request_stop()


def clear_stop():
    lib().pko_clear_stop()


class Rng:
    """sampler.rs:1-19 splitmix64."""

    def __init__(self, seed: int):
        self.s = C.c_uint64(lib().pko_rng_new(seed))

    def next_u64(self) -> int:
        return lib().pko_rng_next_u64(C.byref(self.s))

    def next_f32(self) -> float:
        return lib().pko_rng_next_f32(C.byref(self.s))


def sample(logits: np.ndarray, temp: float, top_p: float, rng: Rng) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return lib().pko_sample(_p(logits), logits.size, temp, top_p, C.byref(rng.s))
