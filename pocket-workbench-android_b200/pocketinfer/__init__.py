"""Python binding of libpocketinfer_b200.so (the C ABI declared in include/pk.h).

This mirrors the reference's operator surface for the decode path
(rust/pocketinfer/src in Aleinto97/pocket-workbench-android):

  q8_quantize        Q8Act::prepare            quant_int.rs:17-56
  matmul             Pool::matmul, int8 path   model.rs:242-321
  Backend            OpenClBackend             backend/opencl.rs:261-500
  Engine             Engine::{load,forward,logits,generate}   model.rs:698-1352

The binding only marshals arguments; every computation runs in the CUDA
library.  There is no CPU fallback: if the library is missing or no GPU is
present, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG_DIR, "lib", "libpocketinfer_b200.so")

PK_OK = 0
PK_ERR = {1: "PK_ERR_INVALID", 2: "PK_ERR_UNSUPPORTED", 3: "PK_ERR_CUDA", 4: "PK_ERR_OOM", 5: "PK_ERR_IO",
          6: "PK_ERR_CONTEXT_FULL", 7: "PK_ERR_STOPPED", 8: "PK_ERR_TIMEOUT"}

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30
ORDER_EXACT, ORDER_FAST = 0, 1  # pk_set_order
MATMUL_MMA_SYNC, MATMUL_TCGEN05 = 0, 1  # pk_set_matmul_path
KV_F32, KV_F16 = 0, 1  # pk_set_kv_type
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

# Every function include/pk.h declares (checked by tests/test_capi_symbols.py).
SYMBOLS = [
    "pk_last_error", "pk_version", "pk_device_binary_version", "pk_supports", "pk_expf", "pk_q8_quantize", "pk_matmul", "pk_matmul_noalloc", "pk_packed_bytes",
    "pk_pack_weights", "pk_matmul_packed", "pk_set_matmul_path", "pk_backend_new", "pk_backend_free", "pk_backend_selftest",
    "pk_backend_supports", "pk_backend_matvec", "pk_create", "pk_load_gguf", "pk_destroy", "pk_model_info_get",
    "pk_forward", "pk_logits", "pk_argmax", "pk_generate", "pk_decode_steps_device", "pk_set_position", "pk_set_order", "pk_set_kv_type",
    "pk_decode_profile", "pk_selftest_bounded_wait", "pk_set_debug", "pk_get_dump", "pk_request_stop",
    "pk_clear_stop", "pk_tp_create", "pk_tp_destroy", "pk_tp_load_gguf", "pk_tp_load_synthetic",
    "pk_tp_handle_bytes", "pk_tp_ipc_handle", "pk_tp_open_peers", "pk_tp_nccl_id_bytes", "pk_tp_nccl_id",
    "pk_tp_use_nccl", "pk_tp_prefill", "pk_tp_decode", "pk_tp_logits",
    "pk_tp_info_get", "pk_tp_split", "pk_tp_pick", "pk_sample_scratch_bytes", "pk_sample",
    "pk_streams_begin", "pk_stream_prefill", "pk_streams_decode", "pk_streams_set_position",
    "pk_tokenizer_load", "pk_tokenizer_free", "pk_tokenizer_info_get", "pk_tokenize", "pk_token_bytes",
    "pk_token_is_eog", "pk_utf8_flush", "pk_text_find", "pk_chat_apply", "pk_chat_prompt", "pk_chat_is_minicpm5", "pk_chat_direct_suffix", "pk_chat_thinking_suffix",
]


class PkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{PK_ERR.get(code, code)}: {msg}")
        self.code = code


class Q8ActC(C.Structure):
    _fields_ = [("q", C.c_void_p), ("d", C.c_void_p), ("sum", C.c_void_p), ("k", C.c_int), ("b", C.c_int)]


class ModelInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_rot",
                                       "n_vocab", "n_ctx")] + \
               [("rope_theta", C.c_float), ("rms_eps", C.c_float), ("weight_bytes", C.c_size_t),
                ("kv_bytes", C.c_size_t), ("stream_bytes", C.c_size_t), ("decode_kernels", C.c_int)]


class GenOpts(C.Structure):
    _fields_ = [("temp", C.c_float), ("top_p", C.c_float), ("seed", C.c_uint64), ("max_tokens", C.c_int),
                ("stop_at_eog", C.c_int)]


class GenStats(C.Structure):
    _fields_ = [("prefill_tokens", C.c_int), ("prefill_cached_tokens", C.c_int), ("prefill_ms", C.c_double),
                ("gen_tokens", C.c_int), ("gen_ms", C.c_double), ("stop", C.c_char * 32)]


class KernelStat(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_int), ("ms", C.c_double), ("bytes", C.c_double)]


class TpInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("rank", "world", "n_layer", "n_embd", "n_head", "n_head_kv", "head_dim",
                                       "n_ff", "n_vocab", "local_heads", "local_kv_heads", "local_ff", "vocab0",
                                       "local_vocab")] + \
               [("weight_bytes", C.c_size_t), ("stream_bytes", C.c_size_t), ("collectives_per_token", C.c_int)]


class TpModel(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "n_vocab",
                                       "n_rot")] + [("rope_theta", C.c_float), ("rms_eps", C.c_float)]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_uint32, C.c_void_p)

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-j4", "-C", PKG_DIR], check=True)
    return LIB_PATH


def lib():
    """Loads the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    P, I, U32, SZ = C.c_void_p, C.c_int, C.c_uint32, C.c_size_t
    sig = {
        "pk_last_error": ([], C.c_char_p), "pk_version": ([], I), "pk_device_binary_version": ([C.POINTER(I)], I), "pk_supports": ([U32], I),
        "pk_q8_quantize": ([P, I, I, C.POINTER(Q8ActC), P], I), "pk_expf": ([P, P, I, P], I),
        "pk_matmul": ([U32, P, SZ, I, I, C.POINTER(Q8ActC), P, P], I),
        "pk_matmul_noalloc": ([U32, P, SZ, I, I, C.POINTER(Q8ActC), P, P], I),
        "pk_packed_bytes": ([U32, I, I], SZ),
        "pk_pack_weights": ([U32, P, SZ, I, I, P, P], I),
        "pk_matmul_packed": ([U32, P, I, I, C.POINTER(Q8ActC), P, P], I),
        "pk_backend_new": ([I, C.POINTER(P)], I), "pk_backend_free": ([P], None),
        "pk_backend_selftest": ([P], I), "pk_backend_supports": ([P, U32], I),
        "pk_backend_matvec": ([P, U32, P, SZ, I, P, P, I], I),
        "pk_create": ([I, I, I, C.POINTER(P)], I), "pk_load_gguf": ([P, C.c_char_p], I),
        "pk_destroy": ([P], None), "pk_model_info_get": ([P, C.POINTER(ModelInfo)], I),
        "pk_forward": ([P, P, P, I, I], I), "pk_logits": ([P, P, I], I),
        "pk_argmax": ([P, C.POINTER(U32)], I),
        "pk_generate": ([P, P, I, C.POINTER(GenOpts), TOKEN_CB, P, P, I, C.POINTER(I), C.POINTER(GenStats)], I),
        "pk_decode_steps_device": ([P, I, P, C.POINTER(C.c_float)], I), "pk_set_matmul_path": ([I], I), "pk_set_position": ([P, I], I), "pk_set_order": ([P, I], I), "pk_set_kv_type": ([P, I], I),
        "pk_streams_begin": ([P, I], I), "pk_stream_prefill": ([P, I, P, I], I),
        "pk_streams_decode": ([P, I, P, C.POINTER(C.c_float)], I), "pk_streams_set_position": ([P, I], I),
        "pk_decode_profile": ([P, C.POINTER(KernelStat), I, C.POINTER(I)], I), "pk_set_debug": ([P, I], I),
        "pk_selftest_bounded_wait": ([P, C.POINTER(I)], I),
        "pk_get_dump": ([P, C.c_char_p, P, I, C.POINTER(I)], I),
        "pk_request_stop": ([], None), "pk_clear_stop": ([], None),
        "pk_tp_create": ([I, I, I, I, C.POINTER(P)], I), "pk_tp_destroy": ([P], None),
        "pk_tp_load_gguf": ([P, C.c_char_p], I), "pk_tp_load_synthetic": ([P, C.POINTER(TpModel), C.c_uint64], I),
        "pk_tp_handle_bytes": ([], I), "pk_tp_ipc_handle": ([P, P], I), "pk_tp_open_peers": ([P, P], I),
        "pk_tp_nccl_id_bytes": ([], I), "pk_tp_nccl_id": ([P], I), "pk_tp_use_nccl": ([P, P], I),
        "pk_tp_prefill": ([P, P, I], I), "pk_tp_decode": ([P, I, P, C.POINTER(C.c_float)], I),
        "pk_tp_logits": ([P, P, I, C.POINTER(I), C.POINTER(I)], I), "pk_tp_info_get": ([P, C.POINTER(TpInfo)], I),
        "pk_tp_split": ([I, I, I, I, I, I, I, I, I, P], I), "pk_tp_pick": ([P, P, I], U32),
        "pk_sample_scratch_bytes": ([I], SZ),
        "pk_sample": ([P, I, C.c_float, C.c_float, P, P, P, P], I),
        "pk_tokenizer_load": ([C.c_char_p, C.POINTER(P)], I), "pk_tokenizer_free": ([P], None),
        "pk_tokenizer_info_get": ([P, P], I), "pk_tokenize": ([P, C.c_char_p, SZ, I, P, SZ, C.POINTER(SZ)], I),
        "pk_token_bytes": ([P, U32, P, SZ, C.POINTER(SZ)], I), "pk_token_is_eog": ([P, U32], I),
        "pk_text_find": ([C.c_char_p, SZ, C.c_char_p, SZ, P, SZ, C.POINTER(SZ)], I),
        "pk_utf8_flush": ([P, C.POINTER(SZ), P, SZ, C.POINTER(SZ)], I),
        "pk_chat_apply": ([P, I, I, I, P, SZ, C.POINTER(SZ)], I), "pk_chat_is_minicpm5": ([C.c_char_p, C.c_char_p], I),
        "pk_chat_prompt": ([P, P, I, I, I, SZ, P, SZ, C.POINTER(SZ), C.POINTER(I), C.POINTER(I)], I),
        "pk_chat_direct_suffix": ([], C.c_char_p), "pk_chat_thinking_suffix": ([], C.c_char_p),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(rc: int):
    if rc != PK_OK:
        raise PkError(rc, lib().pk_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib().pk_last_error().decode(errors="replace")


def supports(ttype: int) -> bool:
    return bool(lib().pk_supports(ttype))


def row_bytes(ttype: int, k: int) -> int:
    be, bb = BLOCK[ttype]
    return k // be * bb


def _stream(stream):
    if stream is None:
        import torch

        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


class Q8Act:
    """Q8Act in device memory (torch tensors): q [b][k] i8, d/sum [b][k/32]."""

    def __init__(self, k: int, b: int, device="cuda"):
        import torch

        self.k, self.b = k, b
        self.q = torch.empty(b * k, dtype=torch.int8, device=device)
        self.d = torch.empty(max(1, b * (k // 32)), dtype=torch.float32, device=device)
        self.sum = torch.empty(max(1, b * (k // 32)), dtype=torch.int32, device=device)
        self.c = Q8ActC(self.q.data_ptr(), self.d.data_ptr(), self.sum.data_ptr(), k, b)


def expf(x, stream=None):
    """The device exp of softmax and SwiGLU (bit-identical to the C library's expf)."""
    import torch

    assert x.is_cuda and x.dtype == torch.float32 and x.is_contiguous()
    out = torch.empty_like(x)
    _check(lib().pk_expf(_ptr(x), _ptr(out), x.numel(), _stream(stream)))
    return out


def sample(logits, temp: float, top_p: float, rng_state: int, stream=None):
    """sampler.rs:21-92 (temp > 0) on a device float32 vector; returns (token, new rng state)."""
    import torch

    assert logits.is_cuda and logits.dtype == torch.float32 and logits.is_contiguous()
    n = logits.numel()
    scratch = torch.empty(lib().pk_sample_scratch_bytes(n) + 256, dtype=torch.uint8, device=logits.device)
    base = (scratch.data_ptr() + 255) // 256 * 256
    r = rng_state & 0xFFFFFFFFFFFFFFFF
    st = torch.tensor([r - (1 << 64) if r >= 1 << 63 else r], dtype=torch.int64, device=logits.device)
    tok = torch.zeros(1, dtype=torch.int32, device=logits.device)
    _check(lib().pk_sample(_ptr(logits), n, temp, top_p, _ptr(st), C.c_void_p(base), _ptr(tok), _stream(stream)))
    torch.cuda.synchronize(logits.device)
    return int(tok.item()) & 0xFFFFFFFF, int(st.item()) & 0xFFFFFFFFFFFFFFFF


def q8_quantize(x, k: int, b: int, stream=None) -> Q8Act:
    """Q8Act::prepare of a feature-major device tensor x [k][b]."""
    assert x.is_cuda and x.dtype.itemsize == 4 and x.numel() == k * b and x.is_contiguous()
    act = Q8Act(k, b, x.device)
    _check(lib().pk_q8_quantize(_ptr(x), k, b, C.byref(act.c), _stream(stream)))
    return act


def matmul(ttype: int, w, k: int, n_rows: int, act: Q8Act, out=None, stream=None):
    """Pool::matmul (int8 path) on raw GGUF rows in device memory; returns out [n_rows][b]."""
    import torch

    if out is None:
        out = torch.empty(n_rows * act.b, dtype=torch.float32, device=w.device)
    _check(lib().pk_matmul(ttype, _ptr(w), row_bytes(ttype, k), k, n_rows, C.byref(act.c), _ptr(out),
                           _stream(stream)))
    return out


def packed_bytes(ttype: int, k: int, n_rows: int) -> int:
    return lib().pk_packed_bytes(ttype, k, n_rows)


def pack_weights(ttype: int, w, k: int, n_rows: int, stream=None):
    import torch

    packed = torch.empty(packed_bytes(ttype, k, n_rows), dtype=torch.uint8, device=w.device)
    _check(lib().pk_pack_weights(ttype, _ptr(w), row_bytes(ttype, k), k, n_rows, _ptr(packed), _stream(stream)))
    return packed


NOALLOC_SCRATCH_BYTES = 16 << 20


def matmul_noalloc(ttype: int, w, k: int, n_rows: int, act: Q8Act, out=None, stream=None):
    """matmul() without a device allocation: packs into the library's fixed scratch."""
    import torch

    if out is None:
        out = torch.empty(n_rows * act.b, dtype=torch.float32, device=w.device)
    _check(lib().pk_matmul_noalloc(ttype, _ptr(w), row_bytes(ttype, k), k, n_rows, C.byref(act.c), _ptr(out),
                                   _stream(stream)))
    return out


def matmul_packed(ttype: int, packed, k: int, n_rows: int, act: Q8Act, out=None, stream=None):
    import torch

    if out is None:
        out = torch.empty(n_rows * act.b, dtype=torch.float32, device=packed.device)
    _check(lib().pk_matmul_packed(ttype, _ptr(packed), k, n_rows, C.byref(act.c), _ptr(out), _stream(stream)))
    return out


def set_matmul_path(path: str):
    """The b > 8 matvec kernel for this process: "mma.sync" (default) or "tcgen05"."""
    _check(lib().pk_set_matmul_path({"mma.sync": MATMUL_MMA_SYNC, "tcgen05": MATMUL_TCGEN05}[path]))


class Backend:
    """OpenClBackend analogue: host weights cached on the device, host x/out."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().pk_backend_new(device, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().pk_backend_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def selftest(self):
        _check(lib().pk_backend_selftest(self.h))

    def supports(self, ttype: int) -> bool:
        return bool(lib().pk_backend_supports(self.h, ttype))

    def matvec(self, ttype: int, w, k: int, x, n_rows: int):
        import numpy as np

        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(n_rows, np.float32)
        _check(lib().pk_backend_matvec(self.h, ttype, w.ctypes.data_as(C.c_void_p), w.nbytes, k,
                                       x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), n_rows))
        return out


class Engine:
    """Engine::load / forward / logits / generate on one GPU."""

    def __init__(self, path: str | None = None, n_ctx: int = 512, max_batch: int = 32, device: int = 0,
                 order: str | None = None, kv: str = "f32"):
        h = C.c_void_p()
        _check(lib().pk_create(device, n_ctx, max_batch, C.byref(h)))
        self.h = h
        self.n_ctx = n_ctx
        if order is not None:
            self.set_order(order)
        if kv != "f32":  # "f16": f16 K/V cache entries (pk_set_kv_type), before the load
            _check(lib().pk_set_kv_type(self.h, {"f32": KV_F32, "f16": KV_F16}[kv]))
        if path is not None:
            self.load(path)

    def set_order(self, order: str):
        """Float order of the b = 1 decode step: "exact" (the reference's) or "fast"."""
        _check(lib().pk_set_order(self.h, {"exact": ORDER_EXACT, "fast": ORDER_FAST}[order]))

    def load(self, path: str):
        _check(lib().pk_load_gguf(self.h, path.encode()))
        self.info = self.model_info()
        self.vocab = self.info["n_vocab"]

    def close(self):
        if getattr(self, "h", None):
            lib().pk_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def model_info(self) -> dict:
        mi = ModelInfo()
        _check(lib().pk_model_info_get(self.h, C.byref(mi)))
        return {n: getattr(mi, n) for n, _ in ModelInfo._fields_}

    def forward(self, ids, positions, want_logits=True):
        import numpy as np

        ids = np.ascontiguousarray(ids, np.uint32)
        pos = np.ascontiguousarray(positions, np.int32)
        _check(lib().pk_forward(self.h, ids.ctypes.data_as(C.c_void_p), pos.ctypes.data_as(C.c_void_p), len(ids),
                                int(want_logits)))

    def logits(self):
        import numpy as np

        out = np.empty(self.vocab, np.float32)
        _check(lib().pk_logits(self.h, out.ctypes.data_as(C.c_void_p), self.vocab))
        return out

    def argmax(self) -> int:
        t = C.c_uint32()
        _check(lib().pk_argmax(self.h, C.byref(t)))
        return t.value

    def generate(self, prompt, max_tokens: int, temp: float = 0.0, top_p: float = 1.0, seed: int = 1,
                 stop_at_eog: bool = True, callback=None) -> dict:
        import numpy as np

        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_tokens, 1), np.uint32)
        n_out = C.c_int()
        st = GenStats()
        opts = GenOpts(temp, top_p, seed, max_tokens, int(stop_at_eog))
        cb = TOKEN_CB(lambda tok, user: int(bool(callback(tok)))) if callback else TOKEN_CB()
        _check(lib().pk_generate(self.h, prompt.ctypes.data_as(C.c_void_p), len(prompt), C.byref(opts), cb, None,
                                 out.ctypes.data_as(C.c_void_p), len(out), C.byref(n_out), C.byref(st)))
        return {"gen_ids": out[: min(n_out.value, len(out))].tolist(), "prefill_tokens": st.prefill_tokens,
                "prefill_cached_tokens": st.prefill_cached_tokens, "prefill_ms": st.prefill_ms,
                "gen_tokens": st.gen_tokens, "gen_ms": st.gen_ms, "stop": st.stop.decode()}

    def decode_steps_device(self, n_steps: int, return_ms: bool = False):
        """n_steps greedy steps kept on the device; optionally the CUDA-event time (ms)."""
        import numpy as np

        out = np.zeros(max(n_steps, 1), np.uint32)
        ms = C.c_float()
        _check(lib().pk_decode_steps_device(self.h, n_steps, out.ctypes.data_as(C.c_void_p), C.byref(ms)))
        ids = out[:n_steps].tolist()
        return (ids, ms.value) if return_ms else ids

    def set_position(self, pos: int):
        _check(lib().pk_set_position(self.h, pos))

    def streams_begin(self, n_streams: int):
        """n_streams independent sequences, each with its own KV cache, decoded together."""
        _check(lib().pk_streams_begin(self.h, n_streams))
        self.n_streams = n_streams

    def stream_prefill(self, s: int, prompt):
        import numpy as np

        p = np.ascontiguousarray(prompt, np.uint32)
        _check(lib().pk_stream_prefill(self.h, s, p.ctypes.data_as(C.c_void_p), len(p)))

    def streams_decode(self, n_steps: int, return_ms: bool = False):
        """n_steps greedy tokens of every stream: a list per stream (optionally the device time, ms)."""
        import numpy as np

        out = np.zeros((max(n_steps, 1), self.n_streams), np.uint32)
        ms = C.c_float()
        _check(lib().pk_streams_decode(self.h, n_steps, out.ctypes.data_as(C.c_void_p), C.byref(ms)))
        ids = [out[:n_steps, s].tolist() for s in range(self.n_streams)]
        return (ids, ms.value) if return_ms else ids

    def streams_set_position(self, pos: int):
        _check(lib().pk_streams_set_position(self.h, pos))

    def decode_profile(self) -> list:
        stats = (KernelStat * 128)()
        n = C.c_int()
        _check(lib().pk_decode_profile(self.h, stats, 128, C.byref(n)))
        return [{"name": s.name.decode(), "launches": s.launches, "ms": s.ms, "bytes": s.bytes}
                for s in stats[: n.value]]

    def selftest_bounded_wait(self) -> int:
        """One persistent-kernel launch whose bounded waits are made to run out;
        returns the status that launch produced (PK_ERR_TIMEOUT = 8 expected)."""
        st = C.c_int()
        _check(lib().pk_selftest_bounded_wait(self.h, C.byref(st)))
        return st.value

    def set_debug(self, on: bool):
        _check(lib().pk_set_debug(self.h, int(on)))

    def dump(self, name: str):
        import numpy as np

        n = C.c_int()
        rc = lib().pk_get_dump(self.h, name.encode(), None, 0, C.byref(n))
        if rc != PK_OK:
            return None
        out = np.empty(n.value, np.float32)
        _check(lib().pk_get_dump(self.h, name.encode(), out.ctypes.data_as(C.c_void_p), n.value, C.byref(n)))
        return out


def request_stop():
    lib().pk_request_stop()


def clear_stop():
    lib().pk_clear_stop()
