"""Prompt text through the library (include/pk.h pk_tokenizer_*, pk_chat_*):
the GGUF's byte-level BPE tokenizer (rust/pocketinfer/src/tokenizer.rs) and
the chat template (chat.rs).  Host code; no GPU is involved."""
from __future__ import annotations

import ctypes as C

from . import PkError, _check, lib


class TokenizerInfo(C.Structure):
    _fields_ = [("n_vocab", C.c_int32), ("n_eos", C.c_int32), ("bos_id", C.c_int64), ("eos_ids", C.c_uint32 * 16),
                ("ignore_merges", C.c_int32), ("pre", C.c_char * 64)]


class ChatMessage(C.Structure):
    _fields_ = [("role", C.c_char_p), ("content", C.c_char_p)]


class Tokenizer:
    """Tokenizer::from_gguf / encode / decode_token / is_eog."""

    def __init__(self, gguf_path: str):
        self.h = C.c_void_p()
        _check(lib().pk_tokenizer_load(gguf_path.encode(), C.byref(self.h)))

    def close(self):
        if self.h:
            lib().pk_tokenizer_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def info(self) -> dict:
        i = TokenizerInfo()
        _check(lib().pk_tokenizer_info_get(self.h, C.byref(i)))
        return {"n_vocab": i.n_vocab, "bos_id": None if i.bos_id < 0 else i.bos_id,
                "eos_ids": list(i.eos_ids[: min(i.n_eos, 16)]), "ignore_merges": bool(i.ignore_merges),
                "pre": i.pre.decode(errors="replace")}

    def encode(self, text: str | bytes, parse_special: bool = True) -> list:
        b = text.encode() if isinstance(text, str) else bytes(text)
        n = C.c_size_t()
        cap = 2 * len(b) + 8  # at most one id per byte (plus specials, which are longer than one byte)
        out = (C.c_uint32 * cap)()
        _check(lib().pk_tokenize(self.h, b, len(b), int(parse_special), C.cast(out, C.c_void_p), cap, C.byref(n)))
        return list(out[: n.value])

    def token_bytes(self, tid: int) -> bytes:
        n = C.c_size_t()
        lib().pk_token_bytes(self.h, tid, None, 0, C.byref(n))  # size query (reports "needs n")
        out = (C.c_uint8 * max(n.value, 1))()
        _check(lib().pk_token_bytes(self.h, tid, C.cast(out, C.c_void_p), n.value, C.byref(n)))
        return bytes(out[: n.value])

    def decode(self, ids) -> bytes:
        return b"".join(self.token_bytes(int(t)) for t in ids)

    def is_eog(self, tid: int) -> bool:
        return bool(lib().pk_token_is_eog(self.h, tid))


class Utf8Stream:
    """flush_utf8 (model.rs:1355-1388) over a stream of token bytes: feed()
    returns the text that is ready; an incomplete trailing sequence waits."""

    def __init__(self):
        self.pending = b""

    def feed(self, b: bytes) -> bytes:
        data = self.pending + bytes(b)
        buf = (C.c_uint8 * max(len(data), 1)).from_buffer_copy(data or b"\0")
        n = C.c_size_t(len(data))
        out = (C.c_uint8 * (3 * len(data) + 1))()
        m = C.c_size_t()
        _check(lib().pk_utf8_flush(C.cast(buf, C.c_void_p), C.byref(n), C.cast(out, C.c_void_p), len(out),
                                   C.byref(m)))
        self.pending = bytes(buf[: n.value])
        return bytes(out[: m.value])


def find(pattern: str, text: str) -> list:
    """The (start, end) code-point spans of the pattern's matches (regexlite.rs find)."""
    p, t = pattern.encode(), text.encode()
    n = C.c_size_t()
    cap = 2 * len(text) + 2
    out = (C.c_uint32 * cap)()
    _check(lib().pk_text_find(p, len(p), t, len(t), C.cast(out, C.c_void_p), cap, C.byref(n)))
    v = list(out[: n.value])
    return list(zip(v[0::2], v[1::2]))


def split(pattern: str, text: str) -> list:
    """Matches and the text between them (regexlite.rs split)."""
    out, last = [], 0
    for s, e in find(pattern, text):
        if s > last:
            out.append(text[last:s])
        out.append(text[s:e])
        last = e
    if last < len(text):
        out.append(text[last:])
    return out or [""]


def chat_apply(messages, minicpm5: bool = True, add_generation_prompt: bool = True) -> str:
    """chat.rs apply(): messages as [(role, content)] or [{"role", "content"}]."""
    pairs = [(m["role"], m["content"]) if isinstance(m, dict) else tuple(m) for m in messages]
    keep = [(r.encode(), c.encode()) for r, c in pairs]
    arr = (ChatMessage * max(len(keep), 1))(*[ChatMessage(r, c) for r, c in keep])
    n = C.c_size_t()
    lib().pk_chat_apply(C.cast(arr, C.c_void_p), len(keep), int(minicpm5), int(add_generation_prompt), None, 0,
                        C.byref(n))
    out = C.create_string_buffer(max(n.value, 1))
    _check(lib().pk_chat_apply(C.cast(arr, C.c_void_p), len(keep), int(minicpm5), int(add_generation_prompt),
                               C.cast(out, C.c_void_p), n.value, C.byref(n)))
    return out.raw[: n.value].decode()


def chat_prompt(tok: Tokenizer, messages, minicpm5: bool = True, direct_answer: bool = False,
                n_ctx: int = 8192) -> dict:
    """The request's prompt ids as the Android bridge builds them (jni.rs:416-456)."""
    pairs = [(m["role"], m["content"]) if isinstance(m, dict) else tuple(m) for m in messages]
    keep = [(r.encode(), c.encode()) for r, c in pairs]
    arr = (ChatMessage * max(len(keep), 1))(*[ChatMessage(r, c) for r, c in keep])
    cap = sum(len(r) + len(c) for r, c in keep) * 2 + 64
    out = (C.c_uint32 * cap)()
    n, dropped, direct = C.c_size_t(), C.c_int(), C.c_int()
    _check(lib().pk_chat_prompt(tok.h, C.cast(arr, C.c_void_p), len(keep), int(minicpm5), int(direct_answer), n_ctx,
                                C.cast(out, C.c_void_p), cap, C.byref(n), C.byref(dropped), C.byref(direct)))
    return {"ids": list(out[: n.value]), "dropped": dropped.value, "direct_applied": bool(direct.value)}


def is_minicpm5(pre: str, name: str) -> bool:
    return bool(lib().pk_chat_is_minicpm5(pre.encode(), name.encode()))


def direct_suffix() -> str:
    return lib().pk_chat_direct_suffix().decode()


def thinking_on_suffix() -> str:
    return lib().pk_chat_thinking_suffix().decode()


__all__ = ["Tokenizer", "Utf8Stream", "find", "split", "chat_apply", "chat_prompt", "is_minicpm5", "direct_suffix", "thinking_on_suffix", "PkError"]
