"""TEST INFRASTRUCTURE ONLY -- the checker for the library's prompt-text code
(include/pk.h pk_tokenizer_*, pk_tokenize, pk_token_bytes, pk_chat_*).

A plain-Python restatement of the reference's host text path, paths relative
to rust/pocketinfer/src/:
  regexlite.rs:28-270  pattern parser (the reference's own subset and corners:
                       "\\S" inside brackets means "not CR", \\p{P}/\\p{S}/\\p{M}
                       match nothing, a lazy "?" after a quantifier is ignored)
  regexlite.rs:299-446 backtracking matcher and find() (the scan stops at the
                       first position whose match is empty)
  regexlite.rs:461-481 split()
  tokenizer.rs:38-300  from_gguf, encode_word, encode_plain, encode, decode_token
  chat.rs:16-109       is_minicpm5, apply_minicpm5, apply_generic, suffixes
  jni.rs:416-456       a chat request's prompt ids: template, direct-answer suffix,
                       dropping old turns until n_ctx - 1024 holds the ids
Character classes use Unicode properties computed here from `unicodedata`
(general categories) and the White_Space list of the Unicode standard, not
the library's generated tables.  Parity is pinned in tests against the `regex`
module and the Hugging Face `tokenizers` BPE on inputs where those agree with
the reference, and the chat template against the reference's own goldens
(tests/chat_template.rs).  Only tests import this module.
"""
from __future__ import annotations

import unicodedata

# PropList.txt White_Space (Unicode 15.0)
_WHITE_SPACE = set(range(0x09, 0x0E)) | {0x20, 0x85, 0xA0, 0x1680} | set(range(0x2000, 0x200B)) | \
    {0x2028, 0x2029, 0x202F, 0x205F, 0x3000}


def is_white_space(c: str) -> bool:
    return ord(c) in _WHITE_SPACE


def is_numeric(c: str) -> bool:  # Rust char::is_numeric: general category Nd | Nl | No
    return unicodedata.category(c) in ("Nd", "Nl", "No")


def is_letter_category(c: str) -> bool:
    """General category L* or Nl: the part of Alphabetic that categories give.
    Alphabetic also holds Other_Alphabetic (mostly combining marks); tests keep
    such characters out of the text they give this oracle."""
    return unicodedata.category(c) in ("Lu", "Ll", "Lt", "Lm", "Lo", "Nl")


# ---------------------------------------------------------------- patterns
NOMAX = None


class _P:
    def __init__(self, pat: str):
        self.c, self.o = pat, 0

    def peek(self):
        return self.c[self.o] if self.o < len(self.c) else None

    def alts(self, in_group):
        out, seq = [], []
        while True:
            ch = self.peek()
            if ch is None or (ch == ")" and in_group):
                break
            if ch == "|":
                self.o += 1
                out.append(seq)
                seq = []
                continue
            n = self.atom()
            if n is not None:
                seq.append(n)
        out.append(seq)
        return out

    def name(self):
        s = ""
        while self.o < len(self.c):
            ch = self.c[self.o]
            self.o += 1
            if ch == "}":
                break
            s += ch
        return s

    def atom(self):
        ch = self.c[self.o]
        self.o += 1
        if ch == "(":
            kind, neg = "group", False
            if self.peek() == "?":
                self.o += 1
                if self.peek() == ":":
                    self.o += 1
                elif self.peek() in ("!", "="):
                    kind, neg = "look", self.peek() == "!"
                    self.o += 1
            alts = self.alts(True)
            if self.peek() == ")":
                self.o += 1
            base = (kind, neg, alts)
        elif ch == "[":
            base = self.bracket()
        elif ch == ".":
            base = ("any",)
        elif ch == "\\":
            if self.o >= len(self.c):
                return None
            e = self.c[self.o]
            self.o += 1
            if e == "p":
                if self.peek() == "{":
                    self.o += 1
                    nm = self.name()
                    items = [("L",)] if nm in ("L", "Lu", "Ll", "Lt", "Lm", "Lo") else [("N",)] if nm == "N" else []
                    base = ("class", False, items)
                else:
                    base = ("char", "p")
            elif e == "s":
                base = ("class", False, [("S",)])
            elif e == "S":
                base = ("class", True, [("S",)])
            elif e == "d":
                base = ("class", False, [("R", "0", "9")])
            elif e == "w":
                base = ("class", False, [("R", "a", "z"), ("R", "A", "Z"), ("R", "0", "9"), ("C", "_")])
            else:
                base = ("char", {"r": "\r", "n": "\n", "t": "\t"}.get(e, e))
        else:
            base = ("char", ch)
        return self.quant(base)

    def quant(self, base):
        ch = self.peek()
        if ch == "*":
            self.o += 1
            mn, mx = 0, NOMAX
        elif ch == "+":
            self.o += 1
            mn, mx = 1, NOMAX
        elif ch == "?":
            self.o += 1
            mn, mx = 0, 1
        elif ch == "{":
            save = self.o
            self.o += 1
            a = b = ""
            while self.peek() is not None and self.peek().isascii() and self.peek().isdigit():
                a += self.c[self.o]
                self.o += 1
            comma = False
            if self.peek() == ",":
                comma = True
                self.o += 1
                while self.peek() is not None and self.peek().isascii() and self.peek().isdigit():
                    b += self.c[self.o]
                    self.o += 1
            if self.peek() == "}" and (a or comma):
                self.o += 1
                mn = int(a) if a else 0
                mx = (NOMAX if comma else mn) if not b else int(b)
            else:
                self.o = save
                return base
        else:
            return base
        if self.peek() == "?":
            self.o += 1
        return ("rep", base, mn, mx)

    def bracket(self):
        neg = self.peek() == "^"
        if neg:
            self.o += 1
        items = []
        while self.o < len(self.c):
            x = self.c[self.o]
            self.o += 1
            if x == "]":
                break
            if x == "\\":
                e = self.c[self.o] if self.o < len(self.c) else "\\"
                self.o += 1 if self.o < len(self.c) else 0
                if e == "s":
                    items.append(("S",))
                elif e == "S":
                    items.append(("notcr",))
                elif e == "d":
                    items.append(("R", "0", "9"))
                elif e in ("r", "n", "t"):
                    items.append(("C", {"r": "\r", "n": "\n", "t": "\t"}[e]))
                elif e == "p":
                    if self.peek() == "{":
                        self.o += 1
                        nm = self.name()
                        if nm in ("L", "Lu", "Ll", "Lt", "Lm", "Lo"):
                            items.append(("L",))
                        elif nm == "N":
                            items.append(("N",))
                else:
                    items.append(("C", e))
                continue
            if self.peek() == "-" and not (self.o + 1 < len(self.c) and self.c[self.o + 1] == "]"):
                self.o += 1
                hi = "-"
                if self.o < len(self.c):
                    h = self.c[self.o]
                    self.o += 1
                    if h == "\\":
                        if self.o < len(self.c):
                            e = self.c[self.o]
                            self.o += 1
                            hi = {"r": "\r", "n": "\n", "t": "\t"}.get(e, e)
                    else:
                        hi = h
                items.append(("R", x, hi))
            else:
                items.append(("C", x))
        return ("class", neg, items)


def _cls(neg, items, c):
    hit = False
    for it in items:
        k = it[0]
        m = (c == it[1] if k == "C" else it[1] <= c <= it[2] if k == "R" else is_letter_category(c) if k == "L"
             else is_numeric(c) if k == "N" else is_white_space(c) if k == "S" else c != "\r")
        if m:
            hit = True
            break
    return hit != neg


def _seq(nodes, i, t, pos, k):
    if i == len(nodes):
        return k(pos)
    nd = nodes[i]
    kind = nd[0]
    if kind == "char":
        return pos < len(t) and t[pos] == nd[1] and _seq(nodes, i + 1, t, pos + 1, k)
    if kind == "any":
        return pos < len(t) and t[pos] not in "\r\n" and _seq(nodes, i + 1, t, pos + 1, k)
    if kind == "class":
        return pos < len(t) and _cls(nd[1], nd[2], t[pos]) and _seq(nodes, i + 1, t, pos + 1, k)
    if kind == "group":
        return any(_seq(alt, 0, t, pos, lambda p2: _seq(nodes, i + 1, t, p2, k)) for alt in nd[2])
    if kind == "look":
        matched = any(_seq(alt, 0, t, pos, lambda _p: True) for alt in nd[2])
        return matched != nd[1] and _seq(nodes, i + 1, t, pos, k)
    # repeat
    _, node, mn, mx = nd

    def rep(p, count):
        if (mx is None or count < mx) and node[0] not in ("rep", "look"):
            if _seq([node], 0, t, p, lambda p2: p2 != p and rep(p2, count + 1)):
                return True
        return count >= mn and _seq(nodes, i + 1, t, p, k)

    return rep(pos, 0)


class Pattern:
    def __init__(self, pat: str):
        self.alts = _P(pat).alts(False)

    def match_at(self, t: str, pos: int):
        for alt in self.alts:
            end = []
            if _seq(alt, 0, t, pos, lambda p: end.append(p) or True):
                return end[-1]
        return None

    def find(self, t: str):
        out, i = [], 0
        while i < len(t):
            found = None
            for j in range(i, len(t)):
                e = self.match_at(t, j)
                if e is not None:
                    if e > j:
                        found = (j, e)
                    break
            if found is None:
                break
            out.append(found)
            i = found[1]
        return out


def split(pat: Pattern, t: str):
    out, last = [], 0
    for s, e in pat.find(t):
        if s > last:
            out.append(t[last:s])
        out.append(t[s:e])
        last = e
    if last < len(t):
        out.append(t[last:])
    return out or [""]


# ---------------------------------------------------------------- tokenizer
_QWEN = (r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}+| ?[^\s\p{L}"
         r"\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")
PRE = {
    "minicpm5": [r"\p{N}{1,3}", _QWEN],
    "qwen2": [_QWEN],
    "llama3": [r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?"
               r"[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"],
    "gpt-2": [r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)"],
}
for _k in ("qwen2.5", "qwen3"):
    PRE[_k] = PRE["qwen2"]
for _k in ("llama-bpe", "llama-v3"):
    PRE[_k] = PRE["llama3"]


def byte_map():
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    cs = list(bs)
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    enc = {b: chr(c) for b, c in zip(bs, cs)}
    return enc, {v: k for k, v in enc.items()}


class Tokenizer:
    """Tokenizer::from_gguf on already-read metadata (tokens as bytes)."""

    def __init__(self, tokens, token_types=None, merges=(), pre="", bos=None, eos=None):
        self.tokens = [bytes(t) for t in tokens]
        self.types = list(token_types) if token_types is not None else [1] * len(self.tokens)
        self.merges = {}
        for i, m in enumerate(merges):
            m = m if isinstance(m, bytes) else m.encode()
            p = m.find(b" ", 1)
            if len(m) > 1 and p >= 1:
                self.merges[(m[:p], m[p + 1:])] = i
        self.enc, self.dec = byte_map()
        self.tok_id = {}
        self.byte_id = {}
        for i, t in enumerate(self.tokens):
            self.tok_id.setdefault(t, i)
            try:
                s = t.decode()
            except UnicodeDecodeError:
                continue
            if len(s) == 1 and s in self.dec:
                self.byte_id.setdefault(self.dec[s], i)
        self.specials = sorted(((t, i) for i, t in enumerate(self.tokens) if self.types[i] in (2, 3, 4)),
                               key=lambda x: -len(x[0]))
        self.pre = pre or ""
        self.patterns = [Pattern(p) for p in PRE.get(self.pre, PRE["gpt-2"])]
        self.ignore_merges = self.pre == "minicpm5"
        self.bos = bos
        eos_ids = [eos] if eos is not None else []
        eos_ids += [i for t, i in self.specials if t in (b"<|im_end|>", b"<|eot|>", b"<|endoftext|>")]
        self.eos = sorted(set(eos_ids))

    def encode_word(self, word: str, out: list):
        encoded = "".join(self.enc[b] for b in word.encode())
        if self.ignore_merges and encoded.encode() in self.tok_id:
            out.append(self.tok_id[encoded.encode()])
            return
        sym = [c.encode() for c in encoded]
        while True:
            best = None
            for i in range(len(sym) - 1):
                r = self.merges.get((sym[i], sym[i + 1]))
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            i = best[1]
            sym[i:i + 2] = [sym[i] + sym[i + 1]]
        for s in sym:
            if s in self.tok_id:
                out.append(self.tok_id[s])
                continue
            for ch in s.decode():
                if ch.encode() in self.tok_id:
                    out.append(self.tok_id[ch.encode()])
                elif ch in self.dec and self.dec[ch] in self.byte_id:
                    out.append(self.byte_id[self.dec[ch]])

    def encode_plain(self, text: str, out: list):
        words = [text]
        for pat in self.patterns:
            words = [p for w in words for p in split(pat, w) if p]
        for w in words:
            self.encode_word(w, out)

    def encode(self, text: str, parse_special: bool = True) -> list:
        out = []
        if not parse_special or not self.specials:
            self.encode_plain(text, out)
            return out
        b = text.encode()
        pos = plain = 0
        while pos < len(b):
            hit = next(((s, i) for s, i in self.specials if s and b.startswith(s, pos)), None)
            if hit:
                if plain < pos:
                    self.encode_plain(b[plain:pos].decode(), out)
                out.append(hit[1])
                pos += len(hit[0])
                plain = pos
            else:
                c0 = b[pos]
                pos += 1 if c0 < 0x80 else 2 if c0 < 0xE0 else 3 if c0 < 0xF0 else 4
        if plain < len(b):
            self.encode_plain(b[plain:].decode(), out)
        return out

    def token_bytes(self, tid: int) -> bytes:
        if tid >= len(self.tokens):
            return b""
        t = self.tokens[tid]
        if self.types[tid] in (2, 3, 4):
            return t
        try:
            s = t.decode()
        except UnicodeDecodeError:
            return t
        return b"".join(bytes([self.dec[c]]) if c in self.dec else c.encode() for c in s)

    def is_eog(self, tid: int) -> bool:
        return tid in self.eos


# ---------------------------------------------------------------- chat template
def is_minicpm5(pre: str, name: str) -> bool:
    return pre == "minicpm5" or "minicpm5" in name.lower()


def apply_minicpm5(msgs, add_generation_prompt=True) -> str:
    out = "<s>"
    if msgs and msgs[0][0] == "system":
        out += "<|im_start|>system\n" + msgs[0][1] + "<|im_end|>\n"
    i = 0
    while i < len(msgs):
        role, content = msgs[i]
        if role == "user" or (role == "system" and i > 0):
            out += "<|im_start|>" + role + "\n" + content + "<|im_end|>\n"
        elif role == "assistant":
            reasoning = ""
            if "</think>" in content:
                reasoning = content.split("</think>")[0].split("<think>")[-1].rstrip("\n")
                content = content.split("</think>")[-1].lstrip("\n")
            out += "<|im_start|>assistant\n"
            if reasoning:
                out += "<think>\n" + reasoning.strip("\n") + "\n</think>\n\n" + content.lstrip("\n")
            elif "<think>" not in content and "</think>" not in content:
                out += "<think>\n\n</think>\n\n" + content.lstrip("\n")
            else:
                out += content
            out += "<|im_end|>\n"
        elif role == "tool":
            out += "<|im_start|>user"
            while i < len(msgs) and msgs[i][0] == "tool":
                out += "\n<tool_response>\n" + msgs[i][1] + "\n</tool_response>"
                i += 1
            out += "<|im_end|>\n"
            continue
        i += 1
    if add_generation_prompt:
        out += "<|im_start|>assistant\n"
    return out


def apply_generic(msgs, add_generation_prompt=True) -> str:
    out = "".join("<|im_start|>" + r + "\n" + c + "<|im_end|>\n" for r, c in msgs)
    return out + ("<|im_start|>assistant\n" if add_generation_prompt else "")


def chat_prompt(tok: Tokenizer, msgs, minicpm5: bool, direct_answer: bool, n_ctx: int):
    """jni.rs:416-456: (ids, dropped turns, direct suffix applied); raises
    OverflowError where the bridge gives up (the context cannot hold it)."""
    limit = n_ctx - 1024 if n_ctx >= 1024 else float("inf")  # usize wrap-around: no limit
    kept = list(range(len(msgs)))
    while True:
        view = [msgs[i] for i in kept]
        prompt = apply_minicpm5(view, True) if minicpm5 else apply_generic(view, True)
        direct = bool(direct_answer and minicpm5 and prompt.endswith("<|im_start|>assistant\n"))
        if direct:
            prompt += "<think>\n\n</think>\n\n"
        ids = tok.encode(prompt, True)
        if len(ids) <= limit:
            return ids, len(msgs) - len(kept), direct
        oldest = 2 if kept and msgs[kept[0]][0] == "system" else 1
        if len(kept) <= oldest + 1:
            raise OverflowError("Latest request exceeds the context window.")
        del kept[oldest]
