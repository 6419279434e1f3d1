"""Prompt text on the host (include/pk.h pk_tokenizer_*, pk_tokenize,
pk_token_bytes, pk_text_find, pk_chat_*): the library against the oracle
restatement (oracle/pktext.py), and the oracle pinned to
  * the reference's chat-template goldens (tests/golden/chat_template.json,
    from rust/pocketinfer/tests/chat_template.rs),
  * the `regex` module's matches of the pre-tokenizer patterns,
  * the Hugging Face `tokenizers` byte-level BPE (merges by rank, and the
    whole-word lookup of ignore_merges),
on texts where those engines and the reference agree (no combining marks,
no characters whose Alphabetic property differs from their L* category).
No GPU is involved: tokenisation is host code."""
import json
import os
import random
import re
import sys

import pytest

sys.setrecursionlimit(100000)

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

ASCII = "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ"
PUNCT = "!\"#$%&()*+,-./:;<=>?@[\\]^_`{|}~"
WORLD = "àèéìòùçñüßÆøåαβγδωжзикл中文字符测试日本語"
DIGITS = "0123456789٣٤½"
SPACES = [" ", " ", " ", "  ", "\n", "\n\n", "\r\n", "\t", " ", "　", " \n "]
APOS = ["'s", "'t", "'re", "'VE", "'m", "'ll", "'D"]
EMOJI = "😀🚀✓"


def rand_text(rng: random.Random, n_words: int) -> str:
    out = []
    for _ in range(n_words):
        r = rng.random()
        if r < 0.45:
            w = "".join(rng.choice(ASCII) for _ in range(rng.randint(1, 9)))
        elif r < 0.6:
            w = "".join(rng.choice(WORLD) for _ in range(rng.randint(1, 5)))
        elif r < 0.72:
            w = "".join(rng.choice(DIGITS) for _ in range(rng.randint(1, 8)))
        elif r < 0.84:
            w = "".join(rng.choice(PUNCT) for _ in range(rng.randint(1, 3)))
        elif r < 0.9:
            w = rng.choice(APOS)
        else:
            w = rng.choice(EMOJI)
        out.append(w)
        out.append(rng.choice(SPACES) if rng.random() < 0.8 else "")
    return "".join(out)


@pytest.fixture(scope="module")
def text(pk):
    from pocketinfer import text as t

    return t


@pytest.fixture(scope="module")
def ot():
    import pktext

    return pktext


# ---------------------------------------------------------------- chat template
def test_chat_template_reference_goldens(text, ot):
    gold = json.load(open(os.path.join(HERE, "golden", "chat_template.json"), encoding="utf-8"))
    assert len(gold["cases"]) == 6
    for c in gold["cases"]:
        msgs = [tuple(m) for m in c["messages"]]
        assert ot.apply_minicpm5(msgs, c["add_generation_prompt"]) == c["expected"], c["name"]
        assert text.chat_apply(msgs, True, c["add_generation_prompt"]) == c["expected"], c["name"]


def test_chat_template_random_conversations(text, ot):
    rng = random.Random(7)
    pieces = ["ciao", "\n", "\n\n", "<think>", "</think>", "ragiono", " ", "4", "x\ny", "<|im_end|>", "è"]
    roles = ["system", "user", "assistant", "tool", "tool", "narrator"]
    for _ in range(400):
        msgs = [(rng.choice(roles), "".join(rng.choice(pieces) for _ in range(rng.randint(0, 6))))
                for _ in range(rng.randint(0, 6))]
        for mini in (True, False):
            for gen in (True, False):
                want = ot.apply_minicpm5(msgs, gen) if mini else ot.apply_generic(msgs, gen)
                assert text.chat_apply(msgs, mini, gen) == want, msgs


def test_chat_helpers(text, ot):
    assert text.direct_suffix() == "<think>\n\n</think>\n\n"
    assert text.thinking_on_suffix() == "<think>\n"
    for pre, name in [("minicpm5", ""), ("", "MiniCPM5-Q4"), ("qwen2", "llama"), ("", ""), ("x", "my-minicpm5.gguf")]:
        assert text.is_minicpm5(pre, name) == ot.is_minicpm5(pre, name)


# ---------------------------------------------------------------- Unicode tables
def _tables():
    src = open(os.path.join(ROOT, "pocket-workbench-android_b200", "csrc", "pk_unicode_tables.inc")).read()
    out = {}
    for name, body in re.findall(r"static const uint32_t (\w+)\[\]\[2\] = \{(.*?)\};", src, re.S):
        s = set()
        for lo, hi in re.findall(r"\{0x([0-9A-F]+), 0x([0-9A-F]+)\}", body):
            s.update(range(int(lo, 16), int(hi, 16) + 1))
        out[name] = s
    return out


def test_unicode_tables_match_the_standard(ot):
    import unicodedata

    t = _tables()
    cps = [c for c in range(0x110000) if not 0xD800 <= c <= 0xDFFF]
    assert t["kNumeric"] == {c for c in cps if unicodedata.category(chr(c)) in ("Nd", "Nl", "No")}
    assert t["kWhiteSpace"] == ot._WHITE_SPACE
    letters = {c for c in cps if ot.is_letter_category(chr(c))}
    assert letters <= t["kAlphabetic"]  # Alphabetic = L* + Nl + Other_Alphabetic
    extra = {unicodedata.category(chr(c)) for c in t["kAlphabetic"] - letters}
    assert extra <= {"Mn", "Mc", "So"}


# ---------------------------------------------------------------- patterns
def test_pattern_find_matches_oracle(text, ot):
    rng = random.Random(11)
    pats = [p for ps in ot.PRE.values() for p in ps] + [
        r"[\S]+", r"\p{P}+|x", r"a*", r"(?:ab|a)(?=b)", r"[^a-c\d]{2,}", r"\w+|.", r"(a|b)+?c", r"x{,2}y",
        r"[-a]+", r"[a-]+", r"\p{L}{2,3}|\s", r"(?!a)\S+"]
    for _ in range(150):
        t = rand_text(rng, rng.randint(0, 14))
        for p in pats:
            assert text.find(p, t) == ot.Pattern(p).find(t), (p, t)


def test_oracle_patterns_pinned_to_regex_module(ot):
    """The four presets' patterns, oracle against the `regex` engine: leftmost
    non-overlapping matches (none of these patterns can match empty)."""
    import regex

    rng = random.Random(5)
    for _ in range(200):
        t = rand_text(rng, rng.randint(1, 14)).replace("Ⅻ", "")
        for pre, ps in ot.PRE.items():
            for p in ps:
                want = [(m.start(), m.end()) for m in regex.finditer(p, t)]
                assert ot.Pattern(p).find(t) == want, (pre, p, t)


# ---------------------------------------------------------------- tokenizer
def _train(pre_patterns, corpus, vocab_size, specials):
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers, trainers

    ht = Tokenizer(models.BPE())
    ht.pre_tokenizer = pre_tokenizers.Sequence(
        [pre_tokenizers.Split(Regex(p), behavior="isolated") for p in pre_patterns]
        + [pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tr = trainers.BpeTrainer(vocab_size=vocab_size, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                             special_tokens=list(specials), show_progress=False)
    ht.train_from_iterator(corpus, tr)
    model = json.loads(ht.to_str())["model"]
    tokens = [None] * len(model["vocab"])
    for tok, i in model["vocab"].items():
        tokens[i] = tok
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    return tokens, merges


def _hf(pre_patterns, tokens, merges, ignore_merges):
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers

    vocab = {t: i for i, t in enumerate(tokens)}
    pairs = [tuple(m.split(" ", 1)) for m in merges]
    ht = Tokenizer(models.BPE(vocab=vocab, merges=pairs, ignore_merges=ignore_merges))
    ht.pre_tokenizer = pre_tokenizers.Sequence(
        [pre_tokenizers.Split(Regex(p), behavior="isolated") for p in pre_patterns]
        + [pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    return ht


SPECIALS = ["<|im_start|>", "<|im_end|>", "<s>", "<|endoftext|>"]


@pytest.fixture(scope="module")
def vocabs(tmp_path_factory, ot):
    """One trained byte-level BPE per preset, written as tokenizer-only GGUFs."""
    from pocketinfer import synth

    rng = random.Random(3)
    corpus = [rand_text(rng, 30) for _ in range(400)]
    d = tmp_path_factory.mktemp("tok")
    out = {}
    for pre in ("gpt-2", "llama3", "qwen2", "minicpm5"):
        tokens, merges = _train(ot.PRE[pre], corpus, 700, SPECIALS)
        types = [3 if t in SPECIALS else 1 for t in tokens]
        path = str(d / f"{pre}.gguf")
        synth.write_tokenizer_gguf(path, tokens, types, merges, pre=pre, bos=tokens.index("<s>"),
                                   eos=tokens.index("<|endoftext|>"))
        o = ot.Tokenizer([t.encode() for t in tokens], types, merges, pre=pre, bos=tokens.index("<s>"),
                         eos=tokens.index("<|endoftext|>"))
        out[pre] = (path, tokens, merges, o)
    return out


def test_oracle_tokenizer_pinned_to_hf_bpe(vocabs, ot):
    rng = random.Random(17)
    for pre, (_, tokens, merges, o) in vocabs.items():
        ht = _hf(ot.PRE[pre], tokens, merges, ignore_merges=(pre == "minicpm5"))
        for _ in range(60):
            t = rand_text(rng, rng.randint(1, 20))
            assert o.encode(t, parse_special=False) == ht.encode(t, add_special_tokens=False).ids, (pre, t)


@pytest.mark.parametrize("pre", ["gpt-2", "llama3", "qwen2", "minicpm5"])
def test_tokenizer_matches_oracle(text, vocabs, pre):
    path, tokens, _, o = vocabs[pre]
    tk = text.Tokenizer(path)
    info = tk.info
    assert info["n_vocab"] == len(tokens) and info["pre"] == pre
    assert info["ignore_merges"] == (pre == "minicpm5")
    assert info["bos_id"] == o.bos and info["eos_ids"] == o.eos
    rng = random.Random(23)
    for i in range(120):
        t = rand_text(rng, rng.randint(0, 20))
        if i % 3 == 0:  # special-token texts inside the prompt
            t = rng.choice(SPECIALS) + t + rng.choice(SPECIALS) + "<|im" + t[:5]
        for ps in (True, False):
            ids = tk.encode(t, ps)
            assert ids == o.encode(t, ps), (pre, ps, t)
            if not ps:  # byte-level BPE over all 256 bytes: the bytes come back
                assert tk.decode(ids) == t.encode()
    for tid in list(range(len(tokens))) + [len(tokens), 10**6]:
        assert tk.token_bytes(tid) == o.token_bytes(tid)
        assert tk.is_eog(tid) == o.is_eog(tid)


def test_tokenizer_corners(text, ot, tmp_path):
    """Reference corners: a repeated token keeps its first id, a repeated merge
    its last rank, merges with no space after the first byte are ignored, no
    token_type array means every token is normal, a symbol missing from the
    vocabulary falls back to its characters and then to the byte tokens, the
    whole-word lookup of ignore_merges, empty and malformed text."""
    from pocketinfer import PkError, synth

    enc, _ = ot.byte_map()
    base = [enc[b] for b in range(256)]
    tokens = base + ["ab", "abc", "ab", "ĠThe", "<|im_end|>", "Ġ", "xyz"]
    merges = ["a b", "ab c", "a b", " x", "Ġ T", "ĠT h", "ĠTh e", "y z", "x yz"]
    for pre in ("gpt-2", "minicpm5"):
        path = str(tmp_path / f"c-{pre}.gguf")
        synth.write_tokenizer_gguf(path, tokens, None, merges, pre=pre)
        tk = text.Tokenizer(path)
        o = ot.Tokenizer([t.encode() for t in tokens], None, merges, pre=pre)
        for t in ["abc ab The xyz", "", "ab", "aab abcabc", " The The", "<|im_end|>x", "xyzxyz"]:
            for ps in (True, False):
                assert tk.encode(t, ps) == o.encode(t, ps), (pre, t, ps)
        assert tk.info["eos_ids"] == []  # no token types: nothing is special
        with pytest.raises(PkError):
            from pocketinfer import lib
            import ctypes as C

            n = C.c_size_t()
            out = (C.c_uint32 * 8)()
            bad = b"ab\xff"
            if lib().pk_tokenize(tk.h, bad, len(bad), 1, C.cast(out, C.c_void_p), 8, C.byref(n)) != 0:
                raise PkError(1, "malformed")
    with pytest.raises(PkError):
        text.Tokenizer(str(tmp_path / "missing.gguf"))
    nometa = str(tmp_path / "nometa.gguf")
    synth.write_tokenizer_gguf(nometa, [], None)
    assert text.Tokenizer(nometa).encode("abc") == []


def test_long_runs(text, ot):
    """Runs of hundreds of thousands of letters, spaces or digits: the one-
    character repeats run as loops, so the matches (checked against the
    `regex` engine) come back without deep recursion, and a whole long text
    tokenizes."""
    import regex

    cases = [(ot.PRE["gpt-2"][0], "a" * 300000 + " b"), (r"\s+(?!\S)|\s+", " " * 200000 + "x"),
             (ot.PRE["minicpm5"][0], "7" * 30001), (ot.PRE["llama3"][0], "\n" * 50000 + "end " + "z" * 70000)]
    for pat, t in cases:
        assert text.find(pat, t) == [(m.start(), m.end()) for m in regex.finditer(pat, t)]


def test_long_text_tokenizes(text, vocabs):
    path, _, _, o = vocabs["gpt-2"]
    tk = text.Tokenizer(path)
    t = "x" * 100000 + " " * 100000 + "9" * 1000
    ids = tk.encode(t, False)
    assert tk.decode(ids) == t.encode()


def test_utf8_flush_matches_decoder(text):
    """flush_utf8 over token bytes cut at random points: after every piece, the
    text so far is Python's decoding (with replacement: one U+FFFD per maximal
    ill-formed part, as Rust's Utf8Error::error_len defines it) of all bytes
    but the held-back tail, and that tail is only a cut-off well-formed
    sequence ("unexpected end of data").  (Python's incremental decoder is not
    the pin: it also holds back ED A0..BF, which Rust reports at once.)"""
    rng = random.Random(29)
    pieces = [c.encode() for c in "aè中😀"] + [b"\x80", b"\xc0", b"\xc2", b"\xe2\x82", b"\xed\xa0\x80", b"\xf0\x80",
                                                b"\xf4\x90\x80\x80", b"\xff", b"\xe0\x9f\x80", b"\xf0\x9f"]
    for _ in range(300):
        data = b"".join(rng.choice(pieces) for _ in range(rng.randint(0, 30)))
        cuts = sorted(rng.sample(range(len(data) + 1), min(len(data) + 1, rng.randint(0, 6))))
        chunks = [data[a:b] for a, b in zip([0] + cuts, cuts + [len(data)])]
        st = text.Utf8Stream()
        got, seen = b"", b""
        for ch in chunks:
            got += st.feed(ch)
            seen += ch
            done = seen[: len(seen) - len(st.pending)]
            assert got == done.decode("utf-8", "replace").encode(), (data, chunks)
            if st.pending:
                assert len(st.pending) <= 3
                with pytest.raises(UnicodeDecodeError) as e:
                    st.pending.decode("utf-8")
                assert e.value.reason == "unexpected end of data"


@pytest.mark.parametrize("pre", ["minicpm5", "gpt-2"])
def test_chat_prompt_matches_bridge(text, ot, vocabs, pre):
    """A chat request's prompt ids (jni.rs:416-456): template, direct-answer
    suffix, and old turns dropped until the ids fit n_ctx - 1024 (the third
    turn first when the first is a system turn), or the request refused."""
    from pocketinfer import PkError

    path, _, _, o = vocabs[pre]
    tk = text.Tokenizer(path)
    rng = random.Random(31)
    roles = ["system", "user", "assistant", "user", "tool"]
    for i in range(150):
        msgs = [(rng.choice(roles) if j else rng.choice(["system", "user"]), rand_text(rng, rng.randint(1, 8)))
                for j in range(rng.randint(1, 7))]
        mini, direct = rng.random() < 0.7, rng.random() < 0.5
        n_ctx = rng.choice([1024 + rng.randint(0, 120), 500, 8192])
        try:
            want = ot.chat_prompt(o, msgs, mini, direct, n_ctx)
        except OverflowError:
            with pytest.raises(PkError) as e:
                text.chat_prompt(tk, msgs, mini, direct, n_ctx)
            assert e.value.code == 6  # PK_ERR_CONTEXT_FULL
            continue
        got = text.chat_prompt(tk, msgs, mini, direct, n_ctx)
        assert (got["ids"], got["dropped"], got["direct_applied"]) == want, (msgs, mini, direct, n_ctx)


def test_chat_messages_must_be_utf8(text, vocabs):
    import ctypes as C

    from pocketinfer import PkError, lib

    tk = text.Tokenizer(vocabs["gpt-2"][0])
    arr = (text.ChatMessage * 2)(text.ChatMessage(b"user", b"ciao"), text.ChatMessage(b"user", b"ab\xff"))
    n, d, f = C.c_size_t(), C.c_int(), C.c_int()
    out = (C.c_uint32 * 64)()
    assert lib().pk_chat_prompt(tk.h, C.cast(arr, C.c_void_p), 2, 1, 0, 8192, C.cast(out, C.c_void_p), 64,
                                C.byref(n), C.byref(d), C.byref(f)) == 1
    assert "UTF-8" in lib().pk_last_error().decode()
    buf = C.create_string_buffer(256)
    m = C.c_size_t()
    assert lib().pk_chat_apply(C.cast(arr, C.c_void_p), 2, 1, 1, C.cast(buf, C.c_void_p), 256, C.byref(m)) == 1
    assert lib().pk_chat_apply(C.cast(arr, C.c_void_p), 1, 1, 1, C.cast(buf, C.c_void_p), 256, C.byref(m)) == 0
    with pytest.raises(PkError):
        text.chat_prompt(tk, [("user", "x" * 50)], n_ctx=1024)  # no room at all: refused
