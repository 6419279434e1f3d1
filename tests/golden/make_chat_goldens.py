"""Writes chat_template.json: the reference's own chat-template goldens,
read as text from rust/pocketinfer/tests/chat_template.rs of the reference
checkout (path as the first argument).  Each case: the messages passed to
apply_minicpm5(&msgs, true) and the string the test asserts, with Rust
string escapes decoded.  Run once where the reference is present; the JSON is
what the tests read."""
import json
import os
import re
import sys

ESC = {"n": "\n", "t": "\t", "r": "\r", '"': '"', "\\": "\\", "0": "\0"}


def rust_str(s: str) -> str:
    return re.sub(r"\\(.)", lambda m: ESC.get(m.group(1), m.group(1)), s)


def main(ref_root: str):
    src = open(os.path.join(ref_root, "rust/pocketinfer/tests/chat_template.rs"), encoding="utf-8").read()
    lit = r'"((?:[^"\\]|\\.)*)"'
    msg = re.compile(r"Message\s*\{\s*role:\s*" + lit + r"\.into\(\),\s*content:\s*" + lit + r"\.into\(\)\s*\}")
    block = re.compile(r"let msgs = vec!\[(.*?)\];\s*let got = apply_minicpm5\(&msgs, (true|false)\);\s*"
                       r"assert_eq!\(got, " + lit + r", " + lit + r"\);", re.S)
    cases = []
    for m in block.finditer(src):
        msgs = [[rust_str(r), rust_str(c)] for r, c in msg.findall(m.group(1))]
        cases.append({"name": rust_str(m.group(4)), "add_generation_prompt": m.group(2) == "true",
                      "messages": msgs, "expected": rust_str(m.group(3))})
    if not cases:
        raise SystemExit("no cases found")
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "chat_template.json")
    with open(out, "w", encoding="utf-8") as f:
        json.dump({"source": "rust/pocketinfer/tests/chat_template.rs", "cases": cases}, f, indent=1,
                  ensure_ascii=False)
    print(f"{len(cases)} cases -> {out}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_chat_goldens.py <reference checkout>")
    main(sys.argv[1])
