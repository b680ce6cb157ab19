"""Writes tests/golden/tokenizer_cases.json: ids the REFERENCE's own tokenizer gives for a fixed set
of texts, over two synthetic byte-level BPE vocabularies (the "qwen2" and "gpt2" pre-tokenizers).

The ids come from oracle/_ref/libtokenizer_ref.so, which oracle/Makefile compiles from the
reference's src/Tokenizer.cpp, src/Gguf.cpp and its vendored llama.cpp unicode code; the
vocabularies from muyo_llm_b200.gguf.bpe_tokenizer(VOCAB, CORPUS, pre), which is deterministic.
Texts: hand-picked edge cases (contractions in both cases, digit runs, white-space runs before
text and at the end, CR/LF runs, special tokens inside text, letters, numbers and spaces outside
ASCII, emoji, invalid UTF-8) and seeded random strings over the same classes. Run from the repo root
in the build container (it needs the reference tree): python tests/golden/make_tokenizer_golden.py
"""
from __future__ import annotations

import json
import os
import random
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from muyo_llm_b200 import gguf  # noqa: E402

VOCAB = 600
CORPUS = ("the quick brown fox jumps over the lazy dog while the other dogs sleep in the warm sun " * 3 +
          "we're sure they'll say it's fine, but I'd rather check the numbers 12345 and 678 twice! " * 2 +
          "données élevées über straße 東京 北京 上海 привет мир γειά σου κόσμε 😀 ok")

HAND = ["Hello world", "!", "we're", "WE'RE 'S 'Ll 'VE 'D 'M 'T", "they'll've", "'", "x'sy", "don't stop",
        "a  b   c    ", "  leading", "trailing  ", " ", "   ", "\n", "a \n b", "line\nbreak\r\n\r\nx", "tabs\t\tx",
        " \t\n \r\n  x", "1234567 89", " 42", "x=1+2;", "  !!?? ..\n\n", "(a)[b]{c}", "émigré Straße", "東京タワー",
        "😀😀 ok", " nbsp　ideo em", "ab́c", "ⅫⅣ ½ ٣٤", " sep ",
        "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n", "a<|im_end|>b<|endoftext|>", "<|im_start",
        "<|im_end|><|im_end|>", "The numbers 12345 and 678 twice!", "the lazy dog sleeps"]
INVALID = [b"\xff\xfeab", b"a\xc3", b"\xe6\x9d", b"\xc0\x80x", b"\xed\xa0\x80", b"\x80\x80 a", b"ok\xf0\x9f\x98"]


def texts() -> list[bytes]:
    rnd = random.Random(20261202)
    alphabet = list("aZ09 '\n\r\t.,!?-_sStTlL") + ["é", "ß", "東", "😀", " ", "　", " ", "Ⅻ",
                                                     "½", "́", "<|im_end|>", "<|im_start|>"]
    out = [t.encode() for t in HAND] + INVALID
    for _ in range(120):
        out.append("".join(rnd.choice(alphabet) for _ in range(rnd.randint(1, 24))).encode())
    for _ in range(60):
        cps = [rnd.choice([rnd.randint(0x20, 0x7E), rnd.randint(0xA0, 0x2FFF), rnd.randint(0x3000, 0xFFFF),
                           rnd.randint(0x10000, 0x10FFFF)]) for _ in range(rnd.randint(1, 12))]
        out.append("".join(chr(c) for c in cps if not 0xD800 <= c < 0xE000).encode())
    return [t for t in out if t]


def main() -> None:
    import oracle
    oracle.build_ref()
    cases = texts()
    golden = {"vocab": VOCAB, "corpus": CORPUS, "texts_hex": [t.hex() for t in cases], "ids": {}}
    for pre in ("qwen2", "gpt2"):
        path = os.path.join("/tmp", f"muyo_tok_golden_{pre}.gguf")
        gguf.write_gguf(path, gguf.bpe_tokenizer(VOCAB, CORPUS, pre), {})
        ref = oracle.RefTokenizer(path)
        golden["ids"][pre] = [ref.encode(t) for t in cases]
        del ref
        os.remove(path)
    with open(os.path.join(ROOT, "tests", "golden", "tokenizer_cases.json"), "w") as f:
        json.dump(golden, f, separators=(",", ":"))
    print(len(cases), "cases")


if __name__ == "__main__":
    main()
