"""The host tokenizer and chat framing (muyo_llm_b200/host/tokenizer.cpp) through the CLI's --tokenize
mode (src/Tokenize.cpp, src/main.cpp:209-226), against the reference's own tokenizer.

- Golden: ids the reference's src/Tokenizer.cpp gave (tests/golden/tokenizer_cases.json, written by
  tests/golden/make_tokenizer_golden.py) for 223 texts over two synthetic byte-level BPE vocabularies,
  one per pre-tokenizer ("qwen2", "gpt2"). Bit-exact ids.
- Live (build container only, where oracle/_ref holds the reference tokenizer): fresh seeded texts,
  the ChatML framing, and the code-point class table against llama.cpp's flags for all 0x110000
  code points.
All CPU: the tokenizer needs no device.
"""
from __future__ import annotations

import importlib
import importlib.util
import json
import os
import random
import re
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN
from muyo_llm_b200 import gguf

build_mod = importlib.import_module("muyo_llm_b200.build")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "muyo_llm_b200", "host")

with open(os.path.join(GOLDEN, "tokenizer_cases.json")) as f:
    CASES = json.load(f)
TEXTS = [bytes.fromhex(h) for h in CASES["texts_hex"]]


def _bin() -> str:
    build_mod.build()
    return build_mod.HOST_BIN


def _vocab_file(tmp_path, pre: str) -> str:
    path = str(tmp_path / f"tok_{pre}.gguf")
    gguf.write_gguf(path, gguf.bpe_tokenizer(CASES["vocab"], CASES["corpus"], pre), {})
    return path


def _tokenize(path: str, text: bytes) -> tuple[list[int] | None, subprocess.CompletedProcess]:
    r = subprocess.run([_bin(), "--tokenize", path, text], capture_output=True, timeout=60)
    m = re.search(rb"-> ?([0-9 ]*)\n", r.stdout)
    return ([int(v) for v in m.group(1).split()] if m else None), r


def _valid_utf8(b: bytes) -> bool:
    try:
        b.decode("utf-8")
        return True
    except UnicodeDecodeError:
        return False


def _ref_available() -> bool:
    oracle_dir = os.path.join(ROOT, "oracle")
    return os.path.exists(os.path.join(oracle_dir, "_ref", "libtokenizer_ref.so"))


def _oracle():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return oracle


def _ref(path: str):
    return _oracle().RefTokenizer(path)


def _decode(tokens: list[str], ids: list[int]) -> bytes:
    """Ids -> bytes through GPT-2's byte map (every vocabulary string here is valid UTF-8)."""
    inverse = {c: b for b, c in gguf.gpt2_byte_symbols()[1].items()}
    return bytes(inverse[c] for i in ids for c in tokens[i] if c in inverse)


@pytest.mark.parametrize("pre", ["qwen2", "gpt2"])
def test_golden_ids_match_reference_tokenizer(tmp_path, pre):
    path = _vocab_file(tmp_path, pre)
    tokens = gguf.bpe_tokenizer(CASES["vocab"], CASES["corpus"], pre)["tokenizer.ggml.tokens"]
    for text, want in zip(TEXTS, CASES["ids"][pre]):
        got, r = _tokenize(path, text)
        assert got == want, (pre, text, got, want, r.stderr[-300:])
        # The mode checks Decode(Encode(text)) == text. Bytes the split could not decode became
        # U+FFFD, and overlong forms their shortest encoding: those texts do not come back.
        if _decode(tokens, want) == text:
            assert r.returncode == 0, (text, r.stderr)
            assert b"anchor OK" in r.stdout and b"round-trip exact" in r.stdout
        else:
            assert not _valid_utf8(text)
            assert r.returncode == 1 and b"round-trip differs" in r.stderr


def test_pre_tokenizers_differ_where_the_rules_do():
    """Qwen2 gives each digit its own piece; GPT-2 keeps a digit run together, so the corpus's merges
    of "12345" apply only there."""
    q, g = CASES["ids"]["qwen2"], CASES["ids"]["gpt2"]
    i = TEXTS.index(b"1234567 89")
    assert len(q[i]) == 10 and len(g[i]) < len(q[i])


def test_special_tokens_and_chat_framing(tmp_path):
    path = _vocab_file(tmp_path, "qwen2")
    V = CASES["vocab"]
    eot, start, end = V - 3, V - 2, V - 1
    text = b"<|im_start|>system\nBe brief.<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    ids, r = _tokenize(path, text)
    assert r.returncode == 0, r.stderr
    assert ids[0] == start and ids.count(start) == 3 and ids.count(end) == 2 and eot not in ids
    # A broken marker is plain text.
    ids, _ = _tokenize(path, b"<|im_start")
    assert start not in ids


def test_tokenize_cli_errors(tmp_path):
    assert subprocess.run([_bin(), "--tokenize", "x.gguf"], capture_output=True).returncode == 2
    r = subprocess.run([_bin(), "--tokenize", str(tmp_path / "missing.gguf"), "hi"], capture_output=True)
    assert r.returncode == 1 and b"[fail]" in r.stderr
    path = str(tmp_path / "novocab.gguf")
    gguf.write_gguf(path, {"general.architecture": "qwen2"}, {})
    r = subprocess.run([_bin(), "--tokenize", path, "hi"], capture_output=True)
    assert r.returncode == 1 and b"tokenizer.ggml.tokens" in r.stderr


def test_unicode_class_table_is_the_generator_output():
    """unicode_classes.inc is what gen_unicode_classes.py writes (Unicode 15.1 L/N, White_Space)."""
    spec = importlib.util.spec_from_file_location("gen_unicode_classes", os.path.join(HOST, "gen_unicode_classes.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    want = np.array(gen.classes(), np.uint8)
    np.testing.assert_array_equal(_table_from_inc(), want)


def _table_from_inc() -> np.ndarray:
    src = open(os.path.join(HOST, "unicode_classes.inc")).read()
    body = {name: re.search(name + r"\[\d+\] = \{(.*?)\};", src, re.S).group(1) for name in ("kUniStart", "kUniClass")}
    starts = [int(v, 16) for v in re.findall(r"0x[0-9A-F]+", body["kUniStart"])]
    kinds = [int(v) for v in re.findall(r"\d+", body["kUniClass"])]
    assert len(starts) == len(kinds)
    out = np.zeros(0x110000, np.uint8)
    for i, (s, k) in enumerate(zip(starts, kinds)):
        out[s:starts[i + 1] if i + 1 < len(starts) else 0x110000] = k
    return out


@pytest.mark.skipif(not _ref_available(), reason="the reference tokenizer is built only where its tree is")
def test_unicode_classes_match_reference_flags():
    f = _oracle().RefTokenizer.unicode_flags()
    want = np.zeros(f.size, np.uint8)
    want[(f & 0x4) != 0] = 1
    want[(f & 0x2) != 0] = 2
    want[(f & 0x100) != 0] = 3
    got = _table_from_inc()
    diff = np.nonzero(got != want)[0]
    assert diff.size == 0, [hex(int(c)) for c in diff[:10]]


@pytest.mark.skipif(not _ref_available(), reason="the reference tokenizer is built only where its tree is")
@pytest.mark.parametrize("pre", ["qwen2", "gpt2"])
def test_fresh_texts_match_reference_live(tmp_path, pre):
    path = _vocab_file(tmp_path, pre)
    ref = _ref(path)
    rnd = random.Random(7 if pre == "qwen2" else 8)
    pool = list("abcXYZ019 '\n\r\t.,;!?") + ["é", "ß", "東", "\U0001F600", " ", "　",
                                            " ", "Ⅻ", "½", "́", "<|im_end|>", "٣"]
    for _ in range(60):
        text = "".join(rnd.choice(pool) for _ in range(rnd.randint(1, 40))).encode()
        got, _ = _tokenize(path, text)
        assert got == ref.encode(text), text
        assert ref.decode(got) == text
