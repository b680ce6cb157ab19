"""The C++ host (muyo_llm_b200/host): the reference's Run<Op>() checks and CLI modes
(src/main.cpp:186-431) on the B200 kernels, with the reference's exit codes (0 ok, 1 failed, 2 usage).

CPU: the binary builds and answers usage errors with 2 and a missing file with 1 before touching a
device. GPU: every op mode passes its known-answer check; --forward on a synthetic tiny Qwen2 GGUF
continues the reference forward's greedy pick and agrees with the Python engine; with a byte-level
BPE vocabulary in the file, a text prompt, a ChatML turn (--chat) and interactive turns (-i) give the
engine's ids over the tokenizer's prompt ids, cut after the end-of-sequence id, and print their text.
"""
from __future__ import annotations

import dataclasses
import importlib
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN
from muyo_llm_b200 import _abi, engine, gguf, synth

build_mod = importlib.import_module("muyo_llm_b200.build")  # the package re-exports build() by name


def _bin() -> str:
    build_mod.build()
    assert os.path.exists(build_mod.HOST_BIN)
    return build_mod.HOST_BIN


def _run(*args, timeout=300):
    return subprocess.run([_bin(), *args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("args", [[], ["--nope"], ["--forward"], ["--gguf", "x.gguf"], ["--tokenize", "a"]])
def test_usage_exit_code(args):
    assert _run(*args).returncode == 2


def test_forward_option_errors_before_any_device_work(tmp_path):
    path = str(tmp_path / "missing.gguf")
    r = _run("--forward", path, "-p", "hello")
    assert r.returncode == 1 and "[fail]" in r.stderr
    r = _run("--forward", path, "--tokens", "1,2", "--chat")
    assert r.returncode == 1
    r = _run("--forward", path, "--tokens", "1,2", "--bogus")
    assert r.returncode == 2


def _generated(stderr: str) -> list[int]:
    """The ids of "[forward] generated N tokens: a b c" (src/FullModel.cpp:1273-1278)."""
    # The last such line; an interactive session's "[chat] you> " prompt precedes it on its line.
    line = re.findall(r"\[forward\] generated \d+ tokens:([ 0-9]*)", stderr)[-1]
    return [int(v) for v in line.split()]


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["--add", "--matvec", "--rmsnorm", "--rope", "--swiglu", "--getrows", "--argmax",
                                  "--softmax", "--attention", "--kvcache", "--layer"])
def test_op_mode_passes_on_gpu(cuda, mode):
    r = _run(mode)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MISMATCH" not in r.stdout


@pytest.mark.gpu
def test_forward_on_tiny_gguf(cuda, tmp_path):
    g = np.load(os.path.join(GOLDEN, "qwen2_tiny.npz"))
    path = str(tmp_path / "tiny.gguf")
    gguf.write_synthetic_qwen2(path, synth.QWEN2_TINY, int(g["seed"]))
    ids = [int(i) for i in g["ids"]]
    r = _run("--forward", path, "--tokens", ",".join(map(str, ids)), "-n", "12")
    assert r.returncode == 0, r.stderr
    got = _generated(r.stderr)
    assert got[0] == int(g["argmax"][-1])  # the reference forward's pick after the last prompt id
    m = engine.Qwen2Model(synth.QWEN2_TINY, gguf_path=path, kv_dtype=_abi.KV_F32)
    assert got == list(m.generate(ids, 12))
    m.close()


@pytest.mark.gpu
def test_forward_sampled_on_tiny_gguf(cuda, tmp_path):
    """--temp / --top-k / --top-p / --repeat-penalty / --seed (src/main.cpp:372-394) drive the device
    sampler: the CLI's ids equal the engine's with the same SamplerParams."""
    path = str(tmp_path / "tiny.gguf")
    gguf.write_synthetic_qwen2(path, synth.QWEN2_TINY, 4)
    ids = [3, 1, 4, 1, 5]
    flags = ["--temp", "0.9", "--top-k", "30", "--top-p", "0.9", "--repeat-penalty", "1.2", "--seed", "42"]
    r = _run("--forward", path, "--tokens", ",".join(map(str, ids)), "-n", "16", *flags)
    assert r.returncode == 0, r.stderr
    got = _generated(r.stderr)
    m = engine.Qwen2Model(synth.QWEN2_TINY, gguf_path=path, kv_dtype=_abi.KV_F32)
    m.set_sampler(temperature=0.9, top_k=30, top_p=0.9, repeat_penalty=1.2, seed=42)
    assert got == list(m.generate(ids, 16))
    m.close()


CORPUS = "the quick brown fox jumps over the lazy dog while the other dogs sleep in the warm sun " * 4
SYSTEM = "You are Qwen, created by Alibaba Cloud. You are a helpful assistant."


def _tok_model(tmp_path, seed=4, eos=None):
    tok = gguf.bpe_tokenizer(synth.QWEN2_TINY.vocab, CORPUS, "qwen2")
    if eos is not None:
        tok["tokenizer.ggml.eos_token_id"] = int(eos)
    path = str(tmp_path / f"tok_{eos}.gguf")
    gguf.write_synthetic_qwen2(path, synth.QWEN2_TINY, seed, tokenizer=tok)
    return path, tok


def _encode(path, text: str) -> list[int]:
    r = _run("--tokenize", path, text)
    line = [ln for ln in r.stdout.splitlines() if "->" in ln][0]
    return [int(v) for v in line.split("->", 1)[1].split()]


def _stdout(tok, turns) -> bytes:
    """What the run prints (src/FullModel.cpp:1068-1091, 1190-1198, 1248-1270): each non-special
    id's bytes, held back while a UTF-8 character is incomplete; a newline before every turn after
    the first, and one at the end after the held-back bytes."""
    inverse = {c: b for b, c in gguf.gpt2_byte_symbols()[1].items()}
    special = {i for i, t in enumerate(tok["tokenizer.ggml.token_type"]) if t in (3, 4)}
    out, pending = bytearray(), bytearray()

    def flush(final):
        done = 0
        while done < len(pending):
            lead = pending[done]
            n = 2 if lead & 0xE0 == 0xC0 else 3 if lead & 0xF0 == 0xE0 else 4 if lead & 0xF8 == 0xF0 else 1
            if not final and done + n > len(pending):
                break
            done += n
        out.extend(pending[:done])
        del pending[:done]

    for k, ids in enumerate(turns):
        if k:
            out.extend(b"\n")
        for i in ids:
            if i not in special:
                pending.extend(inverse[c] for c in tok["tokenizer.ggml.tokens"][i] if c in inverse)
                flush(False)
    flush(True)
    return bytes(out + b"\n")


def _run_bytes(*args, stdin=b""):
    r = subprocess.run([_bin(), *args], input=stdin, capture_output=True, timeout=300)
    return r.returncode, r.stdout, r.stderr.decode("utf-8", "replace")


def _cut(ids, eos):
    ids = list(ids)
    return ids[:ids.index(eos) + 1] if eos in ids else ids


def _engine(path):
    # The tiny file says 64 positions; a ChatML turn in its small vocabulary is longer, so the engine
    # gets the CLI's room (results do not depend on the cache capacity).
    cfg = dataclasses.replace(synth.QWEN2_TINY, max_seq=512)
    return engine.Qwen2Model(cfg, gguf_path=path, kv_dtype=_abi.KV_F32)


@pytest.mark.gpu
def test_forward_text_prompt_stops_at_eos(cuda, tmp_path):
    """-p TEXT: the prompt ids are the tokenizer's, the reply is the engine's greedy ids cut after
    tokenizer.ggml.eos_token_id (here an id the greedy run reaches), and stdout is their text."""
    path, tok = _tok_model(tmp_path)
    prompt = _encode(path, "the lazy dog")
    m = _engine(path)
    full = [int(v) for v in m.generate(prompt, 12)]
    m.close()
    # An end id the run never reaches: all 12 ids. The last id that is new in the run: cut there.
    absent = next(i for i in range(synth.QWEN2_TINY.vocab - 1, -1, -1) if i not in full)
    k = max(i for i in range(len(full)) if full[i] not in full[:i])
    for eos, want in ((absent, full), (full[k], full[:k + 1])):
        path2, tok2 = _tok_model(tmp_path, eos=eos)
        rc, out, err = _run_bytes("--forward", path2, "-p", "the lazy dog", "-n", "12")
        assert rc == 0, err
        assert "[forward] prompt tokens: " + " ".join(map(str, prompt)) in err
        assert _generated(err) == want
        assert out == _stdout(tok2, [want])


@pytest.mark.gpu
@pytest.mark.parametrize("sampled", [False, True])
def test_chat_turn_and_interactive_turns(cuda, tmp_path, sampled):
    """--chat: one ChatML turn (default system prompt) in one generate call. -i: the same first turn
    stepped one position per call (device sampler per step when sampling), then a second turn
    appended after the first reply's ids, as the engine gives over the whole history."""
    path, tok = _tok_model(tmp_path)
    eos = tok["tokenizer.ggml.eos_token_id"]
    flags = ["--temp", "0.8", "--top-k", "20", "--seed", "11"] if sampled else []
    turn1 = _encode(path, f"<|im_start|>system\n{SYSTEM}<|im_end|>\n<|im_start|>user\nhello<|im_end|>\n"
                          "<|im_start|>assistant\n")
    rc, out, err = _run_bytes("--forward", path, "--chat", "-p", "hello", "-n", "10", *flags)
    assert rc == 0, err
    chat_ids = _generated(err)
    m = _engine(path)
    if sampled:
        m.set_sampler(temperature=0.8, top_k=20, seed=11)
    want1 = _cut(m.generate(turn1, 10), eos)
    assert chat_ids == want1
    assert out == _stdout(tok, [want1])

    rc, out, err = _run_bytes("--forward", path, "-i", "-p", "hello", "-n", "10", *flags,
                              stdin=b"how are you\n/exit\n")
    assert rc == 0, err
    assert err.count("[chat] you> ") == 2
    turn2 = _encode(path, "\n<|im_start|>user\nhow are you<|im_end|>\n<|im_start|>assistant\n")
    if not sampled:  # the greedy history replayed from an empty cache gives the same ids
        m.reset()
        want2 = _cut(m.generate(turn1 + want1 + turn2, 10), eos)
    else:  # the engine's sampler stream continues across calls, as the session's does
        m.reset()
        m.set_sampler(temperature=0.8, top_k=20, seed=11)
        assert _cut(m.generate(turn1, len(want1)), eos) == want1
        want2 = _cut(m.generate(turn2, 10), eos)
    m.close()
    assert _generated(err) == want2
    assert out == _stdout(tok, [want1, want2])
