"""The C++ host (muyo_llm_b200/host): the reference's Run<Op>() checks and CLI modes
(src/main.cpp:186-431) on the B200 kernels, with the reference's exit codes (0 ok, 1 failed, 2 usage).

CPU: the binary builds and answers usage errors and unsupported options with 2 before touching a
device. GPU: every op mode passes its known-answer check, and --forward on a synthetic tiny Qwen2
GGUF continues the reference forward's greedy pick and agrees with the Python engine."""
from __future__ import annotations

import importlib
import os
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


@pytest.mark.parametrize("args", [[], ["--nope"], ["--forward"], ["--gguf", "x.gguf"], ["--tokenize", "a", "b"]])
def test_usage_exit_code(args):
    assert _run(*args).returncode == 2


def test_forward_rejects_unsupported_options_before_any_device_work(tmp_path):
    path = str(tmp_path / "missing.gguf")
    r = _run("--forward", path, "-p", "hello")
    assert r.returncode == 2 and "tokenizer" in r.stderr
    r = _run("--forward", path, "--tokens", "1,2", "--chat")
    assert r.returncode == 2
    r = _run("--forward", path, "--tokens", "1,2", "--bogus")
    assert r.returncode == 2


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
    got = [int(v) for v in r.stdout.strip().split(",")]
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
    got = [int(v) for v in r.stdout.strip().split(",")]
    m = engine.Qwen2Model(synth.QWEN2_TINY, gguf_path=path, kv_dtype=_abi.KV_F32)
    m.set_sampler(temperature=0.9, top_k=30, top_p=0.9, repeat_penalty=1.2, seed=42)
    assert got == list(m.generate(ids, 16))
    m.close()
