"""CPU checks of the C-ABI library: it builds, loads without a GPU, exports every symbol that
include/muyo_cuda.h declares, and validates arguments on the host before any CUDA call (so these
calls never touch a device)."""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import ROOT
from muyo_llm_b200 import _abi, build, engine, nodes, synth

HEADER = os.path.join(ROOT, "include", "muyo_cuda.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(muyo_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    build()
    return _abi.lib()


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.lib_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (muyo_\w+)", out))
    declared = declared_symbols()
    assert declared, "no declarations parsed"
    assert declared <= exported, f"declared but not exported: {sorted(declared - exported)}"
    assert declared == set(_abi.SIGNATURES), f"binding drift: {sorted(declared ^ set(_abi.SIGNATURES))}"


def test_version(lib):
    assert lib.muyo_cuda_version().decode().endswith("sm_100a")


def expect(rc_expected, fn, *args, match=None):
    rc = getattr(_abi.lib(), fn)(*args)
    assert rc == rc_expected, (fn, rc, _abi.last_error())
    if match:
        assert match in _abi.last_error(), _abi.last_error()


def test_validation_before_any_cuda_call(lib):
    p = nodes.mat_vec_params(64, 8)
    expect(-1, "muyo_cuda_mat_vec_f16", C.byref(p), None, None, None, None, None, None, match="null")
    p = nodes.mat_vec_params(64, 8, fusion_flags=_abi.MATVEC_SCALE0)
    expect(-5, "muyo_cuda_mat_vec_f16", C.byref(p), 16, 16, 16, None, None, None, match="SCALE")
    p = nodes.mat_vec_params(64, 8, fusion_flags=_abi.MATVEC_BIAS0)
    expect(-1, "muyo_cuda_mat_vec_f16", C.byref(p), 16, 16, 16, None, None, None, match="BIAS0")
    p = nodes.mat_vec_params(64, 9, stride_d=8)
    expect(-1, "muyo_cuda_mat_vec_f32", C.byref(p), 16, 16, 16, None, None, None, match="stride_d")
    g = nodes.argmax_params(100000)
    expect(-1, "muyo_cuda_argmax", C.byref(g), 16, 16, None, 0, None, match="workspace")
    a = nodes.attention_params(14, 2, 48, 2048)
    expect(-5, "muyo_cuda_attention_decode", C.byref(a), 16, 16, 16, None, 16, 16, 1 << 20, None, match="head_dim")
    a = nodes.attention_params(14, 3, 64, 2048)
    expect(-1, "muyo_cuda_attention_decode", C.byref(a), 16, 16, 16, None, 16, 16, 1 << 20, None)
    r = nodes.rope_params(2, 64)
    r.rope_mode = 8
    expect(-1, "muyo_cuda_rope", C.byref(r), 16, 16, None, 16, None, match="mode")
    s = nodes.soft_max_params(2, 64, 1.0)
    s.KY = 2
    expect(-1, "muyo_cuda_soft_max", C.byref(s), 16, None, None, 32, None, match="mask")


def test_model_config_validation(lib):
    bad = engine.config_struct(synth.Qwen2Config(hidden=900, heads=14), _abi.KV_F16)
    h = C.c_void_p()
    expect(-1, "muyo_model_create", C.byref(bad), 0, C.byref(h), match="divisible")
    bad = engine.config_struct(synth.Qwen2Config(heads=14, kv_heads=3), _abi.KV_F16)
    expect(-1, "muyo_model_create", C.byref(bad), 0, C.byref(h))
    bad = engine.config_struct(synth.QWEN2_05B, 7)
    expect(-1, "muyo_model_create", C.byref(bad), 0, C.byref(h), match="kv_dtype")


def test_workspace_sizes(lib):
    c = engine.config_struct(synth.QWEN2_05B, _abi.KV_F16)
    n = lib.muyo_cuda_layer_workspace_size(C.byref(c))
    cfg = synth.QWEN2_05B
    assert n >= 4 * (cfg.q_dim + 2 * cfg.kv_dim + cfg.q_dim + cfg.hidden + cfg.ffn)
    a = nodes.attention_params(14, 2, 64, 2048)
    assert lib.muyo_cuda_attention_workspace_size(C.byref(a)) == 2 * 32 * 7 * 66 * 4
    assert lib.muyo_cuda_argmax_workspace_size(C.byref(nodes.argmax_params(151936))) == 19 * 8
