"""Parity of the split-K GQA decode attention and the KV append (C-ABI) with the oracle.

The attention is checked against oracle_attention (src/Attention.cpp:254-285 generalised to GQA) on
caches filled with seeded N(0,1) keys/values, F32 and F16 caches (the F16 cache is fed to the oracle
rounded, as the GPU stores it), over key counts that hit every chunking edge. The append is checked
against the numpy reference's rotation (tools/reference_qwen2.py:84-93, evaluated in float64 and
rounded once, restated below).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import assert_rel_close
from muyo_llm_b200 import _abi, nodes, synth

pytestmark = pytest.mark.gpu
SEED = 11


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rope_f64(x, pos, base):
    """tools/reference_qwen2.py:84-93 (x [heads][hd] F32; float64 rotation, one rounding)."""
    hd = x.shape[-1]
    half = hd // 2
    j = np.arange(half)
    theta = pos * (base ** (-2.0 * j / hd))
    c, s = np.cos(theta), np.sin(theta)
    out = np.empty_like(x)
    out[:, :half] = x[:, :half] * c - x[:, half:] * s
    out[:, half:] = x[:, :half] * s + x[:, half:] * c
    return out


@pytest.mark.parametrize("kv_dtype", [_abi.KV_F32, _abi.KV_F16])
@pytest.mark.parametrize("heads,kv_heads,hd", [(14, 2, 64), (8, 8, 128), (4, 1, 32), (2, 2, 16)])
@pytest.mark.parametrize("n_keys", [1, 2, 63, 64, 65, 300, 1024, 2048])
def test_attention_decode(cuda, oracle_mod, kv_dtype, heads, kv_heads, hd, n_keys):
    S = 2048
    K = synth.normal_f32(SEED, f"K{kv_heads}{hd}", (kv_heads, S, hd))
    V = synth.normal_f32(SEED, f"V{kv_heads}{hd}", (kv_heads, S, hd))
    q = synth.normal_f32(SEED, f"q{heads}{hd}{n_keys}", (heads, hd))
    if kv_dtype == _abi.KV_F16:
        Kd, Vd = K.astype(np.float16), V.astype(np.float16)
        K, V = Kd.astype(np.float32), Vd.astype(np.float32)
    else:
        Kd, Vd = K, V
    p = nodes.attention_params(heads, kv_heads, hd, S, n_keys=n_keys, kv_dtype=kv_dtype)
    ws_bytes = nodes.attention_workspace_size(p)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(heads * hd, dtype=torch.float32, device="cuda")
    nodes.attention_decode(p, dev(q), dev(Kd), dev(Vd), out, ws, ws_bytes)
    exp = oracle_mod.attention(q, K[:, :n_keys], V[:, :n_keys], heads, kv_heads, 1.0 / math.sqrt(hd))
    assert_rel_close(host(out).reshape(heads, hd), exp, 1e-4, f"attention n={n_keys}")


def test_attention_device_position(cuda, oracle_mod):
    heads, kv_heads, hd, S = 14, 2, 64, 512
    K = synth.normal_f32(SEED, "Kp", (kv_heads, S, hd))
    V = synth.normal_f32(SEED, "Vp", (kv_heads, S, hd))
    q = synth.normal_f32(SEED, "qp", (heads, hd))
    p = nodes.attention_params(heads, kv_heads, hd, S, kv_dtype=_abi.KV_F32)
    ws_bytes = nodes.attention_workspace_size(p)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    Kd, Vd, qd = dev(K), dev(V), dev(q)
    for pos in (0, 100, 511):
        out = torch.empty(heads * hd, dtype=torch.float32, device="cuda")
        nodes.attention_decode(p, qd, Kd, Vd, out, ws, ws_bytes, pos=dev(np.array([pos], np.int32)))
        exp = oracle_mod.attention(q, K[:, :pos + 1], V[:, :pos + 1], heads, kv_heads, 0.125)
        assert_rel_close(host(out).reshape(heads, hd), exp, 1e-4, f"pos {pos}")


@pytest.mark.parametrize("kv_dtype", [_abi.KV_F32, _abi.KV_F16])
@pytest.mark.parametrize("pos", [0, 1, 1023, 2047])
def test_kv_append(cuda, kv_dtype, pos):
    kv_heads, hd, S, base = 2, 64, 2048, 1e6
    k = synth.normal_f32(SEED, f"ka{pos}", (kv_heads, hd))
    v = synth.normal_f32(SEED, f"va{pos}", (kv_heads, hd))
    dt = torch.float16 if kv_dtype == _abi.KV_F16 else torch.float32
    kc = torch.zeros(kv_heads * S * hd, dtype=dt, device="cuda")
    vc = torch.zeros(kv_heads * S * hd, dtype=dt, device="cuda")
    p = nodes.attention_params(14, kv_heads, hd, S, kv_dtype=kv_dtype)
    nodes.kv_append(p, base, dev(k), dev(v), kc, vc, dev(np.array([pos], np.int32)))
    kh = host(kc.float()).reshape(kv_heads, S, hd)
    vh = host(vc.float()).reshape(kv_heads, S, hd)
    ek = rope_f64(k, pos, base)
    if kv_dtype == _abi.KV_F16:
        ek, ev = ek.astype(np.float16).astype(np.float32), v.astype(np.float16).astype(np.float32)
    else:
        ev = v
    assert_rel_close(kh[:, pos], ek, 1e-6, "appended key")
    assert (vh[:, pos] == ev).all()
    assert (np.delete(kh, pos, axis=1) == 0).all() and (np.delete(vh, pos, axis=1) == 0).all()
