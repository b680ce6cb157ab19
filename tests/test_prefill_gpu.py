"""Batched prefill (muyo_model_set_option "prefill"; src/FullModel.cpp feeds a prompt one position
at a time, 1174-1181) and its projection GEMM (muyo_cuda_mat_mul_f16, ggml's mul_mm:
shaders/llama/mul_mm.comp).

* GEMM: against a float64 evaluation of the same F16 weights and F32 activations, at shapes with
  ragged rows, positions and K, and with the BIAS and ACCUMULATE epilogues. Bar: |y - exact| <=
  1e-5 * sum_k |w x| + 1e-6 (the activations enter as two F16 halves, F32 accumulation).
* Model: prefill on against the one-position-at-a-time path: the same generated ids and next-step
  logits within 1e-3 (BASELINE's float tolerance), for one-pass and multi-pass prompts and a chat
  continuation; on the 0.5B architecture, the reference forward's 256 greedy ids bit for bit.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, assert_rel_close
from muyo_llm_b200 import _abi, engine, synth

pytestmark = pytest.mark.gpu


def _mat_mul(w, x, flags=0, bias=None, y0=None):
    N, K = w.shape
    T = x.shape[0]
    p = _abi.MatMulParams(K, N, T, 0, 0, flags)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    yd = torch.from_numpy(y0.copy()).cuda() if y0 is not None else torch.zeros(T, N, device="cuda")
    bd = torch.from_numpy(bias).cuda() if bias is not None else None
    wsb = int(_abi.lib().muyo_cuda_mat_mul_f16_workspace_size(C.byref(p)))
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    _abi.call("muyo_cuda_mat_mul_f16", C.byref(p), C.c_void_p(wd.data_ptr()), C.c_void_p(xd.data_ptr()),
              C.c_void_p(yd.data_ptr()), C.c_void_p(bd.data_ptr() if bd is not None else 0),
              C.c_void_p(ws.data_ptr()), wsb, None)
    torch.cuda.synchronize()
    return yd.cpu().numpy()


@pytest.mark.parametrize("kernel", ["mma_sync", "tcgen05"])
@pytest.mark.parametrize("N,K,T", [(128, 256, 1), (1152, 896, 32), (897, 904, 65), (64, 4864, 128), (200, 8, 3),
                                   (896, 4864, 100)])
def test_mat_mul_f16_against_float64(cuda, N, K, T, kernel):
    rng = np.random.default_rng(N * 7 + K + T)
    w = (rng.uniform(-1, 1, (N, K)) * 0.05).astype(np.float16)
    x = rng.standard_normal((T, K)).astype(np.float32)
    exact = x.astype(np.float64) @ w.astype(np.float64).T
    bound = 1e-5 * (np.abs(x).astype(np.float64) @ np.abs(w.astype(np.float64)).T) + 1e-6
    f = _abi.MATMUL_TCGEN05 if kernel == "tcgen05" else 0
    y = _mat_mul(w, x, f)
    assert np.all(np.abs(y - exact) <= bound)
    b = rng.standard_normal(N).astype(np.float32)
    yb = _mat_mul(w, x, f | _abi.MATMUL_BIAS, bias=b)
    assert np.all(np.abs(yb - (exact + b)) <= bound + 1e-6 * np.abs(b))
    y0 = rng.standard_normal((T, N)).astype(np.float32)
    ya = _mat_mul(w, x, f | _abi.MATMUL_ACCUMULATE, y0=y0)
    assert np.all(np.abs(ya - (exact + y0)) <= bound + 1e-6 * np.abs(y0))


def _model(cfg, t, kv, prefill, tc=False, positions=None):
    m = engine.Qwen2Model(cfg, t, kv_dtype=kv, engine=engine.Qwen2Model.ENGINE_GRAPH)
    if positions:
        _abi.call("muyo_model_set_option", m._m, b"prefill_positions", positions)
    if prefill:
        _abi.call("muyo_model_set_option", m._m, b"prefill", 1)
    # 0: the mma.sync kernel for every projection, 1: tcgen05 for every one, 2 (default): per GEMM
    _abi.call("muyo_model_set_option", m._m, b"prefill_tc", 1 if tc is True else 2 if tc == "auto" else 0)
    return m


@pytest.mark.parametrize("kv", [_abi.KV_F32, _abi.KV_F16])
def test_prefill_matches_stepwise_tiny(cuda, kv):
    cfg = synth.QWEN2_TINY
    t = synth.make_model(cfg, 20261203)
    prompt = [int(i) for i in synth.prompt_ids(9, 40, cfg.vocab)]
    runs = []
    for prefill in (False, True):
        m = _model(cfg, t, kv, prefill)
        a = list(m.generate(prompt, 8))
        b = list(m.generate([5, 6, 7], 6))  # chat-style continuation: the second prompt starts at 48
        _, logits = m.step(int(b[-1]))
        runs.append((a, b, logits, m.position))
        m.close()
    assert runs[0][0] == runs[1][0] and runs[0][1] == runs[1][1]
    assert runs[0][3] == runs[1][3]
    assert_rel_close(runs[1][2], runs[0][2], 1e-3, "logits after the turns, prefill vs stepwise")


def test_prefill_multi_pass_05b_arch(cuda):
    """A 300-position prompt: three prefill passes (128 + 128 + 43 positions), the later ones
    attending to the cache written by the earlier ones."""
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, 31)
    prompt = [int(i) for i in synth.prompt_ids(31, 300, cfg.vocab)]
    out = []
    for prefill in (False, True):
        m = _model(cfg, t, _abi.KV_F16, prefill, positions=128 if prefill else None)
        ids = list(m.generate(prompt, 12))
        _, logits = m.step(ids[-1])
        out.append((ids, logits))
        m.close()
    assert out[0][0] == out[1][0]
    assert_rel_close(out[1][1], out[0][1], 1e-3, "logits after a 300-position prompt")


@pytest.mark.parametrize("tc", [False, True, "auto"])
def test_prefill_512_position_passes_05b_arch(cuda, tc):
    """Option "prefill_positions" = 512: a 700-position prompt in two passes (512 + 187), on either
    GEMM kernel, against one decode step per position."""
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, 33)
    prompt = [int(i) for i in synth.prompt_ids(33, 700, cfg.vocab)]
    out = []
    for prefill in (False, True):
        m = _model(cfg, t, _abi.KV_F16, prefill, tc and prefill, 512 if prefill else None)
        ids = list(m.generate(prompt, 8))
        _, logits = m.step(ids[-1])
        out.append((ids, logits))
        m.close()
    assert out[0][0] == out[1][0]
    assert_rel_close(out[1][1], out[0][1], 1e-3, "logits after a 700-position prompt")


def test_prefill_positions_option_checks(cuda):
    cfg = synth.QWEN2_TINY
    m = engine.Qwen2Model(cfg, synth.make_model(cfg, 1), kv_dtype=_abi.KV_F32)
    for bad in (0, 64, 200, 2048):
        with pytest.raises(_abi.MuyoError):
            _abi.call("muyo_model_set_option", m._m, b"prefill_positions", bad)
    _abi.call("muyo_model_set_option", m._m, b"prefill", 1)
    with pytest.raises(_abi.MuyoError):  # after the activations are allocated
        _abi.call("muyo_model_set_option", m._m, b"prefill_positions", 256)
    m.close()


FULL = os.path.join(GOLDEN, "qwen2_05b_greedy.json")


@pytest.mark.skipif(not os.path.exists(FULL), reason="0.5B golden fixture not generated")
@pytest.mark.parametrize("tc", [False, True, "auto"])
def test_prefill_05b_greedy_bit_identical_to_reference(cuda, tc):
    """With either GEMM kernel (mma.sync, tcgen05) behind the prefill projections, or the default
    choice per GEMM."""
    g = json.load(open(FULL))
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, int(g["seed"]))
    m = _model(cfg, t, _abi.KV_F32, True, tc)
    ids = list(m.generate([int(i) for i in g["prompt"]], len(g["generated"])))
    m.close()
    assert ids == [int(i) for i in g["generated"]]
