"""one Qwen2 decoder layer decode step through muyo_cuda_layer_step, against the
oracle's layer (oracle_qwen2_layer, the per-layer body of tools/reference_qwen2.py:109-157).

hidden 896, 14 query / 2 KV heads of 64, ffn 4864, F16 weights N(0,0.02), F32 QKV bias, eps 1e-6,
theta 1e6; the F16 KV cache (max 2048) holds 1023 seeded N(0,1) keys/values and the token is
decoded at position 1023. Tolerance 1e-3 * (1 + |e|) (BASELINE), checked tighter too.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_rel_close
from muyo_llm_b200 import _abi, engine, synth

pytestmark = pytest.mark.gpu
SEED = 3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def layer_case(kv_f16: bool, pos: int):
    cfg = synth.Qwen2Config(layers=1, vocab=8)
    t = synth.make_model(cfg, SEED)
    hd, S = cfg.head_dim, cfg.max_seq
    kv_np = np.float16 if kv_f16 else np.float32
    kc = np.zeros((cfg.kv_heads, S, hd), kv_np)
    vc = np.zeros((cfg.kv_heads, S, hd), kv_np)
    kc[:, :pos] = synth.normal_f32(SEED, "prefill.k", (cfg.kv_heads, pos, hd)).astype(kv_np)
    vc[:, :pos] = synth.normal_f32(SEED, "prefill.v", (cfg.kv_heads, pos, hd)).astype(kv_np)
    x = synth.normal_f32(SEED, "layer.x", (cfg.hidden,))
    return cfg, t, kc, vc, x


def run_layer_gpu(cfg, t, kc, vc, x, pos, kv_dtype):
    c = engine.config_struct(cfg, kv_dtype)
    p = "blk.0."
    wqkv = np.concatenate([t[p + "attn_q.weight"], t[p + "attn_k.weight"], t[p + "attn_v.weight"]])
    bqkv = np.concatenate([t[p + "attn_q.bias"], t[p + "attn_k.bias"], t[p + "attn_v.bias"]])
    keep = {n: dev(a) for n, a in {"attn_norm": t[p + "attn_norm.weight"], "wqkv": wqkv, "bqkv": bqkv,
                                    "wo": t[p + "attn_output.weight"], "ffn_norm": t[p + "ffn_norm.weight"],
                                    "wgate": t[p + "ffn_gate.weight"], "wup": t[p + "ffn_up.weight"],
                                    "wdown": t[p + "ffn_down.weight"]}.items()}
    w = _abi.LayerWeights(*[keep[n].data_ptr() for n in ("attn_norm", "wqkv", "bqkv", "wo", "ffn_norm", "wgate",
                                                          "wup", "wdown")])
    ws_bytes = _abi.lib().muyo_cuda_layer_workspace_size(c)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    kd, vd, xd = dev(kc), dev(vc), dev(x)
    out = torch.empty_like(xd)
    posd = dev(np.array([pos], np.int32))
    _abi.call("muyo_cuda_layer_step", c, w, kd.data_ptr(), vd.data_ptr(), posd.data_ptr(), xd.data_ptr(),
              out.data_ptr(), ws.data_ptr(), ws_bytes, None)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kd.cpu().numpy(), vd.cpu().numpy(), ws


@pytest.mark.parametrize("kv_f16,pos", [(True, 1023), (False, 1023), (True, 0), (True, 64), (True, 2047)])
def test_layer_step_matches_oracle(cuda, oracle_mod, kv_f16, pos):
    cfg, t, kc, vc, x = layer_case(kv_f16, pos)
    got, kd, vd, ws = run_layer_gpu(cfg, t, kc, vc, x, pos, _abi.KV_F16 if kv_f16 else _abi.KV_F32)
    om = oracle_mod.Qwen2(cfg, t, kv_f16=kv_f16)
    om.kcache[:] = kc.view(np.uint16).reshape(-1) if kv_f16 else kc.reshape(-1)
    om.vcache[:] = vc.view(np.uint16).reshape(-1) if kv_f16 else vc.reshape(-1)
    exp = om.layer(0, x, pos)
    assert_rel_close(got, exp, 1e-3, "layer output")
    assert_rel_close(got, exp, 1e-4, "layer output (tight)")
    # the appended row, and nothing else in the cache changed
    ek = om.kcache.view(np.float16 if kv_f16 else np.float32).reshape(kc.shape).astype(np.float32)
    ev = om.vcache.view(np.float16 if kv_f16 else np.float32).reshape(vc.shape).astype(np.float32)
    assert_rel_close(kd[:, pos].astype(np.float32), ek[:, pos], 2e-3, "appended key")
    assert_rel_close(vd[:, pos].astype(np.float32), ev[:, pos], 2e-3, "appended value")
    assert (np.delete(kd, pos, axis=1) == np.delete(kc, pos, axis=1)).all()
    assert (np.delete(vd, pos, axis=1) == np.delete(vc, pos, axis=1)).all()
    # the attention arrival counters are left at zero for the next call
    assert (ws[:4 * cfg.kv_heads].cpu().numpy() == 0).all()
