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


def test_layer_step_7b_class_matches_oracle(cuda, oracle_mod):
    """The same fused layer at a 7B-class shape (hidden 4096, ffn 14336, 32 query / 8 KV heads of 128,
    F16 cache with 1023 seeded keys/values, the token at position 1023): the kernels take their
    large-K paths (K split over warps, the attention merge over 16 chunks, head size 128)."""
    cfg = synth.Qwen2Config(layers=1, hidden=4096, ffn=14336, heads=32, kv_heads=8, vocab=8)
    pos = 1023
    t = synth.make_model(cfg, SEED)
    hd, S = cfg.head_dim, cfg.max_seq
    kc = np.zeros((cfg.kv_heads, S, hd), np.float16)
    vc = np.zeros((cfg.kv_heads, S, hd), np.float16)
    kc[:, :pos] = synth.normal_f32(SEED, "prefill.k", (cfg.kv_heads, pos, hd)).astype(np.float16)
    vc[:, :pos] = synth.normal_f32(SEED, "prefill.v", (cfg.kv_heads, pos, hd)).astype(np.float16)
    x = synth.normal_f32(SEED, "layer.x", (cfg.hidden,))
    got, kd, vd, _ = run_layer_gpu(cfg, t, kc, vc, x, pos, _abi.KV_F16)
    om = oracle_mod.Qwen2(cfg, t, kv_f16=True)
    om.kcache[:] = kc.view(np.uint16).reshape(-1)
    om.vcache[:] = vc.view(np.uint16).reshape(-1)
    exp = om.layer(0, x, pos)
    assert_rel_close(got, exp, 1e-3, "7B-class layer output")
    ek = om.kcache.view(np.float16).reshape(kc.shape).astype(np.float32)
    ev = om.vcache.view(np.float16).reshape(vc.shape).astype(np.float32)
    assert_rel_close(kd[:, pos].astype(np.float32), ek[:, pos], 2e-3, "appended key")
    assert_rel_close(vd[:, pos].astype(np.float32), ev[:, pos], 2e-3, "appended value")


def test_reference_layer_chain_matches_oracle(cuda, oracle_mod):
    """The reference's own --layer known answer (src/TransformerLayer.cpp:257-286 inputs: hidden 64, 8
    cached keys, ffn 128, F32 weights in small integer patterns, position 0) run as its 14 nodes
    through the op-level entry points: rms_norm, mat_vec_f32 (Q), rope_neox, mat_vec_f32 (scores),
    soft_max (1/8), mat_vec_f32 (values, transposed V), mat_vec_f32 (O), add, rms_norm, gate and up
    mat_vec_f32, swiglu, mat_vec_f32 (down), add. Compared with the oracle's restatement of the CPU
    sequence (:537-590) at the reference's tolerance, 1e-3 * (1 + |e|) (:602)."""
    from muyo_llm_b200 import nodes

    H, S, F = 64, 8, 128
    i = np.arange(H)
    hidden = ((i % 7) - 3).astype(np.float32)
    n1 = (np.float32(0.5) + np.float32(0.01) * (i % 5)).astype(np.float32)
    n2 = (np.float32(0.6) + np.float32(0.01) * (i % 3)).astype(np.float32)
    wq = ((np.arange(H * H) % 3) - 1).astype(np.float32).reshape(H, H)
    wo = (((np.arange(H * H) % 5) - 2) * 0.5).astype(np.float32).reshape(H, H)
    wg = ((np.arange(F * H) % 3) - 1).astype(np.float32).reshape(F, H)
    wu = ((np.arange(F * H) % 4) - 1).astype(np.float32).reshape(F, H)
    wd = (((np.arange(H * F) % 5) - 2) * 0.25).astype(np.float32).reshape(H, F)
    key, d = np.meshgrid(np.arange(S), np.arange(H), indexing="ij")
    keys = (((key + d) % 3) - 1).astype(np.float32)
    vt = (((key * 2 + d) % 7) - 3).astype(np.float32).T.copy()  # [H][S]

    # device chain
    def buf(n):
        return torch.empty(n, dtype=torch.float32, device="cuda")

    dh, dn1, dn2 = dev(hidden), dev(n1), dev(n2)
    xn, q, qr, sc, pr, att, o, x1, xn2, g, u, act, mlp, out = (buf(n) for n in (H, H, H, S, S, H, H, H, H, F, F, F,
                                                                                 H, H))
    pos = dev(np.array([0], np.int32))
    nodes.rms_norm(nodes.rms_norm_params(H, 1e-6), dh, dn1, xn)                       # PreNorm
    nodes.mat_vec_f32(nodes.mat_vec_params(H, H), dev(wq), xn, q)                    # QProj
    nodes.rope(nodes.rope_params(1, H, freq_base=10000.0), q, pos, qr)               # QRope
    nodes.mat_vec_f32(nodes.mat_vec_params(H, S), dev(keys), qr, sc)                 # AttnScores
    nodes.soft_max(nodes.soft_max_params(1, S, 1.0 / 8), sc, pr)                     # AttnWeights
    nodes.mat_vec_f32(nodes.mat_vec_params(S, H), dev(vt), pr, att)                  # AttnOut
    nodes.mat_vec_f32(nodes.mat_vec_params(H, H), dev(wo), att, o)                   # OProj
    nodes.add(nodes.add_params(H), dh, o, x1)                                        # Residual1
    nodes.rms_norm(nodes.rms_norm_params(H, 1e-6), x1, dn2, xn2)                     # PostNorm
    nodes.mat_vec_f32(nodes.mat_vec_params(H, F), dev(wg), xn2, g)                   # GateProj
    nodes.mat_vec_f32(nodes.mat_vec_params(H, F), dev(wu), xn2, u)                   # UpProj
    nodes.swiglu(nodes.swiglu_params(F), g, u, act)                                  # SwiGLU
    nodes.mat_vec_f32(nodes.mat_vec_params(F, H), dev(wd), act, mlp)                 # DownProj
    nodes.add(nodes.add_params(H), x1, mlp, out)                                     # Residual2
    torch.cuda.synchronize()

    # the oracle's restatement of the reference's CPU sequence
    def gemv(w, x):
        return oracle_mod.mat_vec_f32(w, x, ncols=w.shape[1], rows=w.shape[0], batches=1, stride_a=w.shape[1],
                                      batch_stride_a=0, batch_stride_b=0, batch_stride_d=0)

    exn = oracle_mod.rms_norm(hidden, n1, 1e-6)
    eqr = oracle_mod.rope_neox(gemv(wq, exn)[None], 0, float(np.float32(10000.0) ** np.float32(-2.0 / H)))[0]
    epr = oracle_mod.soft_max(gemv(keys, eqr)[None], 1.0 / 8)[0]
    ex1 = oracle_mod.add(hidden, gemv(wo, gemv(vt, epr)))
    exn2 = oracle_mod.rms_norm(ex1, n2, 1e-6)
    exp = oracle_mod.add(ex1, gemv(wd, oracle_mod.swiglu(gemv(wg, exn2), gemv(wu, exn2))))
    assert_rel_close(pr.cpu().numpy(), epr, 1e-5, "attention weights")
    assert_rel_close(out.cpu().numpy(), exp, 1e-3, "layer output (reference tolerance)")
