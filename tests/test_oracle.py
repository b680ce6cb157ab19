"""Pins the C oracle (oracle/oracle.c) before it is trusted as the checker of the CUDA path.

1. The reference's own known-answer checks, with their inputs and tolerances: src/MatVec.cpp,
   src/ElementwiseAdd.cpp, src/GetRows.cpp, src/Argmax.cpp (exact), src/RmsNorm.cpp,
   src/Rope.cpp, src/Swiglu.cpp, src/SoftMax.cpp, src/Attention.cpp, src/KvCache.cpp,
   src/TransformerLayer.cpp (tolerances as written there). The expected values of the float checks
   are recomputed here in float64 from the same formulas.
2. Golden vectors from running the unmodified tools/reference_qwen2.py (tests/golden/make_golden.py):
   the tiny model's per-step greedy ids, step-0 intermediates and last logits, and the first steps
   of the Qwen2.5-0.5B-architecture fixture.
"""
from __future__ import annotations

import json
import math
import sys
import os

import numpy as np
import pytest

from conftest import GOLDEN, assert_rel_close
from muyo_llm_b200 import synth


def test_f16_roundtrip_matches_numpy(oracle_mod):
    x = np.random.default_rng(0).standard_normal(200000).astype(np.float32) * np.float32(300)
    x = np.concatenate([x, np.float32([0.0, -0.0, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 65504, 65519, 65520, 1e-10])])
    with np.errstate(over="ignore"):
        assert (oracle_mod.f2h(x) == x.astype(np.float16).view(np.uint16)).all()
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = np.isfinite(bits.view(np.float16))
    lib = oracle_mod.lib()
    got = np.array([lib.oracle_h2f(int(b)) for b in bits[finite][::97]], np.float32)
    assert (got == bits[finite][::97].view(np.float16).astype(np.float32)).all()


def test_matvec_known_answer(oracle_mod):
    # src/MatVec.cpp:68-80: W[r][c] = (c % 7) - 3, x[c] = (c % 5) - 2, 128 x 256, exact equality.
    rows, cols = 128, 256
    w = np.tile(((np.arange(cols) % 7) - 3).astype(np.float16), (rows, 1))
    x = ((np.arange(cols) % 5) - 2).astype(np.float32)
    exact = sum(((c % 7) - 3) * ((c % 5) - 2) for c in range(cols))
    y = oracle_mod.mat_vec_f16(w, x)
    assert (y == np.float32(exact)).all()


def test_add_known_answer(oracle_mod):
    # src/ElementwiseAdd.cpp:93-99,208: a = 0.5 i, b = 1 + 0.25 i, 1000 elements, exact.
    i = np.arange(1000, dtype=np.float32)
    a, b = np.float32(0.5) * i, np.float32(1.0) + np.float32(0.25) * i
    assert (oracle_mod.add(a, b) == a + b).all()


def test_get_rows_known_answer(oracle_mod):
    # src/GetRows.cpp:47-56,181: table[t][c] = (t % 5) - 2 + 0.001 c, token 7 (exact), here as F16 table.
    t = np.arange(1024)[:, None]
    c = np.arange(512)[None, :]
    table = ((t % 5) - 2 + np.float32(0.001) * c).astype(np.float32).astype(np.float16)
    assert (oracle_mod.get_rows_f16(table, 7) == table[7].astype(np.float32)).all()


def test_argmax_known_answer(oracle_mod):
    # src/Argmax.cpp:51-56,146: logits -1 + 0.001 i, [21] = 5 -> 21.
    x = (-1.0 + np.float32(0.001) * np.arange(32, dtype=np.float32)).astype(np.float32)
    x[21] = 5.0
    assert oracle_mod.argmax(x) == 21
    # Ties: the first index of the maximum (src/Sampler.cpp:35-41).
    y = np.zeros(100, np.float32)
    y[[17, 42, 99]] = 3.0
    assert oracle_mod.argmax(y) == 17


def test_rms_norm_known_answer(oracle_mod):
    # src/RmsNorm.cpp:60-72: x = ((r*512 + c) % 13) - 6, w = 0.5 + 0.001 (c % 11), eps 1e-6, tol 1e-4.
    r, c = np.meshgrid(np.arange(8), np.arange(512), indexing="ij")
    x = (((r * 512 + c) % 13) - 6).astype(np.float32)
    w = (np.float32(0.5) + np.float32(0.001) * (np.arange(512) % 11)).astype(np.float32)
    x64 = x.astype(np.float64)
    exp = x64 / np.sqrt((x64 ** 2).mean(axis=1, keepdims=True) + 1e-6) * w
    assert_rel_close(oracle_mod.rms_norm(x, w, 1e-6), exp, 1e-4, "rms_norm")


def test_rope_known_answer(oracle_mod):
    # src/Rope.cpp:41-64,191-204: 8 channels c - 3, pos 3, base 1e4, tol 1e-5.
    x = (np.arange(8) - 3).astype(np.float32)
    theta_scale = np.float32(10000.0) ** np.float32(-2.0 / 8)
    j = np.arange(4)
    theta = 3 * np.power(float(theta_scale), j)
    exp = np.concatenate([x[:4] * np.cos(theta) - x[4:] * np.sin(theta), x[:4] * np.sin(theta) + x[4:] * np.cos(theta)])
    assert_rel_close(oracle_mod.rope_neox(x[None], 3, float(theta_scale))[0], exp, 1e-5, "rope")


def test_swiglu_known_answer(oracle_mod):
    # src/Swiglu.cpp:63-67,187: g = 0.01 ((i % 17) - 8), u = 0.5 + 0.01 (i % 7), 600 elements, tol 1e-5.
    i = np.arange(600)
    g = (np.float32(0.01) * ((i % 17) - 8)).astype(np.float32)
    u = (np.float32(0.5) + np.float32(0.01) * (i % 7)).astype(np.float32)
    g64 = g.astype(np.float64)
    assert_rel_close(oracle_mod.swiglu(g, u), g64 / (1 + np.exp(-g64)) * u, 1e-5, "swiglu")


def test_soft_max_known_answer(oracle_mod):
    # src/SoftMax.cpp:51-55,164-183: (c % 9) - 4 over 64 columns, scale 1/8, tol 1e-5.
    x = ((np.arange(64) % 9) - 4).astype(np.float32)
    v = x.astype(np.float64) / 8
    e = np.exp(v - v.max())
    assert_rel_close(oracle_mod.soft_max(x[None], 0.125)[0], e / e.sum(), 1e-5, "soft_max")


def _ref_attention64(q, keys, values, scale):
    s = keys.astype(np.float64) @ q.astype(np.float64) * scale
    p = np.exp(s - s.max())
    p /= p.sum()
    return p @ values.astype(np.float64)


def test_attention_known_answer(oracle_mod):
    # src/Attention.cpp:79-105,254-286: hd 8, 16 keys, tol 1e-4.
    hd, n = 8, 16
    q = ((np.arange(hd) % 5) - 2).astype(np.float32)
    key, d = np.meshgrid(np.arange(n), np.arange(hd), indexing="ij")
    keys = (((key + d) % 3) - 1).astype(np.float32)
    values = (((key * 2 + d) % 7) - 3).astype(np.float32)
    got = oracle_mod.attention(q[None], keys[None], values[None], 1, 1, 1 / math.sqrt(hd))[0]
    assert_rel_close(got, _ref_attention64(q, keys, values, 1 / math.sqrt(hd)), 1e-4, "attention")


def test_kv_cache_known_answer(oracle_mod):
    # src/KvCache.cpp:98-102,356-406: hd 16, query (d % 5) - 2, token t key ((3t + d) % 5) - 2 roped at t,
    # value ((t + d) % 5) - 2, attention over t + 1 keys; tol 1e-4.
    hd = 16
    d = np.arange(hd)
    q = ((d % 5) - 2).astype(np.float32)
    theta_scale = float(np.float32(10000.0) ** np.float32(-2.0 / hd))
    keys, values = [], []
    for t in range(2):
        k = (((t * 3 + d) % 5) - 2).astype(np.float32)
        keys.append(oracle_mod.rope_neox(k[None], t, theta_scale)[0])
        values.append((((t + d) % 5) - 2).astype(np.float32))
        K, V = np.stack(keys), np.stack(values)
        got = oracle_mod.attention(q[None], K[None], V[None], 1, 1, 1 / math.sqrt(hd))[0]
        assert_rel_close(got, _ref_attention64(q, K, V, 1 / math.sqrt(hd)), 1e-4, f"kv_cache token {t}")


def test_transformer_layer_known_answer(oracle_mod):
    # src/TransformerLayer.cpp:257-286 inputs, 537-602 CPU sequence (single head, F32 weights), tol 1e-3.
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

    def gemv(w, x):
        return oracle_mod.mat_vec_f32(w, x, ncols=w.shape[1], rows=w.shape[0], batches=1, stride_a=w.shape[1],
                                      batch_stride_a=0, batch_stride_b=0, batch_stride_d=0)

    xn = oracle_mod.rms_norm(hidden, n1, 1e-6)
    q = gemv(wq, xn)
    qr = oracle_mod.rope_neox(q[None], 0, float(np.float32(10000.0) ** np.float32(-2.0 / H)))[0]
    probs = oracle_mod.soft_max(gemv(keys, qr)[None], 1.0 / 8)[0]
    attn = gemv(vt, probs)
    x1 = oracle_mod.add(hidden, gemv(wo, attn))
    xn2 = oracle_mod.rms_norm(x1, n2, 1e-6)
    out = oracle_mod.add(x1, gemv(wd, oracle_mod.swiglu(gemv(wg, xn2), gemv(wu, xn2))))

    # float64 restatement of the same sequence
    h64 = hidden.astype(np.float64)
    xn64 = h64 / np.sqrt((h64 ** 2).mean() + 1e-6) * n1
    s64 = keys @ (wq @ xn64) / 8
    p64 = np.exp(s64 - s64.max())
    p64 /= p64.sum()
    x164 = h64 + wo @ (vt @ p64)
    xn264 = x164 / np.sqrt((x164 ** 2).mean() + 1e-6) * n2
    g64, u64 = wg @ xn264, wu @ xn264
    exp = x164 + wd @ (g64 / (1 + np.exp(-g64)) * u64)
    assert_rel_close(out, exp, 1e-3, "transformer layer")


def test_qwen2_tiny_matches_reference_forward(oracle_mod):
    """Greedy ids, step-0 layer-0 intermediates and last logits of the unmodified
    tools/reference_qwen2.py on the seeded tiny model."""
    g = np.load(os.path.join(GOLDEN, "qwen2_tiny.npz"))
    cfg = synth.QWEN2_TINY
    model = synth.make_model(cfg, int(g["seed"]))
    m = oracle_mod.Qwen2(cfg, model)
    # layer-0 output at step 0 (REF_DUMP b0.out, tools/reference_qwen2.py:158-159)
    emb = model["token_embd.weight"][int(g["ids"][0])].astype(np.float32)
    assert (emb == g["dump_embedding"]).all()
    out0 = m.layer(0, emb, 0)
    assert_rel_close(out0, g["dump_b0_out"], 1e-5, "layer 0 output, step 0")
    m.reset()
    for step, tok in enumerate(g["ids"]):
        arg, logits = m.step(int(tok), step)
        assert arg == g["argmax"][step], f"step {step}"
        if step == 0:
            assert_rel_close(logits, g["dump_logits"], 1e-5, "step-0 logits")
    assert_rel_close(logits, g["last_logits"], 1e-5, "last logits")


@pytest.mark.skipif(not os.path.exists(os.path.join(GOLDEN, "qwen2_05b_greedy.json")), reason="fixture not generated")
def test_qwen2_05b_first_steps_match_reference(oracle_mod):
    """First 4 steps of the 0.5B-architecture golden: the reference's argmax and its printed top-5."""
    doc = json.load(open(os.path.join(GOLDEN, "qwen2_05b_greedy.json")))
    cfg = synth.QWEN2_05B
    model = synth.make_model(cfg, doc["seed"])
    oracle_mod.set_threads(os.cpu_count() or 1)
    m = oracle_mod.Qwen2(cfg, model)
    seq = doc["prompt"] + doc["generated"]
    for step in range(4):
        arg, logits = m.step(seq[step], step)
        assert arg == doc["reference_argmax"][step]
        top = doc["reference_top5_first_steps"][str(step)]
        for tid, val in top:
            assert abs(float(logits[tid]) - val) <= 1e-4 + 1e-3 * abs(val), (step, tid, logits[tid], val)


SAMPLER_CASES = [
    dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=7),
    dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=123),
    dict(temperature=0.5, top_k=1, top_p=0.95, repeat_penalty=1.3, repeat_last_n=-1, seed=5),
    dict(temperature=1.2, top_k=200, top_p=1.0, repeat_penalty=0.9, repeat_last_n=8, seed=2**63 + 11),
    dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.2, repeat_last_n=16, seed=1),
]


@pytest.mark.parametrize("case", range(len(SAMPLER_CASES)))
def test_sampler_restatement_matches_the_reference_sampler(oracle_mod, case):
    """oracle_sample (with its own mt19937_64) against the reference's Sampler compiled unmodified
    from src/Sampler.cpp (oracle/_ref): 40 consecutive draws, identical tokens and identical
    penalised / scaled logits. Logits are continuous random values (no exact ties, whose order
    std::partial_sort leaves unspecified); the history repeats tokens, so penalties compound."""
    if oracle_mod.build_ref() is None:
        pytest.skip("the reference sampler (oracle/_ref) is not built here")
    kw = SAMPLER_CASES[case]
    ours, ref = oracle_mod.Sampler(**kw), oracle_mod.RefSampler(**kw)
    rng = np.random.default_rng(1000 + case)
    vocab = 151936
    history = list(rng.integers(0, vocab, 20))
    history += history[:5]
    for step in range(40):
        logits = (rng.standard_normal(vocab) * 3).astype(np.float32)
        la, lb = logits.copy(), logits.copy()
        ta, tb = ours.sample(la, history), ref.sample(lb, history)
        assert ta == tb, (case, step, ta, tb)
        assert np.array_equal(la, lb)
        history.append(ta)


def test_sampler_restatement_matches_reference_fixtures(oracle_mod):
    """oracle_sample against tests/golden/sampler_cases.json, the reference's own Sampler's draws on
    the same seeded inputs (written by tests/golden/make_sampler_golden.py): every drawn id and the
    bits of the logits the sampler leaves behind, for 5 parameter sets x 40 consecutive draws. This
    pins the restatement where the reference tree (and so oracle/_ref) is absent."""
    import hashlib
    import json

    sys.path.insert(0, GOLDEN)
    import make_sampler_golden as msg

    doc = json.load(open(os.path.join(GOLDEN, "sampler_cases.json")))
    assert len(doc["cases"]) == len(msg.CASES)
    for c, case in enumerate(doc["cases"]):
        kw = dict(case["params"], seed=int(case["params"]["seed"]))
        assert kw == msg.CASES[c]
        ours = oracle_mod.Sampler(**kw)
        history, next_logits = msg.inputs(c)
        for step, (tok, digest) in enumerate(zip(case["tokens"], case["logits_sha256"])):
            logits = next_logits()
            t = ours.sample(logits, history)
            assert t == tok, (c, step, t, tok)
            assert hashlib.sha256(logits.tobytes()).hexdigest() == digest, (c, step)
            history.append(t)


def test_mt19937_64_known_answer(oracle_mod):
    """std::mt19937_64's standard check value: the 10000th output of a default-seeded (5489)
    engine is 9981545732273789042 (C++11 [rand.predef])."""
    import ctypes as C

    L = oracle_mod.lib()
    st = C.create_string_buffer(int(L.oracle_mt64_bytes()))
    L.oracle_mt64_seed(st, 5489)
    for _ in range(9999):
        L.oracle_mt64_next(st)
    assert L.oracle_mt64_next(st) == 9981545732273789042
