"""Whole-model decode (muyo_model_*, the RunFullModel engine) against the reference's numpy forward
and the oracle.

* Tiny Qwen2 (2 layers): per-step greedy ids and logits of the unmodified tools/reference_qwen2.py
  (tests/golden/qwen2_tiny.npz), F32 KV cache as the reference's.
* Qwen2.5-0.5B architecture: 32 seeded prompt ids, 256 greedy ids, F32 KV cache:
  bit-identical to the reference forward's ids (tests/golden/qwen2_05b_greedy.json). With the F16
  KV cache BASELINE names: bit-identical to the oracle's F16-cache greedy ids (same fixture), and the
  first steps' logits within 1e-3 of the oracle's.
* Engine behaviour: generate == step-by-step, chat-style continuation, reset, GGUF loading, errors.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, assert_rel_close
from muyo_llm_b200 import _abi, engine, gguf, synth

pytestmark = pytest.mark.gpu
FULL = os.path.join(GOLDEN, "qwen2_05b_greedy.json")


@pytest.fixture(scope="module")
def tiny():
    g = np.load(os.path.join(GOLDEN, "qwen2_tiny.npz"))
    return g, synth.make_model(synth.QWEN2_TINY, int(g["seed"]))


ENGINES = [engine.Qwen2Model.ENGINE_PERSISTENT, engine.Qwen2Model.ENGINE_GRAPH]


@pytest.mark.parametrize("eng", ENGINES)
def test_tiny_matches_reference_forward(cuda, tiny, eng):
    g, t = tiny
    m = engine.Qwen2Model(synth.QWEN2_TINY, t, kv_dtype=_abi.KV_F32, engine=eng)
    for step, tok in enumerate(g["ids"]):
        arg, logits = m.step(int(tok))
        assert arg == g["argmax"][step], f"step {step}"
        if step == 0:
            assert_rel_close(logits, g["dump_logits"], 1e-4, "step-0 logits")
    assert_rel_close(logits, g["last_logits"], 1e-4, "last logits")
    assert m.position == len(g["ids"])
    m.close()


@pytest.mark.parametrize("eng", ENGINES)
@pytest.mark.parametrize("kv_dtype", [_abi.KV_F32, _abi.KV_F16])
def test_generate_equals_stepwise(cuda, tiny, kv_dtype, eng):
    g, t = tiny
    m = engine.Qwen2Model(synth.QWEN2_TINY, t, kv_dtype=kv_dtype, engine=eng)
    prompt = [int(i) for i in g["ids"][:5]]
    gen = m.generate(prompt, 20)
    m.reset()
    assert m.position == 0
    seq = list(prompt)
    for s in range(len(prompt) + 20):
        nxt, _ = m.step(seq[s], want_logits=False)
        if s + 1 >= len(seq):
            seq.append(nxt)
    assert list(gen) == seq[len(prompt):len(prompt) + 20]
    # Chat-style continuation (src/FullModel.cpp:1229-1251): a second call appends to the live cache.
    # The first call feeds prompt + a (its last generated id included), so appending turn X must
    # equal one-shot decoding of prompt + a + X.
    m.reset()
    a = m.generate(prompt, 6)
    b = m.generate([7], 4)
    assert m.position == len(prompt) + 6 + 1 + 4
    m.reset()
    one_shot = m.generate(prompt + [int(i) for i in a] + [7], 4)
    assert list(b) == list(one_shot)
    m.close()


def test_gguf_load_matches_set_tensor(cuda, tiny, tmp_path):
    g, t = tiny
    path = str(tmp_path / "tiny.gguf")
    gguf.write_synthetic_qwen2(path, synth.QWEN2_TINY, int(g["seed"]))
    a = engine.Qwen2Model(synth.QWEN2_TINY, t, kv_dtype=_abi.KV_F32)
    b = engine.Qwen2Model(synth.QWEN2_TINY, gguf_path=path, kv_dtype=_abi.KV_F32)
    ids = [int(i) for i in g["ids"]]
    assert list(a.generate(ids, 10)) == list(b.generate(ids, 10))
    a.close()
    b.close()


def test_engine_errors(cuda, tiny):
    g, t = tiny
    cfg = synth.QWEN2_TINY
    m = engine.Qwen2Model(cfg, t, kv_dtype=_abi.KV_F16)
    with pytest.raises(_abi.MuyoError) as e:
        m.generate([1, 2, 3], cfg.max_seq)  # exceeds the cache
    assert e.value.rc == -6
    with pytest.raises(_abi.MuyoError) as e:
        m.step(cfg.vocab)
    assert e.value.rc == -1
    m.close()
    partial = dict(t)
    del partial["blk.1.ffn_down.weight"]
    with pytest.raises(_abi.MuyoError) as e:
        engine.Qwen2Model(cfg, partial, kv_dtype=_abi.KV_F16)
    assert "ffn_down" in str(e.value)
    bad = dict(t)
    bad["blk.0.attn_q.weight"] = t["blk.0.attn_q.weight"][:-1]
    with pytest.raises(_abi.MuyoError):
        engine.Qwen2Model(cfg, bad, kv_dtype=_abi.KV_F16)


@pytest.fixture(scope="module")
def full():
    doc = json.load(open(FULL))
    return doc, synth.make_model(synth.QWEN2_05B, doc["seed"])


@pytest.mark.skipif(not os.path.exists(FULL), reason="0.5B golden fixture not generated")
@pytest.mark.parametrize("eng", ENGINES)
def test_05b_greedy_bit_identical_to_reference(cuda, full, eng):
    doc, t = full
    m = engine.Qwen2Model(synth.QWEN2_05B, t, kv_dtype=_abi.KV_F32, engine=eng)
    gen = m.generate(doc["prompt"], doc["n_predict"])
    mism = [i for i, (a, b) in enumerate(zip(gen, doc["generated"])) if a != b]
    assert not mism, f"first mismatch at generated[{mism[0]}]: {gen[mism[0]]} vs {doc['generated'][mism[0]]}"
    m.close()


@pytest.mark.skipif(not os.path.exists(FULL), reason="0.5B golden fixture not generated")
@pytest.mark.parametrize("eng", ENGINES)
def test_05b_f16_cache(cuda, full, oracle_mod, eng):
    doc, t = full
    m = engine.Qwen2Model(synth.QWEN2_05B, t, kv_dtype=_abi.KV_F16, engine=eng)
    if "oracle_kv_f16_generated" in doc:
        gen = m.generate(doc["prompt"], doc["n_predict"])
        assert list(gen) == doc["oracle_kv_f16_generated"]
        m.reset()
    om = oracle_mod.Qwen2(synth.QWEN2_05B, t, kv_f16=True)
    oracle_mod.set_threads(os.cpu_count() or 1)
    for step in range(3):
        tok = doc["prompt"][step]
        arg, logits = m.step(tok)
        oarg, ologits = om.step(tok, step)
        assert arg == oarg
        assert_rel_close(logits, ologits, 1e-3, f"step {step} logits")
    m.close()


@pytest.mark.parametrize("kv_dtype", [_abi.KV_F32, _abi.KV_F16])
def test_engines_agree_on_05b_arch(cuda, kv_dtype):
    """Persistent and graph engines: identical greedy ids and near-identical logits on the 0.5B
    architecture (independent of the golden fixture)."""
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, 99)
    prompt = [int(i) for i in synth.prompt_ids(99, 12, cfg.vocab)]
    outs = []
    for eng in ENGINES:
        m = engine.Qwen2Model(cfg, t, kv_dtype=kv_dtype, engine=eng)
        gen = m.generate(prompt, 40)
        m.reset()
        _, logits = m.step(prompt[0])
        outs.append((list(gen), logits))
        m.close()
    assert outs[0][0] == outs[1][0]
    # The engines add their F32 partial sums in different orders (last-bit differences); with an F16
    # cache such a difference can flip the F16 rounding of a key or value. Each engine is held to 1e-3
    # of the oracle (test_05b_f16_cache), so two of them are within 2e-3 of each other.
    tol = 1e-4 if kv_dtype == _abi.KV_F32 else 2e-3
    assert_rel_close(outs[0][1], outs[1][1], tol, "step-0 logits, persistent vs graph")


@pytest.mark.parametrize("kv_dtype", [_abi.KV_F32, _abi.KV_F16])
def test_graph_engine_launch_options_are_bit_identical(cuda, tiny, kv_dtype):
    """Programmatic dependent launch, the L2 prefetch of later kernels' weights and the weight tiles
    copied to shared memory change when kernels start and where weights are read from, not what is
    computed: ids and logits of the graph engine with all three off and all three on are
    bit-identical, on the tiny model and on an 0.5B-architecture sequence of 81 positions (two
    64-key attention chunks, so the merge runs)."""
    g, t = tiny
    cfg = synth.QWEN2_05B
    big = synth.make_model(cfg, 20261201)
    for c, tensors, prompt, n in [(synth.QWEN2_TINY, t, [int(i) for i in g["ids"][:5]], 50),
                                  (cfg, big, synth.prompt_ids(20261201, 8, cfg.vocab), 72)]:
        runs = []
        for pdl in (False, True):
            m = engine.Qwen2Model(c, tensors, kv_dtype=kv_dtype, engine=engine.Qwen2Model.ENGINE_GRAPH, pdl=pdl,
                                  prefetch=pdl, smem_weights=pdl)
            ids = m.generate(prompt, n)
            _, logits = m.step(int(ids[-1]))
            runs.append((ids, logits))
            m.close()
        assert list(runs[0][0]) == list(runs[1][0])
        assert np.array_equal(runs[0][1], runs[1][1])
