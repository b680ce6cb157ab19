"""Non-greedy decoding inside the step graph (muyo_model_set_sampler) against the reference's
RunFullModel loop (src/FullModel.cpp:1058-1116, 1174-1202): feed a turn's ids, then per generated
id one Sampler::Sample draw on that position's logits with every cached id as history.

A model with the sampler decodes two turns. A second model without it replays the same ids one
step at a time (muyo_model_step), which yields the logits each draw saw: the kernels and their
order are the same and deterministic, so these logits are bit-identical. The oracle's Sampler, seeded alike
and drawing only at generated positions, must then pick every generated id exactly.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from muyo_llm_b200 import _abi, engine, synth

pytestmark = pytest.mark.gpu

CASES = [
    dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=7),
    dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=123),
    dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.3, repeat_last_n=16, seed=1),
    dict(temperature=1.5, top_k=200, top_p=0.5, repeat_penalty=0.9, repeat_last_n=-1, seed=2**63 + 5),
]


def _replay(cfg, tensors, kv_dtype, fed):
    """Logits after each position of `fed`, from step-by-step decoding without a sampler."""
    m = engine.Qwen2Model(cfg, tensors, kv_dtype=kv_dtype, engine=engine.Qwen2Model.ENGINE_GRAPH)
    out = [m.step(int(t))[1] for t in fed]
    m.close()
    return out


def _check_turns(cfg, tensors, kv_dtype, kw, turns, oracle_mod):
    m = engine.Qwen2Model(cfg, tensors, kv_dtype=kv_dtype, engine=engine.Qwen2Model.ENGINE_GRAPH)
    m.set_sampler(**kw)
    fed, draw_at = [], []
    for prompt, n in turns:
        gen = [int(i) for i in m.generate(prompt, n)]
        fed += list(prompt)
        draw_at += range(len(fed), len(fed) + n)
        fed += gen
    assert m.position == len(fed)
    m.close()
    logits = _replay(cfg, tensors, kv_dtype, fed)
    ours = oracle_mod.Sampler(**kw)
    for n in draw_at:
        want = ours.sample(logits[n - 1].copy(), fed[:n])
        assert fed[n] == want, (kw, n)
    return fed


@pytest.mark.parametrize("case", range(len(CASES)))
def test_sampled_generate_matches_reference_loop_tiny(cuda, oracle_mod, case):
    cfg = synth.QWEN2_TINY
    t = synth.make_model(cfg, 20261202)
    p = [int(i) for i in synth.prompt_ids(5, 6, cfg.vocab)]
    _check_turns(cfg, t, _abi.KV_F32, CASES[case], [(p, 14), ([7, 9], 10)], oracle_mod)


def test_sampled_generate_matches_reference_loop_05b_arch(cuda, oracle_mod):
    """Full 151936-entry vocabulary: the top-k radix select over the LM head's logits in the graph."""
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, 77)
    p = [int(i) for i in synth.prompt_ids(77, 8, cfg.vocab)]
    fed = _check_turns(cfg, t, _abi.KV_F16, CASES[0], [(p, 20), (p[:3], 8)], oracle_mod)
    assert len(set(fed[8:28])) > 1


def test_sampler_settings(cuda):
    cfg = synth.QWEN2_TINY
    t = synth.make_model(cfg, 3)
    p = [1, 2, 3, 4]
    m = engine.Qwen2Model(cfg, t, kv_dtype=_abi.KV_F32, engine=engine.Qwen2Model.ENGINE_GRAPH)
    greedy = list(m.generate(p, 12))
    m.reset()
    m.set_sampler(temperature=1.0, top_k=0, top_p=1.0, seed=11)
    first = list(m.generate(p, 12))
    m.reset()
    m.set_sampler(temperature=1.0, top_k=0, top_p=1.0, seed=11)  # re-seeding repeats the draws
    assert list(m.generate(p, 12)) == first
    m.reset()
    m.set_sampler()  # the reference's defaults: the greedy pick
    assert list(m.generate(p, 12)) == greedy
    m.close()
    # the persistent kernel has no sampler node
    m = engine.Qwen2Model(cfg, t, kv_dtype=_abi.KV_F32, engine=engine.Qwen2Model.ENGINE_PERSISTENT)
    m.set_sampler(temperature=0.7, seed=1)
    with pytest.raises(_abi.MuyoError) as e:
        m.generate(p, 4)
    assert _abi.ERRORS.get(e.value.rc) == "MUYO_EUNSUPPORTED"
    m.close()


def test_sampler_limits_on_model(cuda):
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, 1)
    m = engine.Qwen2Model(cfg, t, kv_dtype=_abi.KV_F16, engine=engine.Qwen2Model.ENGINE_GRAPH)
    with pytest.raises(_abi.MuyoError) as e:
        m.set_sampler(temperature=1.0, top_k=0)  # 151936 candidates: more than the device sampler's 4096
    assert _abi.ERRORS.get(e.value.rc) == "MUYO_EUNSUPPORTED"
    assert len(m.generate([1, 2], 3)) == 3  # the model stays usable (greedy)
    m.close()
