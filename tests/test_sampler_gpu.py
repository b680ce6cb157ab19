"""The device sampler (muyo_cuda_sample) against the oracle's restatement of Sampler::Sample
(oracle.c oracle_sample, itself pinned draw for draw to the reference's src/Sampler.cpp in
tests/test_oracle.py): the same seeded mt19937_64 stream, 40 consecutive draws per case, identical
tokens and bit-identical penalised / scaled logits. Weights use double exp on both sides; a 1-ulp
difference between the device's and the host library's exp could move a draw only if the running
sum met the nucleus or sample threshold within that ulp."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from muyo_llm_b200 import _abi

pytestmark = pytest.mark.gpu

# (vocab, sampler parameters, draws, history length). Vocabularies: Qwen2's 151936 (one cluster of
# 8 CTAs), ragged and tiny ones (CTAs with no ids), 256000 (the largest 8-CTA slice) and 300000 (a
# 16-CTA cluster). 700 draws cross two refills of the engine's 312 words.
CASES = [
    (151936, dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=7), 40, 20),
    (3000, dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=123), 40, 20),
    (151936, dict(temperature=0.5, top_k=1, top_p=0.95, repeat_penalty=1.3, repeat_last_n=-1, seed=5), 40, 20),
    (151936, dict(temperature=1.2, top_k=200, top_p=1.0, repeat_penalty=0.9, repeat_last_n=8, seed=2**63 + 11), 40, 20),
    (151936, dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.2, repeat_last_n=16, seed=1), 40, 20),
    (151936, dict(temperature=0.7, top_k=4096, top_p=0.99, repeat_penalty=1.05, repeat_last_n=32, seed=99), 40, 20),
    (1000, dict(temperature=1.0, top_k=0, top_p=1.0, repeat_penalty=1.0, repeat_last_n=64, seed=31), 700, 4),
    (3001, dict(temperature=0.9, top_k=100, top_p=0.8, repeat_penalty=1.5, repeat_last_n=-1, seed=8), 30, 3000),
    (5, dict(temperature=2.0, top_k=0, top_p=0.99, repeat_penalty=1.1, repeat_last_n=3, seed=4), 60, 10),
    (256000, dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=12), 12, 64),
    (300000, dict(temperature=0.6, top_k=500, top_p=0.9, repeat_penalty=1.2, repeat_last_n=128, seed=13), 8, 200),
    (300000, dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.2, repeat_last_n=128, seed=14), 8, 200),
    (151936, dict(temperature=1.0, top_k=1500, top_p=0.97, repeat_penalty=1.0, repeat_last_n=64, seed=15), 10, 20),
    (151936, dict(temperature=1.1, top_k=3000, top_p=0.9, repeat_penalty=1.1, repeat_last_n=64, seed=16), 10, 20),
]


def _params(kw):
    return _abi.SamplerParams(kw["temperature"], kw["top_k"], kw["top_p"], kw["repeat_penalty"], kw["repeat_last_n"],
                              0, kw["seed"])


@pytest.mark.parametrize("case", range(len(CASES)))
def test_device_sampler_matches_oracle(cuda, oracle_mod, case):
    vocab, kw, draws, n_hist = CASES[case]
    ours = oracle_mod.Sampler(**kw)
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    _abi.call("muyo_sampler_seed", C.c_void_p(state.data_ptr()), kw["seed"], None)
    p = _params(kw)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(2000 + case)
    history = list(rng.integers(0, vocab, n_hist))
    history += history[:5] + history[:2]  # repeated ids: penalised once per occurrence
    for step in range(draws):
        logits = (rng.standard_normal(vocab) * 3).astype(np.float32)
        dev = torch.from_numpy(logits.copy()).cuda()
        hd = torch.tensor(history, dtype=torch.int32, device="cuda")
        _abi.call("muyo_cuda_sample", C.byref(p), C.c_void_p(dev.data_ptr()), vocab, C.c_void_p(hd.data_ptr()),
                  len(history), C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), None)
        want = ours.sample(logits, history)
        torch.cuda.synchronize()
        assert int(tok.item()) == want, (case, step)
        assert np.array_equal(dev.cpu().numpy(), logits), (case, step)
        history.append(want)


@pytest.mark.parametrize("top_k", [64, 20])
@pytest.mark.parametrize("cluster", [8, 16])
def test_device_sampler_cluster_sizes_agree(cuda, oracle_mod, cluster, top_k):
    """A forced cluster of 8 or 16 CTAs (MuyoSamplerParams.cluster_ctas) splits the row differently
    and must draw the same ids and leave the same logits as the oracle. 50 ids share the maximum:
    with top-k 20 the cut falls inside the tie (the lowest indices are taken)."""
    vocab = 151936
    kw = dict(temperature=0.9, top_k=top_k, top_p=0.9, repeat_penalty=1.2, repeat_last_n=32, seed=21)
    ours = oracle_mod.Sampler(**kw)
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    _abi.call("muyo_sampler_seed", C.c_void_p(state.data_ptr()), kw["seed"], None)
    p = _params(kw)
    p.cluster_ctas = cluster
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(77)
    history = [int(i) for i in rng.integers(0, vocab, 40)]
    for step in range(16):
        logits = (rng.standard_normal(vocab) * 2).astype(np.float32)
        logits[rng.integers(0, vocab, 50)] = logits.max()  # ties at the top: the lower index first
        dev = torch.from_numpy(logits.copy()).cuda()
        hd = torch.tensor(history, dtype=torch.int32, device="cuda")
        _abi.call("muyo_cuda_sample", C.byref(p), C.c_void_p(dev.data_ptr()), vocab, C.c_void_p(hd.data_ptr()),
                  len(history), C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), None)
        want = ours.sample(logits, history)
        torch.cuda.synchronize()
        assert int(tok.item()) == want, (cluster, step)
        assert np.array_equal(dev.cpu().numpy(), logits), (cluster, step)
        history.append(want)


@pytest.mark.parametrize("shape", ["constant", "heavy_tail"])
def test_device_sampler_selection_fallbacks(cuda, oracle_mod, shape):
    """Logit rows that take the selection's slower exact paths. constant: every id ties, so more
    keys share the selected digit than rank 0 gathers, and the cut falls inside the tie (the k lowest
    ids). heavy_tail: -exp(N(0, 3^2)), whose top-k spans many octaves, so the one-octave pass-0
    filter counts too few keys and the full pass runs."""
    vocab = 151936
    kw = dict(temperature=0.7, top_k=40, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=3)
    ours = oracle_mod.Sampler(**kw)
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    _abi.call("muyo_sampler_seed", C.c_void_p(state.data_ptr()), kw["seed"], None)
    p = _params(kw)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(5)
    for step in range(12):
        if shape == "constant":
            logits = np.full(vocab, 0.25 * step - 1.0, np.float32)
        else:
            logits = (-np.exp(rng.standard_normal(vocab) * 3)).astype(np.float32)
        dev = torch.from_numpy(logits.copy()).cuda()
        _abi.call("muyo_cuda_sample", C.byref(p), C.c_void_p(dev.data_ptr()), vocab, None, 0,
                  C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), None)
        want = ours.sample(logits, [])
        torch.cuda.synchronize()
        assert int(tok.item()) == want, (shape, step)
        assert np.array_equal(dev.cpu().numpy(), logits), (shape, step)
        if shape == "constant":
            assert want < 40


def test_device_sampler_limits(cuda):
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    logits = torch.zeros(151936, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = _params(dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=0))
    rc = _abi.lib().muyo_cuda_sample(C.byref(p), C.c_void_p(logits.data_ptr()), 151936, None, 0,
                                     C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), None)
    assert _abi.ERRORS.get(rc) == "MUYO_EUNSUPPORTED"
