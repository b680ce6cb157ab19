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

CASES = [
    (151936, dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1, repeat_last_n=64, seed=7)),
    (3000, dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=123)),
    (151936, dict(temperature=0.5, top_k=1, top_p=0.95, repeat_penalty=1.3, repeat_last_n=-1, seed=5)),
    (151936, dict(temperature=1.2, top_k=200, top_p=1.0, repeat_penalty=0.9, repeat_last_n=8, seed=2**63 + 11)),
    (151936, dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.2, repeat_last_n=16, seed=1)),
    (151936, dict(temperature=0.7, top_k=4096, top_p=0.99, repeat_penalty=1.05, repeat_last_n=32, seed=99)),
]


def _params(kw):
    return _abi.SamplerParams(kw["temperature"], kw["top_k"], kw["top_p"], kw["repeat_penalty"], kw["repeat_last_n"],
                              0, kw["seed"])


@pytest.mark.parametrize("case", range(len(CASES)))
def test_device_sampler_matches_oracle(cuda, oracle_mod, case):
    vocab, kw = CASES[case]
    ours = oracle_mod.Sampler(**kw)
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    _abi.call("muyo_sampler_seed", C.c_void_p(state.data_ptr()), kw["seed"], None)
    p = _params(kw)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(2000 + case)
    history = list(rng.integers(0, vocab, 20))
    history += history[:5]
    for step in range(40):
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


def test_device_sampler_limits(cuda):
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    logits = torch.zeros(151936, dtype=torch.float32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = _params(dict(temperature=1.0, top_k=0, top_p=0.9, repeat_penalty=1.0, repeat_last_n=64, seed=0))
    rc = _abi.lib().muyo_cuda_sample(C.byref(p), C.c_void_p(logits.data_ptr()), 151936, None, 0,
                                     C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), None)
    assert _abi.ERRORS.get(rc) == "MUYO_EUNSUPPORTED"
