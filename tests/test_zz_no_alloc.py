"""The workspace-free argmax (muyo_cuda_argmax_noalloc) against the workspace argmax.

muyo_cuda_argmax_noalloc serves callers that cannot give the library device memory. It keeps its
partials in a static device array instead of a caller workspace. These checks call both entry
points through the C-ABI on the same device inputs:
- the indices must be equal (argmax is compare-only, so the tolerance is zero);
- two noalloc calls in a row must both be right, so a partial left over from the first call cannot
  leak into the second;
- a call past the static array's limit must be refused before anything is launched.

This file is collected last so that the first noalloc call of a full run comes after every other
test. It must also pass when run alone in a fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from muyo_llm_b200 import _abi, nodes

pytestmark = pytest.mark.gpu
CHUNK = 8192  # logits per partial (one CTA of the argmax)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def argmax_noalloc(x, rows):
    p = nodes.argmax_params(x.numel() // rows, rows)
    d = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    _abi.call("muyo_cuda_argmax_noalloc", C.byref(p), _ptr(x), _ptr(d), None)
    return d


def argmax_workspace(x, rows):
    p = nodes.argmax_params(x.numel() // rows, rows)
    ws_bytes = nodes.argmax_workspace_size(p)
    ws = torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device="cuda")
    d = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    nodes.argmax(p, x, d, ws, ws_bytes)
    return d


def _randn(shape, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda", dtype=torch.float32)


def test_noalloc_limit_value(cuda):
    assert _abi.lib().muyo_cuda_argmax_noalloc_max_pairs() == 8192


@pytest.mark.parametrize("rows,cols", [(1, 151936), (1, 32), (7, 151936), (431, 151936), (1, CHUNK * 8192)])
def test_noalloc_matches_workspace_twice(cuda, rows, cols):
    """Two noalloc calls in a row on different inputs, each against the workspace argmax."""
    first = _randn((rows, cols), 1000 + rows)
    second = _randn((rows, cols), 2000 + rows)
    # Plant the maximum of the second input where the first input's maximum is not, so that a
    # partial left over from the first call would give a wrong index.
    first_idx = torch.argmax(first, dim=1)
    plant = (first_idx + cols // 2 + 1) % cols
    second[torch.arange(rows, device="cuda"), plant] = 50.0
    got1 = argmax_noalloc(first, rows)
    got2 = argmax_noalloc(second, rows)
    want1 = argmax_workspace(first, rows)
    want2 = argmax_workspace(second, rows)
    torch.cuda.synchronize()
    assert torch.equal(got1, want1)
    assert torch.equal(got2, want2)
    assert torch.equal(got2.long(), plant)


def test_noalloc_ties_and_back_to_back_on_one_stream(cuda):
    """Ties keep the first index; ten calls queued back to back on one stream all come out right."""
    x = torch.zeros(151936, device="cuda")
    x[torch.tensor([5000, 9000, 151000], device="cuda")] = 2.0
    assert int(argmax_noalloc(x, 1)[0]) == 5000
    base = _randn((3, 151936), 77)
    outs, wants = [], []
    for k in range(10):
        y = base.clone()
        y[:, (k * 13331) % 151936] = 9.0 + k
        outs.append(argmax_noalloc(y, 3))
        wants.append(argmax_workspace(y, 3))
    torch.cuda.synchronize()
    for got, want in zip(outs, wants):
        assert torch.equal(got, want)


def test_noalloc_rejects_past_the_limit(cuda):
    """8193 partials (one more than the static array holds) is refused; nothing is written."""
    rows, cols = 8193, CHUNK
    p = nodes.argmax_params(cols, rows)
    x = torch.zeros(1, device="cuda")  # never read: the call is rejected before any launch
    d = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    rc = _abi.lib().muyo_cuda_argmax_noalloc(C.byref(p), _ptr(x), _ptr(d), None)
    assert _abi.ERRORS.get(rc) == "MUYO_EINVAL"
    assert "exceeds the static scratch" in _abi.last_error()
    torch.cuda.synchronize()
    assert int(d[0]) == -7
    # The limit itself is accepted.
    ok = _randn((8192, CHUNK), 5)
    assert torch.equal(argmax_noalloc(ok, 8192), argmax_workspace(ok, 8192))
