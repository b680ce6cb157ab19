"""Kernel sweeps of the op-level entry points: the F16 GEMV at the decode and 7B-class shapes, and
the norm / elementwise / argmax ops at decode shapes (latency) and at multi-row shapes whose traffic
is several times L2 (bandwidth). Each result is one dict: algorithmic bytes per call, the mean
device time per call (CUDA events over back-to-back calls on one stream, after warm-up) and the
achieved GB/s.

Every GEMV case rotates through enough weight copies that the bytes touched between two reads of
the same copy exceed L2 (126 MB). The multi-row op cases move more than 4x L2 per call, so no call
finds its operands in L2.
"""
from __future__ import annotations

import math

import torch

from . import nodes

L2_BYTES = 126 * 1024 * 1024

GEMV_SHAPES = [  # (rows, cols): config 1, the 0.5B decode projections and LM head, 7B-class shapes
    (128, 256), (896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896),
    (4096, 4096), (14336, 4096), (128256, 4096),
]


def _time_calls(fn, n_buf: int, iters: int, warmup: int = 3) -> float:
    """Mean milliseconds per call of fn(i) over `iters` calls, i rotating over n_buf buffers."""
    for i in range(max(warmup, 3)):
        fn(i % n_buf)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i % n_buf)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _result(name, shape, alg_bytes, ms, peak_gbs, **extra):
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    r = {"kernel": name, "shape": shape, "alg_bytes": int(alg_bytes), "us": ms * 1e3, "GB_s": gbs,
         "frac_of_peak": gbs / peak_gbs}
    r.update(extra)
    return r


def gemv(shapes=None, iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7):
    """muyo_cuda_mat_vec_f16 on W [rows][cols] F16 U[-1,1], x U[-1,1]: y = W x."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for rows, cols in shapes or GEMV_SHAPES:
        wbytes = rows * cols * 2
        n_buf = max(1, math.ceil(4 * L2_BYTES / wbytes)) if wbytes < 4 * L2_BYTES else 1
        W = [torch.rand(rows * cols, generator=g, device="cuda").mul_(2).sub_(1).half() for _ in range(n_buf)]
        x = torch.rand(cols, generator=g, device="cuda").mul_(2).sub_(1)
        y = torch.empty(rows, device="cuda")
        p = nodes.mat_vec_params(cols, rows)
        n = iters or max(20, 4 * n_buf)
        ms = _time_calls(lambda i: nodes.mat_vec_f16(p, W[i], x, y), n_buf, n)
        alg = wbytes + cols * 4 + rows * 4
        out.append(_result("k_mat_vec_f16", f"{rows}x{cols}", alg, ms, peak_gbs, weight_copies=n_buf, calls=n))
        del W
        torch.cuda.empty_cache()
    return out


def ops(iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7):
    """Decode-shape latency and multi-row bandwidth of rms_norm, add, swiglu and argmax, plus the
    decode-only ops (rope, soft_max, get_rows) at their decode shapes."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device="cuda")

    out = []
    # rms_norm: rows x n, weight n; in + out + weight bytes
    for rows, n, mode in [(1, 896, "latency"), (8, 512, "latency"), (16384, 4096, "bandwidth")]:
        x, w, d = randn(rows * n), randn(n), torch.empty(rows * n, device="cuda")
        p = nodes.rms_norm_params(n, 1e-6, rows)
        ms = _time_calls(lambda i: nodes.rms_norm(p, x, w, d), 1, iters or (50 if mode == "bandwidth" else 200))
        out.append(_result("k_rms_norm", f"{rows}x{n}", 2 * rows * n * 4 + n * 4, ms, peak_gbs, mode=mode))
    # add: three n-element arrays
    for n, mode in [(896, "latency"), (64 * 1024 * 1024, "bandwidth")]:
        a, b, d = randn(n), randn(n), torch.empty(n, device="cuda")
        p = nodes.add_params(n)
        ms = _time_calls(lambda i: nodes.add(p, a, b, d), 1, iters or (50 if mode == "bandwidth" else 200))
        out.append(_result("k_add_contig", f"{n}", 3 * n * 4, ms, peak_gbs, mode=mode))
    # swiglu: gate, up, out
    for rows, n, mode in [(1, 4864, "latency"), (4096, 14336, "bandwidth")]:
        a, b, d = randn(rows * n), randn(rows * n), torch.empty(rows * n, device="cuda")
        p = nodes.swiglu_params(n, rows)
        ms = _time_calls(lambda i: nodes.swiglu(p, a, b, d), 1, iters or (50 if mode == "bandwidth" else 200))
        out.append(_result("k_swiglu", f"{rows}x{n}", 3 * rows * n * 4, ms, peak_gbs, mode=mode))
    # argmax: rows x n logits in, one index per row out
    for rows, n, mode in [(1, 151936, "latency"), (1024, 128256, "bandwidth")]:
        x, d = randn(rows * n), torch.empty(rows, dtype=torch.int32, device="cuda")
        p = nodes.argmax_params(n, rows)
        wsb = nodes.argmax_workspace_size(p)
        ws = torch.empty(max(wsb, 8), dtype=torch.uint8, device="cuda")
        ms = _time_calls(lambda i: nodes.argmax(p, x, d, ws, wsb), 1, iters or (50 if mode == "bandwidth" else 200))
        out.append(_result("k_argmax_partial+final", f"{rows}x{n}", rows * n * 4 + rows * 4, ms, peak_gbs, mode=mode))
    # rope: 14 q + 2 k heads of 64 at position 1023, base 1e6
    x, d = randn(16 * 64), torch.empty(16 * 64, device="cuda")
    pos = torch.tensor([1023], dtype=torch.int32, device="cuda")
    p = nodes.rope_params(16, 64, freq_base=1e6)
    ms = _time_calls(lambda i: nodes.rope(p, x, pos, d), 1, iters or 200)
    out.append(_result("k_rope", "16x64", 2 * 16 * 64 * 4 + 4, ms, peak_gbs, mode="latency"))
    # soft_max: 14 heads x 2048 columns
    x, d = randn(14 * 2048), torch.empty(14 * 2048, device="cuda")
    p = nodes.soft_max_params(14, 2048, 0.125)
    ms = _time_calls(lambda i: nodes.soft_max(p, x, d), 1, iters or 200)
    out.append(_result("k_soft_max", "14x2048", 2 * 14 * 2048 * 4, ms, peak_gbs, mode="latency"))
    # get_rows: one row of the 151936 x 896 F16 embedding
    table = randn(151936 * 896).half()
    ids, d = torch.tensor([12345], dtype=torch.int32, device="cuda"), torch.empty(896, device="cuda")
    p = nodes.get_rows_params(896, 151936)
    ms = _time_calls(lambda i: nodes.get_rows_f16(p, table, ids, d), 1, iters or 200)
    out.append(_result("k_get_rows", "1 of 151936x896", 896 * 2 + 896 * 4 + 4, ms, peak_gbs, mode="latency"))
    return out
