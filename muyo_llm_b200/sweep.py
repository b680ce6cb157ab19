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


SAMPLER_CASES = [  # (label, SamplerParams fields): the reference's flags (src/main.cpp:372-394)
    ("T0.8 top-k 40 top-p 0.95 penalty 1.1", dict(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1.1)),
    ("greedy + penalty 1.1", dict(temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.1)),
    ("T0.8 top-k 4096 top-p 0.95", dict(temperature=0.8, top_k=4096, top_p=0.95, repeat_penalty=1.0)),
]


LAYER_ARCHS = {  # (hidden, ffn, heads, kv_heads): BASELINE config 3 and a 7B-class layer
    "0.5b": (896, 4864, 14, 2),
    "7b": (4096, 14336, 32, 8),
}


def layer(iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7, archs=("0.5b", "7b"), pos: int = 1023):
    """muyo_cuda_layer_step (the five fused kernels of one decoder layer: rms_norm + QKV + bias,
    RoPE + KV append + split-K attention, merge + O + residual, rms_norm + gate/up + SwiGLU,
    down + residual) at position `pos` with an F16 cache of 2048 positions. Weights N(0, 0.02) F16;
    enough weight sets rotate that no call finds its weights in L2. Algorithmic bytes: every weight
    once, the KV rows 0..pos read, the new row written."""
    import numpy as np

    from . import _abi

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    out = []
    for arch in archs:
        H, F, nh, nkv = LAYER_ARCHS[arch]
        hd = H // nh
        qkv_rows = H + 2 * nkv * hd
        S = 2048
        cfg = _abi.Qwen2Config(1, H, F, nh, nkv, 8, S, 1e-6, 1e6, _abi.KV_F16)
        wbytes = (qkv_rows * H + H * H + 3 * F * H) * 2
        n_set = max(1, math.ceil(2 * L2_BYTES / wbytes))

        def mat(r, c):
            return (torch.randn(r, c, generator=g, device="cuda") * 0.02).half()

        sets = []
        for _ in range(n_set):
            t = {"attn_norm": torch.ones(H, device="cuda"), "wqkv": mat(qkv_rows, H),
                 "bqkv": torch.randn(qkv_rows, generator=g, device="cuda") * 0.02, "wo": mat(H, H),
                 "ffn_norm": torch.ones(H, device="cuda"), "wgate": mat(F, H), "wup": mat(F, H), "wdown": mat(H, F)}
            w = _abi.LayerWeights(*[t[n].data_ptr() for n in ("attn_norm", "wqkv", "bqkv", "wo", "ffn_norm", "wgate",
                                                              "wup", "wdown")])
            sets.append((t, w))
        kc = (torch.randn(nkv, S, hd, generator=g, device="cuda")).half()
        vc = (torch.randn(nkv, S, hd, generator=g, device="cuda")).half()
        posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
        x = torch.randn(H, generator=g, device="cuda")
        y = torch.empty(H, device="cuda")
        ws_bytes = _abi.lib().muyo_cuda_layer_workspace_size(cfg)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream

        def call(i):
            _abi.call("muyo_cuda_layer_step", cfg, sets[i][1], kc.data_ptr(), vc.data_ptr(), posd.data_ptr(),
                      x.data_ptr(), y.data_ptr(), ws.data_ptr(), ws_bytes, stream)

        n = iters or 200
        ms = _time_calls(call, n_set, n)
        alg = wbytes + qkv_rows * 4 + 2 * H * 4 + 2 * nkv * (pos + 1) * hd * 2 + 2 * nkv * hd * 2
        out.append(_result("muyo_cuda_layer_step", [H, F, nh, nkv, hd], alg, ms, peak_gbs, arch=arch, pos=pos,
                           weight_sets=n_set, kernels=5))
        del sets, kc, vc
        torch.cuda.empty_cache()
    return out


def sampler(iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7, n_prompt: int = 32, n_predict: int = 256):
    """muyo_cuda_sample on a 151936-entry logits row (N(0, 3^2), 64 history ids), device time per call:
    a CUDA graph of `iters` (restore copy of the row, sample) pairs, minus a graph of the copies
    alone. Then whole decode steps with the sampler in the step graph (config 4: Qwen2.5-0.5B
    architecture, F16 KV, 32 prompt + 256 generated ids) against the greedy graph."""
    import ctypes as C

    from . import _abi, engine, synth

    V, n = 151936, iters or 200
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    base = torch.randn(V, generator=g, device="cuda") * 3
    lg = base.clone()
    hist = torch.randint(0, V, (64,), generator=g, device="cuda", dtype=torch.int32)
    state = torch.zeros(int(_abi.lib().muyo_sampler_state_bytes()), dtype=torch.uint8, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()

    def graph_ms(body):
        with torch.cuda.stream(stream):
            body()  # first call outside the capture (attribute and placement checks)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream, capture_error_mode="thread_local"):
            for _ in range(n):
                body()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        gr.replay()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    copy_ms = graph_ms(lambda: lg.copy_(base))
    out = []
    runs = [(label, kw, 0) for label, kw in SAMPLER_CASES]
    runs += [(SAMPLER_CASES[0][0], SAMPLER_CASES[0][1], c) for c in (8, 16)]  # forced cluster sizes
    for label, kw, cluster in runs:
        _abi.call("muyo_sampler_seed", C.c_void_p(state.data_ptr()), seed, None)
        p = _abi.SamplerParams(kw["temperature"], kw["top_k"], kw["top_p"], kw["repeat_penalty"], 64, cluster, seed)

        def body():
            lg.copy_(base)
            _abi.call("muyo_cuda_sample", C.byref(p), C.c_void_p(lg.data_ptr()), V, C.c_void_p(hist.data_ptr()), 64,
                      C.c_void_p(state.data_ptr()), C.c_void_p(tok.data_ptr()), C.c_void_p(stream.cuda_stream))

        ms = graph_ms(body) - copy_ms
        alg = V * 4 * (2 if kw["temperature"] > 0 else 1) + 64 * 4  # logits read (+ written back), history
        out.append(_result("k_sample", f"{V} ({label})", alg, ms, peak_gbs, mode="latency (L2-resident row)",
                           restore_copy_us=copy_ms * 1e3, cluster_ctas=cluster or "auto"))
    cfg = synth.QWEN2_05B
    m = engine.Qwen2Model(cfg, synth.make_model(cfg, seed), kv_dtype=_abi.KV_F16,
                          engine=engine.Qwen2Model.ENGINE_GRAPH)
    prompt = [int(i) for i in synth.prompt_ids(seed, n_prompt, cfg.vocab)]
    for label, kw in [("greedy", None)] + SAMPLER_CASES[:1]:
        if kw:
            m.set_sampler(repeat_last_n=64, seed=seed, **kw)
        best = float("inf")
        for _ in range(3):
            m.reset()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            m.generate(prompt, n_predict)
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        steps = n_prompt + n_predict
        out.append({"kernel": "decode step graph", "shape": f"config 4 ({label})", "us": best * 1e3 / steps,
                    "tokens_per_s": steps / (best * 1e-3), "mode": f"{n_prompt} prompt + {n_predict} generated ids"})
    m.close()
    return out


def prefill(iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7, n_prompt: int = 32, n_predict: int = 256,
            gemm_only: bool = False):
    """Batched prefill. (1) muyo_cuda_mat_mul_f16 at the 0.5B layer's projection shapes for 128
    positions: device time per call (CUDA graph of back-to-back calls), weight GB/s and tensor
    TFLOP/s. (2) Prompt-only prefill (positions 0 .. P-2 of a P-id prompt, then the one decode step
    that forms the first logits) against P decode steps, P = 32, 128, 512. (3) Config 4 end to end
    (32 prompt + 256 generated ids) with and without batched prefill."""
    import ctypes as C

    from . import _abi, engine, synth

    out = []
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    stream = torch.cuda.Stream()
    n_calls = iters or 50
    for N, K, T, what, kern in [(n, k, t, w_, kk) for (n, k, t, w_) in
                                [(1152, 896, 128, "QKV"), (896, 896, 128, "O"), (9728, 896, 128, "gate|up"),
                                 (896, 4864, 128, "down"), (9728, 896, 512, "gate|up")]
                                for kk in ("mma_sync", "tcgen05")]:
        w = (torch.rand(N * K, generator=g, device="cuda") * 0.1 - 0.05).half()
        x = torch.randn(T * K, generator=g, device="cuda")
        y = torch.empty(T * N, device="cuda")
        p = _abi.MatMulParams(K, N, T, 0, 0, _abi.MATMUL_TCGEN05 if kern == "tcgen05" else 0)
        wsb = int(_abi.lib().muyo_cuda_mat_mul_f16_workspace_size(C.byref(p)))
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")

        def call():
            _abi.call("muyo_cuda_mat_mul_f16", C.byref(p), C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()),
                      C.c_void_p(y.data_ptr()), None, C.c_void_p(ws.data_ptr()), wsb, C.c_void_p(stream.cuda_stream))

        with torch.cuda.stream(stream):
            call()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream, capture_error_mode="thread_local"):
            for _ in range(n_calls):
                call()
        gr.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        gr.replay()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / n_calls
        alg = N * K * 2 + T * K * 4 + T * N * 4
        r = _result("k_pf_split + " + ("k_pf_gemm_tc" if kern == "tcgen05" else "k_pf_gemm"),
                    f"{N}x{K}, {T} positions ({what})", alg, ms, peak_gbs, tensor=kern,
                    tflops=2 * N * K * T / (ms * 1e-3) / 1e12, mode="weights L2-resident between calls")
        out.append(r)
    if gemm_only:  # a short program for profiling the GEMM kernels
        return out
    cfg = synth.QWEN2_05B
    t = synth.make_model(cfg, seed)
    models = {}
    # True: prefill with the defaults (512-position passes, GEMM kernel chosen per projection); the
    # others name the kernel (mma_sync, tcgen05, auto = per projection) and the pass length.
    variants = ("auto_128", "mma_sync_128", "tcgen05_128", "mma_sync_512", "tcgen05_512")
    for pf in (False, True) + variants:
        models[pf] = engine.Qwen2Model(cfg, t, kv_dtype=_abi.KV_F16, engine=engine.Qwen2Model.ENGINE_GRAPH)
        if pf in variants:
            _abi.call("muyo_model_set_option", models[pf]._m, b"prefill_positions", int(pf.rsplit("_", 1)[1]))
            _abi.call("muyo_model_set_option", models[pf]._m, b"prefill_tc",
                      {"auto": 2, "mma_sync": 0, "tcgen05": 1}[pf.rsplit("_", 1)[0]])
        if pf:
            _abi.call("muyo_model_set_option", models[pf]._m, b"prefill", 1)

    def timed(m, prompt, n):
        best = float("inf")
        for _ in range(3):
            m.reset()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            m.generate(prompt, n)
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        return best

    for P in (32, 128, 512, 1024):
        prompt = [int(i) for i in synth.prompt_ids(seed, P, cfg.vocab)]
        off, on = timed(models[False], prompt, 1), timed(models[True], prompt, 1)
        ms = {f"ms_prefill_{v}": timed(models[v], prompt, 1) for v in variants}
        out.append({"kernel": "prompt to first token", "shape": f"config 4 arch, {P}-id prompt",
                    "ms_stepwise": off, "ms_prefill": on, **ms, "speedup": off / on,
                    "prompt_tokens_per_s_prefill": P / (on * 1e-3),
                    "mode": "prefill of P-1 positions + 1 step; ms_prefill: the defaults (512-position passes, "
                            "kernel per projection)"})
    prompt = [int(i) for i in synth.prompt_ids(seed, n_prompt, cfg.vocab)]
    for pf in (False, True):
        ms = timed(models[pf], prompt, n_predict)
        out.append({"kernel": "generate", "shape": f"config 4 ({n_prompt} prompt + {n_predict} generated)",
                    "batched_prefill": pf, "ms": ms, "tokens_per_s": (n_prompt + n_predict) / (ms * 1e-3)})
    for m in models.values():
        m.close()
    return out


SHARDED_SHAPES = [(151936, 896), (4096, 4096), (14336, 4096), (128256, 4096)]


def gemv_sharded(rank: int, world: int, dist=None, iters: int = 0, peak_gbs: float = 6462.1, seed: int = 7,
                 shapes=None, check: bool = False):
    """Row-sharded GEMV (muyo_llm_b200/shard.py) over `world` GPUs, one rank per GPU: each rank holds
    ceil(M / world) rows of W. Per shape, two timings on the device (max over ranks):
    * kernel: the local muyo_cuda_mat_vec_f16_argmax alone -> per-GPU GB/s of its shard;
    * e2e: the whole sharded call - local GEMV + argmax, NCCL all-gather of the (value, index) pairs,
      the cross-rank pick, NCCL all-gather of the output slices -> aggregate GB/s of the full matrix.
    * fused (N > 1): muyo_cuda_mat_vec_f16_allgather, the same result from one kernel per GPU that
      stores its slice and pair into every GPU over NVLink.
    Shards rotate over enough copies that more than 4x L2 is touched between two reads of one copy.
    With `check`, every rank also compares the gathered output of both paths with one GPU's GEMV of
    the whole matrix (bit-identical: each row's arithmetic does not depend on the sharding) and the
    token with that output's first-index maximum; `parity` is true when every rank agrees."""
    from . import shard

    g = torch.Generator(device="cuda")
    g.manual_seed(seed * 1000 + rank)

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    out = []
    for rows, cols in shapes or SHARDED_SHAPES:
        begin, end = shard.shard_rows(rows, world, rank)
        local, per = end - begin, shard.rows_per_rank(rows, world)
        wbytes = max(local, 1) * cols * 2
        n_buf = max(1, math.ceil(4 * L2_BYTES / wbytes)) if wbytes < 4 * L2_BYTES else 1
        W = [torch.rand(max(local, 1) * cols, generator=g, device="cuda").mul_(2).sub_(1).half().view(max(local, 1), cols)
             for _ in range(n_buf)]
        x = torch.rand(cols, generator=g, device="cuda").mul_(2).sub_(1)
        if dist is not None:
            dist.broadcast(x, 0)  # x is replicated
        backends = []
        for w in W:
            be = shard.CudaNcclBackend(w, begin, local) if dist is not None else _LocalBackend(w, begin, local)
            be.set_output(torch.zeros(per, dtype=torch.float32, device="cuda"))
            backends.append(be)
        calls = [shard.RowShardedGemv(rows, world, rank, be) for be in backends]
        n = iters or max(20, 4 * n_buf)

        def timed(fn):
            for i in range(3):
                fn(i % n_buf)
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for i in range(n):
                fn(i % n_buf)
            e.record()
            barrier()
            return max_over_ranks(s.elapsed_time(e) / n)

        ms_k = timed(lambda i: backends[i].gemv_argmax(x))
        ms_e = timed(lambda i: calls[i](x))
        ms_p = None
        ms_g = None
        parity = None
        if dist is not None and local > 0:
            p2p = shard.P2PShardedGemv(W[0], rows, world, rank)

            def fused(i):
                p2p.w = W[i]
                p2p(x)

            ms_p = timed(fused)
            p2p.check()
            if check:
                parity = _sharded_parity(calls[0], p2p, W[0], x, rows, cols, world, begin, local, dist)
            # The same calls captured in a CUDA graph (an even number, so the host's output-slot parity
            # stays right) and replayed: host issue time leaves the measurement.
            ng = 2 * max(4, (n_buf + 1) // 2)
            graph = torch.cuda.CUDAGraph()
            barrier()
            with torch.cuda.graph(graph):
                for i in range(ng):
                    fused(i % n_buf)
            reps = max(2, n // ng)
            for _ in range(2):
                graph.replay()
            barrier()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            for _ in range(reps):
                graph.replay()
            e_.record()
            barrier()
            ms_g = max_over_ranks(s_.elapsed_time(e_) / (reps * ng))
            p2p.check()
            del graph
            dist.barrier()
            p2p.close()
        total = rows * cols * 2 + cols * 4 + rows * 4
        local_bytes = local * cols * 2 + cols * 4 + local * 4
        out.append({"kernel": "k_mat_vec_f16 + argmax, row-sharded", "shape": f"{rows}x{cols}", "n_gpus": world,
                    "rows_per_gpu": per, "kernel_us": ms_k * 1e3, "kernel_GB_s_per_gpu": local_bytes / (ms_k * 1e-3) / 1e9,
                    "kernel_frac_of_peak": local_bytes / (ms_k * 1e-3) / 1e9 / peak_gbs,
                    "e2e_us": ms_e * 1e3, "e2e_GB_s_aggregate": total / (ms_e * 1e-3) / 1e9,
                    "e2e_includes": "local GEMV+argmax, NCCL all_gather of pairs and of the F32 output, pick",
                    "fused_us": None if ms_p is None else ms_p * 1e3,
                    "fused_GB_s_aggregate": None if ms_p is None else total / (ms_p * 1e-3) / 1e9,
                    "fused_includes": "one kernel per GPU: local GEMV, output stored into every GPU over NVLink, pairs "
                                      "and flags through peer memory, pick",
                    "fused_graph_us": None if ms_g is None else ms_g * 1e3,
                    "fused_graph_GB_s_aggregate": None if ms_g is None else total / (ms_g * 1e-3) / 1e9,
                    "issue": "e2e_us and fused_us: each call issued from Python (host issue time included); "
                             "fused_graph_us: the fused calls replayed from a CUDA graph",
                    "parity": parity,
                    "shard_copies": n_buf, "calls": n})
        del W, backends, calls
        torch.cuda.empty_cache()
    return out


def _sharded_parity(call, p2p, w_local, x, rows, cols, world, begin, local, dist) -> dict:
    """Both sharded paths against one GPU computing the whole matrix: the full W is rebuilt on every
    rank from the ranks' shards (NCCL all-gather of the padded shards) and its GEMV taken by
    muyo_cuda_mat_vec_f16. `ok` (on every rank): the two paths' gathered outputs are bit-identical
    and each token is the first index of the maximum of its output; the outputs are within
    1e-4 (1 + |e|) of one GPU's (a shard of K >= 2048 columns may split K over other warp counts
    than the whole matrix, so its F32 sums can differ in the last bits); `bit_identical` and
    `token_equal`: against one GPU exactly."""
    from . import shard

    per = shard.rows_per_rank(rows, world)
    pad = torch.zeros(per, cols, dtype=torch.float16, device="cuda")
    pad[:local] = w_local[:local]
    every = torch.empty(world * per, cols, dtype=torch.float16, device="cuda")
    dist.all_gather_into_tensor(every, pad)
    full_w = torch.cat([every[r * per:r * per + (shard.shard_rows(rows, world, r)[1] - shard.shard_rows(rows, world, r)[0])]
                        for r in range(world)])
    full = torch.empty(rows, dtype=torch.float32, device="cuda")
    nodes.mat_vec_f16(nodes.mat_vec_params(cols, rows), full_w, x, full)
    tok_n, y_n = call(x)
    p2p.w = w_local
    tok_p = p2p(x)
    y_p = p2p.output()
    torch.cuda.synchronize()
    yn, yp, ref = y_n.cpu().numpy(), y_p.cpu().numpy(), full.cpu().numpy()
    tn, tp = int(tok_n.item()), int(tok_p.item())
    close = bool((abs(yn.astype("float64") - ref) <= 1e-4 * (1 + abs(ref.astype("float64")))).all())
    ok = bool((yn == yp).all()) and tn == tp == int(yn.argmax()) and close
    exact = bool((yn == ref).all())
    same_tok = tn == int(ref.argmax())
    t = torch.tensor([int(ok), int(exact), int(same_tok)], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    del full_w, every, pad
    return {"ok": bool(t[0].item()), "bit_identical": bool(t[1].item()), "token_equal": bool(t[2].item())}


class _LocalBackend:
    """One GPU, no process group: the gathers are the local tensors themselves."""

    def __init__(self, w, begin, local):
        from . import shard

        self.inner = shard.CudaNcclBackend(w, begin, local)

    def set_output(self, y):
        self.inner.set_output(y)

    def gemv_argmax(self, x):
        return self.inner.gemv_argmax(x)

    def all_gather(self, t):
        return t[None]

    def pick(self, pairs):
        return self.inner.pick(pairs)
