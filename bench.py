#!/usr/bin/env python3
"""Decode throughput of the Qwen2.5-0.5B-architecture model on B200.

One bench step = one whole sequence of config 4: reset the KV cache, feed the 32 seeded prompt ids
one token at a time, then decode 256 greedy ids (each fed back, as src/FullModel.cpp:1173-1208
does): 288 decode steps through the 24-layer model and the 151936-row LM head, F16 weights, F16 KV
cache. `value` = decode tokens (prompt + generated, one decode step each) per second over the whole
job: with N GPUs, N independent seeded streams (one per GPU, weak scaling; the decode chain does not
shard), summed. Timed on the device with CUDA events around K sequences, max over ranks.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--engine graph|persistent]
  python bench.py --suite gemv [--shapes 14336x4096,...]   # F16 GEMV sweep, one JSON line per shape
  python bench.py --suite ops                              # op latency + multi-row bandwidth sweep
  python bench.py --suite sampler                          # device sampler per call + sampled decode steps
  python bench.py --suite prefill                          # batched-prefill GEMM, prompt-to-first-token, config 4
  python bench.py --suite layer                            # one fused decoder layer: config 3 and a 7B-class layer
  torchrun --nproc-per-node N bench.py --suite gemv_sharded  # row-sharded GEMV + NCCL gathers (C5)

`--impl reference` times the reference's CPU forward on the host cores instead: the C oracle port
(oracle/oracle.c, the reference's numpy forward restated in C, row-parallel on all host threads;
the reference's own GPU path is Vulkan and cannot run on this box), on a bounded sample of the same
workload (the first decode steps of a config-4 sequence).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (Qwen2-0.5B shape); F16 GEMV HBM GB/s vs ~8 TB/s peak"
UNIT = "tokens/s"
N_PROMPT, N_PREDICT = 32, 256
SEED = 20261201


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    for p in (os.path.join(ROOT, "MEASURED_PEAKS.json"),):
        if os.path.exists(p):
            try:
                d = json.load(open(p))
                return float(d["hbm_gbs"]), "measured"
            except Exception:
                pass
    return 6650.0, "fallback"


def bytes_per_token(cfg, pos_avg: float, kv_bytes: int = 2) -> float:
    """Algorithmic HBM bytes of one decode step: every weight once (F16 matrices, F32 biases and
    norms), the embedding row, the KV rows read (pos + 1 per layer and KV head) and written."""
    H, F, V, L = cfg.hidden, cfg.ffn, cfg.vocab, cfg.layers
    qkv = cfg.q_dim + 2 * cfg.kv_dim
    per_layer = qkv * H * 2 + H * cfg.q_dim * 2 + 3 * H * F * 2  # F16 matrices
    per_layer += qkv * 4 + 2 * H * 4  # F32 QKV bias and the two norms
    kv = 2 * cfg.kv_dim * kv_bytes * (pos_avg + 1) + 2 * cfg.kv_dim * kv_bytes
    return L * (per_layer + kv) + V * H * 2 + H * 4 + H * 2


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one graph-engine decode step, summed over
# its 122 launches in one ncu capture at positions 0..7 with warm caches; the command and the per-kernel
# split are in profiles/decode_step_dram_traffic_c4short.md.
GRAPH_STEP_DRAM_BYTES = 1014109440
GRAPH_STEP_DRAM_POS_AVG = 3.5


def step_traffic(cfg, pos_avg: float) -> float:
    """The measured DRAM bytes of one graph-engine decode step (GRAPH_STEP_DRAM_BYTES) plus the
    algorithmic difference in KV-cache reads between the captured positions and pos_avg."""
    return GRAPH_STEP_DRAM_BYTES + bytes_per_token(cfg, pos_avg) - bytes_per_token(cfg, GRAPH_STEP_DRAM_POS_AVG)


def host_threads() -> int:
    """Physical cores this process may run on (SMT siblings share a core's vector units, and the
    oracle's row loops gain nothing from them)."""
    allowed = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        import psutil

        physical = psutil.cpu_count(logical=False) or allowed
    except Exception:
        physical = allowed
    return max(1, min(allowed, physical))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([c.strip() for c in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(6)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_baseline(cfg, tensors, prompt, n_tokens: int, seq_len: int = N_PROMPT + N_PREDICT):
    """The oracle port on the host's physical cores: wall time of n_tokens decode steps at positions
    spread evenly over a config-4 sequence (0 .. seq_len - 1). A step's cost is the same whatever
    the cache holds (the weights dominate; attention reads rows 0..pos), so the sample costs what
    the whole sequence costs per token."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    threads = host_threads()
    oracle.set_threads(threads)
    om = oracle.Qwen2(cfg, tensors, kv_f16=True)
    om.step(int(prompt[0]), 0)  # warm the F16 table and page in the weights
    om.reset()
    positions = [round(i * (seq_len - 1) / max(n_tokens - 1, 1)) for i in range(n_tokens)]
    t0 = time.perf_counter()
    for i, pos in enumerate(positions):
        om.step(int(prompt[i % len(prompt)]), pos)
    dt = time.perf_counter() - t0
    return {"value": n_tokens / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_tokens} decode steps at positions {positions[0]}..{positions[-1]} spread over a config-4 "
                      f"sequence (oracle/oracle.c, F16 KV cache, {threads} threads on physical cores, row-parallel)"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from muyo_llm_b200 import synth

    cfg = synth.QWEN2_05B
    tensors = synth.make_model(cfg, SEED)
    prompt = synth.prompt_ids(SEED, N_PROMPT, cfg.vocab)
    n_tok = 8
    times = []
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(cfg, tensors, prompt, n_tok)
        if i >= args.warmup:
            times.append(n_tok / cb["value"])
    sec = sum(times) / len(times)
    value = n_tok / sec
    cb["value"] = value
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 0, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 weights / f32 compute", "data": "synthetic (seeded random-init)",
            "config": {"workload": f"config 4 sample: {n_tok} decode steps per step, positions spread over 0..287",
                       "model": "Qwen2.5-0.5B arch",
                       "global_batch": 1, "seq_len": n_tok, "parallelism": "host threads"},
            "cpu_baseline": cb, "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(args, rank, world, local_rank):
    import torch

    from muyo_llm_b200 import _abi, engine, synth

    torch.cuda.set_device(local_rank)
    _abi.call("muyo_cuda_init", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    cfg = synth.QWEN2_05B
    tensors = synth.make_model(cfg, SEED)
    prompt = synth.prompt_ids(SEED + rank, args.n_prompt, cfg.vocab)  # an independent stream per GPU
    eng = engine.Qwen2Model.ENGINE_GRAPH if args.engine == "graph" else engine.Qwen2Model.ENGINE_PERSISTENT
    model = engine.Qwen2Model(cfg, tensors, kv_dtype=_abi.KV_F16, device=local_rank, engine=eng)
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    prompt_dev = torch.from_numpy(prompt).cuda()
    out_dev = torch.empty(args.n_predict, dtype=torch.int32, device="cuda")

    def one_sequence():
        _abi.call("muyo_model_reset", model._m, sptr)
        model.generate_device(prompt_dev.data_ptr(), args.n_prompt, args.n_predict, out_dev.data_ptr(), sptr)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        one_sequence()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            one_sequence()
        ev1.record(stream)
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    steps_per_seq = args.n_prompt + args.n_predict
    value = steps_per_seq * world / (ms / 1e3)

    # e2e: the public host API, pinned host prompt in, generated ids out, per sequence
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.reset(sptr)
        model.generate(prompt, args.n_predict, sptr)
    barrier()
    e2e_s = max_over_ranks((time.perf_counter() - t0) / args.steps)
    e2e = {"value": steps_per_seq * world / e2e_s, "unit": UNIT, "h2d_bytes_per_step": args.n_prompt * 4,
           "d2h_bytes_per_step": args.n_predict * 4}

    # roofline: one decode step (a CUDA-graph replay of 5*layers+1 kernels) against HBM bandwidth
    peak, peak_kind = measured_peaks()
    pos_avg = (steps_per_seq - 1) / 2
    alg = bytes_per_token(cfg, pos_avg)
    per_token_s = (ms / 1e3) / steps_per_seq
    achieved = alg / per_token_s / 1e9
    if args.engine == "graph":
        kernel = "decode step (CUDA graph of 5*layers+1 kernels); algorithmic bytes per token / time per token"
        launches = (5 * cfg.layers + 1 + 1) * steps_per_seq * args.steps  # + the control kernel per sequence
    else:
        kernel = ("k_decode_stream: one launch per sequence runs all 288 decode steps; algorithmic bytes "
                  "of the 288 steps / sequence time")
        launches = 2 * args.steps  # control kernel + persistent kernel per sequence
    traffic = step_traffic(cfg, pos_avg) if args.engine == "graph" else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "traffic_unit": "bytes per decode step", "algorithmic_bytes_per_step": alg,
                "peak_kind": peak_kind, "kernel": kernel}
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(cfg, tensors, prompt, 8)
    model.close()
    # With N > 1: BASELINE config 5 after the decode measurement, on the same ranks - the LM head
    # (151936 x 896, cross-GPU greedy pick) and the 7B-class GEMVs row-sharded over the N GPUs, through
    # the NCCL gathers and through the fused NVLink kernel; each rank checks its gathered output and
    # token against one GPU computing the whole matrix.
    sharded = None
    if world > 1 and not args.no_sharded:
        from muyo_llm_b200 import sweep

        torch.cuda.synchronize()
        dist.barrier()
        sharded = sweep.gemv_sharded(rank, world, dist, 0, measured_peaks()[0], check=True)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 weights / f32 compute", "data": "synthetic (seeded random-init)",
                "config": {"workload": (f"config 4: Qwen2.5-0.5B arch, {args.n_prompt}-token prompt + {args.n_predict} "
                                        "greedy, F16 KV, cap 2048"
                                        + ("" if (args.n_prompt, args.n_predict) == (N_PROMPT, N_PREDICT)
                                           else " (shortened: a profiling run, not the config-4 workload)")),
                           "model": "Qwen2.5-0.5B architecture (random init)", "global_batch": world,
                           "seq_len": steps_per_seq, "parallelism": f"replicas x{world} (independent streams)",
                           "l2": "inputs larger than L2 (988 MB of weights per step)",
                           "generated_tokens_per_s": value * args.n_predict / steps_per_seq,
                           "ms_per_token": ms / steps_per_seq},
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cb, "clocks": clocks.summary(),
                "gpu_launches": launches, "engine": args.engine}
        if sharded is not None:
            line["sharded_gemv"] = sharded
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_suite(args):
    """Kernel sweeps (muyo_llm_b200/sweep.py): one JSON line per case, then a clocks line."""
    import torch

    from muyo_llm_b200 import _abi, sweep

    rank, world, local_rank = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local_rank)
    _abi.call("muyo_cuda_init", local_rank)
    peak, peak_kind = measured_peaks()
    if args.suite == "gemv_sharded":
        dist = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",") if s] or None
        with ClockSampler(local_rank) as clocks:
            res = sweep.gemv_sharded(rank, world, dist, args.iters, peak, shapes=shapes)
        if rank == 0:
            for r in res:
                r.update({"suite": args.suite, "peak_GB_s": peak, "peak_kind": peak_kind})
                print(json.dumps(r), flush=True)
            print(json.dumps({"suite": args.suite, "clocks": clocks.summary()}), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    with ClockSampler(0) as clocks:
        if args.suite == "gemv":
            shapes = [tuple(int(v) for v in s.split("x")) for s in args.shapes.split(",") if s] or None
            res = sweep.gemv(shapes, args.iters, peak)
        elif args.suite == "prefill":
            res = sweep.prefill(args.iters, peak, n_prompt=args.n_prompt, n_predict=args.n_predict,
                                gemm_only=args.shapes == "gemm")
        elif args.suite == "layer":
            res = sweep.layer(args.iters, peak)
        elif args.suite == "sampler":
            res = sweep.sampler(args.iters, peak, n_prompt=args.n_prompt, n_predict=args.n_predict)
        else:
            res = sweep.ops(args.iters, peak)
    for r in res:
        r.update({"suite": args.suite, "peak_GB_s": peak, "peak_kind": peak_kind})
        print(json.dumps(r), flush=True)
    print(json.dumps({"suite": args.suite, "clocks": clocks.summary()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true", help="N > 1: skip the config-5 row-sharded GEMV lines")
    ap.add_argument("--engine", default="graph", choices=["persistent", "graph"])
    ap.add_argument("--suite", default="decode",
                    choices=["decode", "gemv", "ops", "gemv_sharded", "sampler", "prefill", "layer"],
                    help="decode: the config-4 headline line (default); gemv / ops: kernel sweeps, one JSON line "
                         "per case (1 GPU)")
    ap.add_argument("--shapes", default="", help="gemv suite: comma-separated ROWSxCOLS list (default: all); "
                    "prefill suite: 'gemm' times the GEMM cases only")
    ap.add_argument("--iters", type=int, default=0, help="gemv / ops suite: calls timed per case (0: automatic)")
    ap.add_argument("--n-prompt", type=int, default=N_PROMPT,
                    help="decode suite: prompt ids per sequence (config 4: 32; smaller only for profiling)")
    ap.add_argument("--n-predict", type=int, default=N_PREDICT,
                    help="decode suite: generated ids per sequence (config 4: 256; smaller only for profiling)")
    args = ap.parse_args()
    rank, world, local_rank = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    if args.suite != "decode":
        run_suite(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
