"""Row-sharded LM-head GEMV with the cross-GPU greedy pick (muyo_llm_b200/shard.py) on real GPUs:
two ranks, one per GPU, NCCL all-gathers of the (value, index) pairs and of the F32 slices.

Each rank builds the same seeded 151936 x 896 F16 matrix (the Qwen2.5-0.5B LM head) and x, computes
its contiguous row range through muyo_cuda_mat_vec_f16_argmax, and must agree with one GPU computing
the whole GEMV: identical greedy index (argmax is compare-only) and identical logits (each row's
arithmetic does not depend on the sharding). Planted maxima on either side of the shard boundary and a
tie across it check the first-index rule. Needs 2 GPUs; skipped otherwise.
"""
from __future__ import annotations

import datetime
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROWS, COLS = 151936, 896


def _inputs(plant):
    rng = np.random.default_rng(20261202)
    w = (rng.uniform(-1, 1, (ROWS, COLS)) * 0.05).astype(np.float16)
    x = rng.standard_normal(COLS).astype(np.float32)
    for row, val in plant:
        w[row] = np.float16(0.0)
        w[row, 0] = np.float16(val)
    x[0] = 1.0
    return w, x


def _worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from muyo_llm_b200 import _abi, nodes, shard

    torch.cuda.set_device(rank)
    _abi.call("muyo_cuda_init", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        out = []
        for plant in ([(1000, 40.0)], [(ROWS // 2 + 3, 40.0)], [(ROWS // 2 - 1, 40.0), (ROWS // 2, 40.0)]):
            w, x = _inputs(plant)
            begin, end = shard.shard_rows(ROWS, world, rank)
            per = shard.rows_per_rank(ROWS, world)
            wd = torch.from_numpy(w[begin:end]).cuda()
            xd = torch.from_numpy(x).cuda()
            be = shard.CudaNcclBackend(wd, begin, end - begin)
            be.set_output(torch.zeros(per, dtype=torch.float32, device="cuda"))
            token, logits = shard.RowShardedGemv(ROWS, world, rank, be)(xd)
            torch.cuda.synchronize()
            if rank == 0:
                full = torch.empty(ROWS, dtype=torch.float32, device="cuda")
                nodes.mat_vec_f16(nodes.mat_vec_params(COLS, ROWS), torch.from_numpy(w).cuda(), xd, full)
                p = nodes.argmax_params(ROWS)
                wsb = nodes.argmax_workspace_size(p)
                ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
                ref = torch.empty(1, dtype=torch.int32, device="cuda")
                nodes.argmax(p, full, ref, ws, wsb)
                torch.cuda.synchronize()
                out.append((int(token.item()), int(ref.item()), bool(torch.equal(logits, full)), plant[0][0]))
        if rank == 0:
            results.put(out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_row_sharded_lm_head_two_gpus(cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for token, ref, same_logits, planted in results.get(timeout=10):
        assert token == ref == planted
        assert same_logits


def _p2p_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from muyo_llm_b200 import _abi, nodes, shard

    torch.cuda.set_device(rank)
    _abi.call("muyo_cuda_init", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        out = []
        plants = ([(1000, 40.0)], [(ROWS // 2 + 3, 40.0)], [(ROWS // 2 - 1, 40.0), (ROWS // 2, 40.0)])
        begin, end = shard.shard_rows(ROWS, world, rank)
        op = None
        for plant in plants:
            w, x = _inputs(plant)
            wd = torch.from_numpy(w[begin:end]).cuda()
            xd = torch.from_numpy(x).cuda()
            if op is None:
                op = shard.P2PShardedGemv(wd, ROWS, world, rank)
            op.w = wd
            for _ in range(3):  # repeated calls: the epoch advances, the flags never need resetting
                token = op(xd)
            y = op.output()
            torch.cuda.synchronize()
            op.check()
            full = torch.empty(ROWS, dtype=torch.float32, device="cuda")
            nodes.mat_vec_f16(nodes.mat_vec_params(COLS, ROWS), torch.from_numpy(w).cuda(), xd, full)
            torch.cuda.synchronize()
            out.append((int(token.item()), plant[0][0], bool(torch.equal(y, full))))
        # Back-to-back calls with no host synchronisation, a different planted maximum each call (x
        # selects which planted row wins): each call's token and output slot, copied out on the stream
        # right after the call, must be that call's, whichever rank runs ahead.
        plants = [(1000, 1), (100000, 2), (ROWS // 2 - 1, 3), (ROWS // 2, 4), (ROWS - 1, 5), (5, 6)]
        rng = np.random.default_rng(7)
        w = (rng.uniform(-1, 1, (ROWS, COLS)) * 0.05).astype(np.float16)
        for row, col in plants:
            w[row] = np.float16(0.0)
            w[row, col] = np.float16(40.0)
        xs = []
        for _, col in plants:
            x = rng.standard_normal(COLS).astype(np.float32)
            for _, c in plants:
                x[c] = 0.0
            x[col] = 1.0
            xs.append(torch.from_numpy(x).cuda())
        op.w = torch.from_numpy(w[begin:end]).cuda()
        tokens = torch.empty(len(plants), dtype=torch.int32, device="cuda")
        outs = [torch.empty(ROWS, dtype=torch.float32, device="cuda") for _ in plants]
        dist.barrier()
        for k in range(len(plants)):
            tok = op(xs[k])
            tokens[k:k + 1].copy_(tok)
            outs[k].copy_(op.output())
        torch.cuda.synchronize()
        op.check()
        wfull = torch.from_numpy(w).cuda()
        back_to_back, fulls = [], []
        for k, (row, _) in enumerate(plants):
            full = torch.empty(ROWS, dtype=torch.float32, device="cuda")
            nodes.mat_vec_f16(nodes.mat_vec_params(COLS, ROWS), wfull, xs[k], full)
            torch.cuda.synchronize()
            fulls.append(full)
            back_to_back.append((int(tokens[k].item()), row, bool(torch.equal(outs[k], full))))
        out.extend(back_to_back)
        # Two of those calls captured in a CUDA graph and replayed twice: the call count lives on the
        # device, so each replay advances the epoch and the slots (two calls keep the host's slot
        # parity, used for the captured output copies, in step with the device's).
        g_tokens = torch.empty(2, dtype=torch.int32, device="cuda")
        g_outs = [torch.empty(ROWS, dtype=torch.float32, device="cuda") for _ in range(2)]
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for k in range(2):
                tok = op(xs[k])
                g_tokens[k:k + 1].copy_(tok)
                g_outs[k].copy_(op.output())
        for _ in range(2):
            g_tokens.fill_(-1)
            for o in g_outs:
                o.zero_()
            graph.replay()
            torch.cuda.synchronize()
            op.check()
            out.extend((int(g_tokens[k].item()), plants[k][0], bool(torch.equal(g_outs[k], fulls[k])))
                       for k in range(2))
        del graph
        # More ranks than rows: rank 1's shard is empty and still takes part in the exchange.
        wt = rng.standard_normal((1, COLS)).astype(np.float16)
        b1, e1 = shard.shard_rows(1, world, rank)
        tiny = shard.P2PShardedGemv(torch.from_numpy(wt[b1:e1].copy()).cuda(), 1, world, rank)
        tok = tiny(xs[0])
        y1 = tiny.output()
        torch.cuda.synchronize()
        tiny.check()
        full1 = torch.empty(1, dtype=torch.float32, device="cuda")
        nodes.mat_vec_f16(nodes.mat_vec_params(COLS, 1), torch.from_numpy(wt).cuda(), xs[0], full1)
        torch.cuda.synchronize()
        out.append((int(tok.item()), 0, bool(torch.equal(y1, full1))))
        tiny.close()
        # rank 1 sits one call out: rank 0's wait for its flag must expire and be reported
        dist.barrier()
        timed_out = None
        if rank == 0:
            op(xd)
            torch.cuda.synchronize()
            try:
                op.check()
                timed_out = False
            except _abi.MuyoError as e:
                timed_out = e.rc == -3
            # the group is dead after a timeout: a further call is refused, not run
            try:
                op(xd)
                timed_out = False
            except _abi.MuyoError as e:
                timed_out = timed_out and e.rc == -6
        dist.barrier()
        results.put((rank, out, timed_out))
        op.close()  # the ranks' epochs now differ, so the group is not used again
    finally:
        dist.destroy_process_group()


def test_fused_gemv_allgather_two_gpus(cuda):
    """muyo_cuda_mat_vec_f16_allgather: the shards go to every GPU over NVLink stores and the
    pairs and flags through peer memory. The full output is bit-identical to one GPU's GEMV on
    every rank, and the token is the planted first-index maximum, also for back-to-back calls with a
    different maximum each (the output and pair slots alternate by call) and for calls replayed from a
    CUDA graph (the call count lives on the device), and with more ranks than rows (an empty shard
    takes part in the exchange). A rank that skips a call
    makes the others' bounded wait expire with MUYO_ETIMEOUT (no hang), after which the group
    refuses further calls (MUYO_ESTATE)."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 30000 + os.getpid() % 1000
    procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = sorted(results.get(timeout=10) for _ in range(2))
    for rank, out, timed_out in got:
        for token, planted, same in out:
            assert token == planted and same, (rank, token, planted, same)
        if rank == 0:
            assert timed_out is True
