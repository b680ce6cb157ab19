"""The multi-GPU row-sharded GEMV + cross-rank greedy pick (muyo_llm_b200.shard), run as world-size-2 and -4
gloo ranks on CPU. Each rank computes its row range with the oracle (the CPU stand-in for the CUDA
kernel); the partition, padding, gather and pair reduction are the product code."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from muyo_llm_b200 import shard

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_partition_covers_rows():
    for rows in (1, 7, 896, 151936, 128256):
        for world in (1, 2, 4, 8):
            spans = [shard.shard_rows(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert all(e - b <= shard.rows_per_rank(rows, world) for b, e in spans)


def test_combine_pairs_rule():
    assert shard.combine_pairs([1.0, 3.0, 3.0], [5, 9, 2]) == 2
    assert shard.combine_pairs([-np.inf], [np.iinfo(np.int32).max]) == 0


class _CpuBackend:
    def __init__(self, w_shard, begin, per):
        import torch.distributed as dist

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle

        self.oracle, self.dist = oracle, dist
        self.w, self.begin, self.per = w_shard, begin, per

    def gemv_argmax(self, x):
        import torch

        y = np.zeros(self.per, np.float32)
        pair = np.array([-np.inf, np.iinfo(np.int32).max], np.float64)
        if self.w.shape[0]:
            y[: self.w.shape[0]] = self.oracle.mat_vec_f16(self.w, x)
            i = self.oracle.argmax(y[: self.w.shape[0]])
            pair = np.array([y[i], self.begin + i], np.float64)
        return torch.from_numpy(y), torch.from_numpy(pair)

    def all_gather(self, t):
        import torch

        out = [torch.empty_like(t) for _ in range(self.dist.get_world_size())]
        self.dist.all_gather(out, t)
        return torch.stack(out)

    def pick(self, pairs):
        p = pairs.numpy()
        return shard.combine_pairs(p[:, 0], p[:, 1])


def _rank(rank, world, port, rows, cols, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        w = rng.uniform(-1, 1, (rows, cols)).astype(np.float16)
        x = rng.uniform(-1, 1, cols).astype(np.float32)
        b, e = shard.shard_rows(rows, world, rank)
        per = shard.rows_per_rank(rows, world)
        g = shard.RowShardedGemv(rows, world, rank, _CpuBackend(w[b:e], b, per))
        token, logits = g(x)
        q.put((rank, int(token), logits.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,world", [(1001, 2), (4096, 2), (3, 2), (1001, 4), (3, 4)])
def test_row_sharded_gemv_gloo(rows, world):
    """Every rank ends with the full output and the first-index maximum, also with ragged shards
    and with more ranks than rows (empty shards)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    oracle.build()
    cols = 96
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, rows, cols, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    rng = np.random.default_rng(0)
    w = rng.uniform(-1, 1, (rows, cols)).astype(np.float16)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    full = oracle.mat_vec_f16(w, x)
    for _rank_id, token, logits in results:
        assert token == oracle.argmax(full)
        assert (logits == full).all()
