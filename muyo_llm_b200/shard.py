"""Row-sharded F16 GEMV across the GPUs of one node, with the output gathered and a cross-GPU greedy
pick: the multi-GPU form of the LM head (src/FullModel.cpp:973-998: lm_head GEMV -> argmax) and of
the 7B-class GEMV sweep.

Partition: rows are split into `world` contiguous ranges of ceil(M / world) rows (the last range is
shorter); rank r computes its range with muyo_cuda_mat_vec_f16_argmax, which also writes the
range's (max value, first global index) pair. One exchange step follows over NCCL:
  * all_gather of the 8-byte pairs, then muyo_cuda_argmax_pairs picks the first-index maximum
    (src/Sampler.cpp:32-43 across ranks: larger value, then lower index);
  * all_gather of the F32 output slices (padded to equal length), sliced back to M rows.
The x vector is replicated. There is no TMA or peer-memory load in this path: NCCL moves the data.

The gather/partition logic is written once against a small backend interface so that it runs with
the CUDA+NCCL backend on GPUs and with a CPU backend under gloo in tests.
"""
from __future__ import annotations

import numpy as np


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous row range; ranges have ceil(rows / world) rows, the last ones
    fewer (possibly none)."""
    per = -(-rows // world)
    begin = min(rows, rank * per)
    return begin, min(rows, begin + per)


def rows_per_rank(rows: int, world: int) -> int:
    return -(-rows // world)


def combine_pairs(values, indices) -> int:
    """Host statement of the cross-rank greedy rule: the maximum value, ties to the lower index."""
    best_v, best_i = -np.inf, np.iinfo(np.int32).max
    for v, i in zip(np.asarray(values, np.float32), np.asarray(indices, np.int64)):
        if v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    return 0 if best_i == np.iinfo(np.int32).max else int(best_i)


class RowShardedGemv:
    """One rank's view of a row-sharded y = W x with the greedy pick.

    backend: ``gemv_argmax(x) -> (y_local[rows_per], pair[2] (value, index as f32-bits))`` computes the
    local range (rows past the shard end may hold anything), ``all_gather(t) -> stacked`` gathers an
    equal-sized tensor from every rank, ``pick(pairs) -> token`` reduces the gathered pairs.
    """

    def __init__(self, rows: int, world: int, rank: int, backend):
        self.rows, self.world, self.rank = rows, world, rank
        self.begin, self.end = shard_rows(rows, world, rank)
        self.per = rows_per_rank(rows, world)
        self.backend = backend

    def __call__(self, x, want_logits: bool = True):
        y_local, pair = self.backend.gemv_argmax(x)
        token = self.backend.pick(self.backend.all_gather(pair))
        if not want_logits:
            return token, None
        gathered = self.backend.all_gather(y_local)
        return token, gathered.reshape(-1)[: self.rows]


class CudaNcclBackend:
    """libmuyo_cuda kernels on this rank's GPU + torch.distributed (NCCL) for the exchange."""

    def __init__(self, w_shard, row_begin: int, rows_local: int, group=None):
        import torch

        from . import _abi, nodes

        self.torch, self._abi, self.nodes = torch, _abi, nodes
        self.w = w_shard  # torch float16 [rows_local, K] on this rank's device
        self.row_begin, self.rows_local = row_begin, rows_local
        self.group = group
        K = w_shard.shape[1]
        self.params = nodes.mat_vec_params(K, max(rows_local, 1))
        self.ws_bytes = nodes.argmax_workspace_size(nodes.argmax_params(max(rows_local, 1)))
        dev = w_shard.device
        self.ws = torch.empty(max(self.ws_bytes, 8), dtype=torch.uint8, device=dev)
        self.pair = torch.empty(2, dtype=torch.int32, device=dev)
        self.token = torch.empty(1, dtype=torch.int32, device=dev)

    def set_output(self, y_local):
        self.y = y_local

    def gemv_argmax(self, x):
        torch = self.torch
        if self.rows_local == 0:  # empty shard: an identity pair that never wins
            self.pair.copy_(torch.tensor([np.float32(-np.inf).view(np.int32), np.iinfo(np.int32).max],
                                         dtype=torch.int32))
            return self.y, self.pair
        self._abi.call("muyo_cuda_mat_vec_f16_argmax", self.params, self.w.data_ptr(), x.data_ptr(), self.y.data_ptr(),
                       self.row_begin, self.pair.data_ptr(), self.ws.data_ptr(), self.ws_bytes,
                       torch.cuda.current_stream().cuda_stream)
        return self.y, self.pair

    def all_gather(self, t):
        torch = self.torch
        out = torch.empty((torch.distributed.get_world_size(self.group),) + tuple(t.shape), dtype=t.dtype,
                          device=t.device)
        torch.distributed.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out

    def pick(self, pairs):
        self._abi.call("muyo_cuda_argmax_pairs", pairs.data_ptr(), pairs.shape[0], self.token.data_ptr(),
                       self.torch.cuda.current_stream().cuda_stream)
        return self.token


class P2PShardedGemv:
    """The same row-sharded GEMV + greedy pick as one kernel per GPU that writes its shard and its
    (max, index) pair straight into every rank's buffer over NVLink (muyo_cuda_mat_vec_f16_allgather)
    instead of two NCCL all-gathers. A collective: every rank constructs it (the CUDA IPC handles are
    exchanged once over the process group) and calls it in the same order.

    w_shard: torch float16 [rows_local, K] on this rank's GPU (rows [begin, end) of the full matrix).
    """

    def __init__(self, w_shard, rows: int, world: int, rank: int, group=None):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import _abi, nodes

        self.torch, self._abi, self.C = torch, _abi, C
        self.rows, self.world, self.rank = rows, world, rank
        self.begin, self.end = shard_rows(rows, world, rank)
        self.w = w_shard
        self.params = nodes.mat_vec_params(w_shard.shape[1], max(self.end - self.begin, 1))
        self.params.rows = self.end - self.begin
        n = int(_abi.lib().muyo_p2p_handle_bytes())
        handle = (C.c_ubyte * n)()
        g = C.c_void_p()
        _abi.call("muyo_p2p_create", world, rank, rows, C.byref(g), handle)
        self.g = g
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=w_shard.device)
        every = torch.empty(world * n, dtype=torch.uint8, device=w_shard.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        blob = bytes(every.cpu().numpy().tobytes())
        _abi.call("muyo_p2p_connect", g, C.create_string_buffer(blob, len(blob)))
        dist.barrier(group=group)  # every rank has opened every handle before the first call
        self.token = torch.empty(1, dtype=torch.int32, device=w_shard.device)

    def __call__(self, x, stream=None):
        """Returns the greedy index (device int32 [1]); the full output is at `output()`."""
        s = stream if stream is not None else self.torch.cuda.current_stream().cuda_stream
        self._abi.call("muyo_cuda_mat_vec_f16_allgather", self.g, self.params, self.w.data_ptr(), x.data_ptr(),
                       self.begin, self.token.data_ptr(), s)
        return self.token

    def output_ptr(self) -> int:
        """Device address of the latest call's full [rows] F32 output (calls alternate between two
        slots; peers rewrite a slot only after this rank's next call, so read it on the same stream
        before issuing that call)."""
        yp = self.C.c_void_p()
        self._abi.call("muyo_p2p_output", self.g, self.C.byref(yp))
        return yp.value

    def output(self):
        """A copy of the latest call's full [rows] F32 output on this rank (stream-ordered)."""
        torch = self.torch
        out = torch.empty(self.rows, dtype=torch.float32, device=self.w.device)
        self._abi.call("muyo_cuda_copy_f32", _copy_params(self.rows), self.output_ptr(), out.data_ptr(),
                       torch.cuda.current_stream().cuda_stream)
        return out

    def check(self):
        self._abi.call("muyo_p2p_check", self.g)

    def close(self):
        if getattr(self, "g", None):
            self._abi.lib().muyo_p2p_destroy(self.g)
            self.g = None


def _copy_params(n: int):
    from . import _abi

    return _abi.UnaryParams(n, n, 1, 1, 1, 1, n, n, n, n, 1, 1, 1, 1, n, n, n, 0, 0)
