"""Host logic of the column-parallel layer on CPU: 2 gloo ranks (127.0.0.1).

The sharding and the all-gather + layout fix are checked with gloo; the local
fused GEMM of each rank is the native kernel, exercised by the GPU tests.
Here each rank's slice is produced by the FP64 oracle, so the test isolates
the exchange and layout logic.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, m: int, n: int, k: int, errors) -> None:
    sys.path.insert(0, str(REPO))
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from gemm_lab_qualification_b200 import sharded, workloads
        from oracle import reference as oracle
        a, w, bias = workloads.uniform_inputs(m, n, k)
        w_r = sharded.shard_rows(w, rank, world)
        b_r = sharded.shard_rows(bias, rank, world)
        assert w_r.shape == (n // world, k)
        local = torch.from_numpy(oracle.linear_reference(a, w_r, b_r, silu=True, samples=4)).to(torch.float64)
        out = torch.empty((m, n), dtype=torch.float64)
        sharded.gather_columns(local, out)
        full = oracle.linear_reference(a, w, bias, silu=True, samples=4)
        assert np.array_equal(out.numpy(), full), "gathered layout differs from the unsharded result"
        with pytest.raises(ValueError):
            sharded.shard_rows(torch.zeros(n + 1, 2), rank, world)
        # the fused gather needs 16-byte rows: refused before any device work
        with pytest.raises(ValueError, match="multiple of 8"):
            sharded.ColumnParallelLinear(torch.zeros(n, 13, dtype=torch.float16), torch.zeros(n, dtype=torch.float16),
                                         device=torch.device("cpu"), fused_gather=True)
        dist.barrier()
    except BaseException as exc:  # report to the parent, never hang it
        errors.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("m,n,k", [(3, 8, 16), (32, 256, 64)])
def test_column_parallel_gather_two_ranks(m, n, k):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, m, n, k, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_shard_rows_partition():
    from gemm_lab_qualification_b200 import sharded
    w = torch.arange(24).reshape(8, 3)
    parts = [sharded.shard_rows(w, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts), w)
    with pytest.raises(ValueError):
        sharded.shard_rows(w, 0, 3)
