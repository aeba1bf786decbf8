"""Fused GEMM + all-gather (glq_linear_gather) on the GPU.

The column-parallel layer's exchange runs inside the tcgen05 kernel: its
epilogue stores every output element into every rank's output buffer, the
last CTA publishes an epoch into every rank's signal slots and waits,
bounded, for all ranks' epochs.

On one GPU the protocol is driven by ONE launch whose "peer" buffers are
local allocations: the peer's publication is either pre-set by the test
(so the wait completes without any other kernel) or never made (so the
bounded wait runs out and the kernel reports it in the device error word).
No two kernels that wait on each other ever share a GPU.  The multi-rank test
runs one process per GPU and is skipped with fewer than two GPUs.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from gemm_lab_qualification_b200 import _native as native
from gemm_lab_qualification_b200 import workloads
from oracle import reference as oracle

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
U_ATOL, U_RTOL = oracle.UNIFORM_ATOL, oracle.UNIFORM_RTOL
ERR_TIMEOUT_PEER = 1 << 5


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.fixture(autouse=True)
def clean_error_word(cuda_device):
    native.device_error(clear=True)
    yield
    assert native.device_error(clear=True) == 0, "a bounded in-kernel wait expired"


def emulated_call(dev, a, b, bias, rank, world, epoch, preset_peers=True, n=None):
    """One rank's launch with `world` local output buffers standing in for
    the ranks' buffers; returns (outputs, signals, counter, path)."""
    m = a.shape[0]
    n = b.shape[1] if n is None else n
    outs = [torch.full((m, n * world), 123, dtype=a.dtype, device=dev) for _ in range(world)]
    sigs = [torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=dev) for _ in range(world)]
    if preset_peers:
        for r in range(world):
            if r != rank:
                sigs[rank][r] = epoch  # peer r has already published into this rank's slots
    counter = torch.zeros(4, dtype=torch.int32, device=dev)
    path = native.linear_gather(a, b, bias, native.EPILOGUE_BIAS_SILU, [o.data_ptr() for o in outs], n * world,
                                rank * n, rank, [s.data_ptr() for s in sigs], counter.data_ptr(), epoch)
    torch.cuda.synchronize()
    return outs, sigs, counter, path


@pytest.mark.parametrize("m,layout", [(32, "w_nk"), (1, "w_nk"), (8, "b_kn"), (128, "w_nk")])
def test_gather_fanout_single_launch(cuda_device, m, layout):
    """Rank 1 of 2: its slice lands in both ranks' buffers at its column offset,
    both ranks' slot [1] hold the epoch, the counter is back to zero."""
    a, w, bias = workloads.uniform_inputs(m, 4096, 4096)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    b = dw.t() if layout == "w_nk" else dw.t().contiguous()
    outs, sigs, counter, path = emulated_call(cuda_device, da, b, db, rank=1, world=2, epoch=7)
    assert path[0] == ("tc_kn" if layout == "b_kn" else "tc_splitk")
    expected = oracle.linear_reference(a, w, bias, silu=True)
    for o in outs:
        oracle.compare(host(o[:, 4096:]), expected, U_ATOL, U_RTOL)
        assert bool((o[:, :4096] == 123).all()), "another rank's columns were written"
    assert torch.equal(outs[0], outs[1])
    assert int(sigs[0][1]) == 7 and int(sigs[1][1]) == 7
    assert int(sigs[1][0]) == 7  # pre-set by the test (the emulated rank 0)
    assert int(sigs[0][0]) == 0  # rank 0 never ran
    assert int(counter[0]) == 0


def test_gather_consecutive_epochs_single_rank(cuda_device):
    """world = 1: the protocol completes on its own slot; epochs advance, the
    counter returns to zero after every call, results match."""
    a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
    da, db_w, db = a.to(cuda_device), w.to(cuda_device).t(), bias.to(cuda_device)
    out = torch.empty((32, 4096), dtype=torch.float16, device=cuda_device)
    sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    expected = oracle.linear_reference(a, w, bias, silu=True)
    for epoch in (1, 2, 3):
        out.fill_(0)
        path = native.linear_gather(da, db_w, db, native.EPILOGUE_BIAS_SILU, [out.data_ptr()], 4096, 0, 0,
                                    [sig.data_ptr()], counter.data_ptr(), epoch)
        torch.cuda.synchronize()
        oracle.compare(host(out), expected, U_ATOL, U_RTOL)
        assert int(sig[0]) == epoch and int(counter[0]) == 0
    # same bits as the plain call on the same (tiled, split-K) kernel
    plain = torch.empty_like(out)
    assert native.linear(da, db_w, plain, db, native.EPILOGUE_BIAS_SILU, split_k=path[1]) == path
    torch.cuda.synchronize()
    assert torch.equal(plain.view(torch.int16), out.view(torch.int16))


def test_gather_peer_timeout_sets_status(cuda_device):
    """A peer that never publishes: the bounded wait runs out (about 1 s), the
    kernel returns, the device error word reports it, the context stays usable."""
    a, w, bias = workloads.uniform_inputs(8, 1024, 1024)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    outs, sigs, counter, _ = emulated_call(cuda_device, da, dw.t(), db, rank=0, world=2, epoch=3,
                                           preset_peers=False)
    assert native.device_error(clear=True) & ERR_TIMEOUT_PEER
    expected = oracle.linear_reference(a, w, bias, silu=True)
    oracle.compare(host(outs[0][:, :1024]), expected, U_ATOL, U_RTOL)
    assert int(sigs[1][0]) == 3 and int(counter[0]) == 0
    # the device still runs ordinary work
    y = torch.empty((8, 1024), dtype=torch.float16, device=cuda_device)
    native.linear(da, dw.t(), y, db, native.EPILOGUE_BIAS_SILU)
    torch.cuda.synchronize()
    oracle.compare(host(y), expected, U_ATOL, U_RTOL)


def test_gather_rejects_non_tensor_core_layouts(cuda_device):
    a, w, bias = workloads.uniform_inputs(8, 512, 512)
    da, dw, db = a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device)
    out = torch.empty((8, 512), dtype=torch.float16, device=cuda_device)
    sig = torch.zeros(native.MAX_RANKS, dtype=torch.int64, device=cuda_device)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    with pytest.raises(native.GlqError) as e:
        native.linear_gather(da.t().contiguous().t(), dw.t(), db, native.EPILOGUE_BIAS_SILU, [out.data_ptr()], 512,
                             0, 0, [sig.data_ptr()], counter.data_ptr(), 1)
    assert e.value.status == 1
    torch.cuda.synchronize()
    assert int(sig[0]) == 0


def test_column_parallel_fused_single_rank(cuda_device, tmp_path):
    """The fused-gather layer on a one-rank group (torch symmetric memory)."""
    import torch.distributed as dist
    from gemm_lab_qualification_b200 import sharded
    store = dist.FileStore(str(tmp_path / "store"), 1)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, device_id=cuda_device)
    try:
        a, w, bias = workloads.uniform_inputs(32, 4096, 4096)
        layer = sharded.ColumnParallelLinear(w, bias, "silu", device=cuda_device, fused_gather=True, max_rows=32)
        da = a.to(cuda_device)
        y1 = layer(da).clone()
        y2 = layer(da)
        torch.cuda.synchronize()
        expected = oracle.linear_reference(a, w, bias, silu=True)
        oracle.compare(host(y1), expected, U_ATOL, U_RTOL)
        assert torch.equal(y1, y2)
        assert layer.gather.epoch == 2
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, errors) -> None:
    sys.path.insert(0, str(REPO))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                device_id=dev, timeout=datetime.timedelta(seconds=60))
        from gemm_lab_qualification_b200 import _native, sharded, workloads as wl
        from oracle import reference as orc
        expected = None
        for m in (32, 1):
            a, w, bias = wl.uniform_inputs(m, 1024 * world, 4096)
            layer = sharded.ColumnParallelLinear(w, bias, "silu", device=dev, fused_gather=True, max_rows=m)
            da = a.to(dev)
            outs = [layer(da).clone() for _ in range(3)]
            torch.cuda.synchronize()
            expected = orc.linear_reference(a, w, bias, silu=True)
            for y in outs:
                orc.compare(y.float().cpu().numpy().astype(np.float64), expected, orc.UNIFORM_ATOL, orc.UNIFORM_RTOL)
            assert _native.device_error(clear=True) == 0
            dist.barrier()
    except BaseException as exc:  # report to the parent, never hang it
        errors.put(f"rank {rank}: {exc!r}")
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_column_parallel_fused_multi_gpu():
    """One process per visible GPU (2 to 8): the fused layer on every rank
    equals the unsharded FP64 reference, three calls in a row (both buffer
    parities), for M = 32 (split-K tiles) and M = 1."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
