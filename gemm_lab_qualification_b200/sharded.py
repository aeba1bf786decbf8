"""Column-parallel (N-sharded) linear layer across the GPUs of one node.

W [N, K] and bias [N] are split along N into P equal row slices, one per
rank; every rank holds the full activations A [M, K] and computes its slice
y_r = act(A @ W_r^T + b_r).  Two ways to assemble y [M, N] on every rank:

* ``fused_gather=True`` (the B200 path): one kernel per rank,
  glq_linear_gather.  Its epilogue stores each output element straight into
  every rank's output buffer over NVLink (peer pointers from torch symmetric
  memory), then the last CTA publishes an epoch into every rank's signal
  slots and waits, bounded, for all ranks' epochs.  No collective launch, no
  layout copy: the output is row-major [M, N] in place.  Outputs alternate
  between two buffers by epoch parity, so a rank's next call never writes
  into the buffer a peer may still be reading.
* ``fused_gather=False``: the local kernel, then an NCCL all-gather of the
  [M, N/P] slices and one strided copy [P, M, N/P] -> [M, N].

One process per GPU (torch.distributed); no TMA multicast anywhere.  The
symmetric buffers are requested without NVLink multicast objects (only
plain peer mappings are used).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from . import _native, kernels


def shard_rows(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank*N/P, (rank+1)*N/P) of a [N, ...] tensor (N divisible by P)."""
    n = t.shape[0]
    if n % world:
        raise ValueError(f"N = {n} is not divisible by {world} ranks")
    ns = n // world
    return t[rank * ns:(rank + 1) * ns]


def gather_columns(local: torch.Tensor, out: torch.Tensor, group=None,
                   gathered: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather the per-rank [M, N/P] slices into row-major out [M, N]."""
    world = dist.get_world_size(group)
    m, ns = local.shape
    if tuple(out.shape) != (m, ns * world):
        raise ValueError("output must be [M, N/P * P]")
    if gathered is None:
        gathered = torch.empty((world, m, ns), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local.contiguous(), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), local.contiguous(), group=group)
    out.view(m, world, ns).copy_(gathered.permute(1, 0, 2))
    return out


class ColumnParallelLinear:
    """y = SiLU(A @ W^T + b) (or A @ W^T with bias=None) with W split along N."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, activation: str | None = "silu",
                 group=None, device: torch.device | None = None, fused_gather: bool = False,
                 max_rows: int = 128) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if activation not in (None, "silu"):
            raise ValueError("activation must be None or 'silu'")
        if activation == "silu" and bias is None:
            raise ValueError("the fused SiLU epilogue takes a bias")
        self.activation = activation
        self.n, self.k = weight.shape
        if fused_gather and self.k % 8 != 0:
            # The gather is fused into the tcgen05 kernel, which reads A and W
            # through TMA: rows must be 16-byte pitched.
            raise ValueError("the fused gather needs K to be a multiple of 8 (16-byte rows of A and W)")
        device = device if device is not None else weight.device
        self.weight = shard_rows(weight, self.rank, self.world).to(device).contiguous()
        self.bias = shard_rows(bias, self.rank, self.world).to(device).contiguous() if bias is not None else None
        self.gather = FusedGather(max_rows, self.n, weight.dtype, device, group) if fused_gather else None

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y = act(A @ W^T + b) [M, N] on every rank.  With the fused gather and
        no ``out`` the result is a view of the gather buffers, valid until the
        call after next."""
        m = a.shape[0]
        if self.gather is not None:
            epi = _native.EPILOGUE_BIAS_SILU if self.activation == "silu" else (
                _native.EPILOGUE_BIAS if self.bias is not None else _native.EPILOGUE_NONE)
            y = self.gather(a, self.weight.t(), self.bias, epi)
            if out is None:
                return y
            out.copy_(y)
            return out
        ns = self.weight.shape[0]
        local = torch.empty((m, ns), dtype=a.dtype, device=a.device)
        kernels.linear_into(a, self.weight.t(), local, self.bias, self.activation)
        if out is None:
            out = torch.empty((m, self.n), dtype=a.dtype, device=a.device)
        return gather_columns(local, out, self.group)


def _symm_mem():
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import torch.distributed._symmetric_memory as symm_mem
    return symm_mem


class FusedGather:
    """Symmetric output buffers and signal slots for glq_linear_gather.

    Layout of each rank's symmetric allocation (bytes): two output buffers of
    [max_rows, n_total] elements, then GLQ_MAX_RANKS uint64 signal slots,
    then this rank's uint32 arrival counter.  Every rank must construct it
    collectively (same arguments, same order).
    """

    _ALIGN = 256

    def __init__(self, max_rows: int, n_total: int, dtype: torch.dtype, device: torch.device, group=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _native.MAX_RANKS:
            raise ValueError(f"at most {_native.MAX_RANKS} ranks")
        self.max_rows, self.n_total, self.dtype = max_rows, n_total, dtype
        esz = torch.empty((), dtype=dtype).element_size()
        align = self._ALIGN
        self.y_bytes = (max_rows * n_total * esz + align - 1) // align * align
        self.sig_off = 2 * self.y_bytes
        self.counter_off = self.sig_off + _native.MAX_RANKS * 8
        total = self.counter_off + align
        symm_mem = _symm_mem()
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        target = group if group is not None else dist.group.WORLD
        self.handle = symm_mem.rendezvous(self.buf, target)
        self.bases = [int(p) for p in self.handle.buffer_ptrs]
        self.epoch = 0
        # Per-parity peer output pointers and the signal slots, built once.
        self._y_ptrs = [[base + parity * self.y_bytes for base in self.bases] for parity in (0, 1)]
        self._sig_ptrs = [base + self.sig_off for base in self.bases]
        self._counter = self.bases[self.rank] + self.counter_off
        dist.barrier(group)  # every rank's slots are zero before anyone publishes

    def output(self, parity: int, rows: int) -> torch.Tensor:
        """This rank's gathered output of the call with this epoch parity."""
        start = parity * self.y_bytes
        elems = self.max_rows * self.n_total
        flat = self.buf[start:start + elems * torch.empty((), dtype=self.dtype).element_size()]
        return flat.view(self.dtype).view(self.max_rows, self.n_total)[:rows]

    def __call__(self, a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None, epilogue: int,
                 split_k: int = 0) -> torch.Tensor:
        """y [M, n_total] on every rank; b is this rank's [K, N/P] operand."""
        m = a.shape[0]
        n_local = b.shape[1]
        if m > self.max_rows or n_local * self.world != self.n_total:
            raise ValueError("call does not fit the gather buffers")
        if a.dtype != self.dtype:
            raise ValueError("dtype differs from the gather buffers")
        self.epoch += 1
        parity = self.epoch & 1
        status, _, _ = kernels._binding().linear_gather(a, b, bias, epilogue, self._y_ptrs[parity], self.n_total,
                                                        self.rank * n_local, self.rank, self._sig_ptrs,
                                                        self._counter, self.epoch, split_k, kernels._flags())
        if status != _native.STATUS_OK:
            raise _native.GlqError(status, "glq_linear_gather")
        return self.output(parity, m)
