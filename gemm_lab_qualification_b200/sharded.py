"""Column-parallel (N-sharded) linear layer across the GPUs of one node.

W [N, K] and bias [N] are split along N into P equal row slices, one per
rank; every rank holds the full activations A [M, K], computes its slice
y_r = act(A @ W_r^T + b_r) with the native kernels, and one all-gather over
NVLink (NCCL) assembles y [M, N].  The gathered buffer is [P, M, N/P]; the
layout fix to row-major [M, N] is one strided copy.

The reference has no multi-GPU path; this is the sharding its BASELINE
configuration asks for.  One process per GPU (torch.distributed), NCCL for
the exchange; no TMA multicast anywhere.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import kernels


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
                 group=None, device: torch.device | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if activation not in (None, "silu"):
            raise ValueError("activation must be None or 'silu'")
        if activation == "silu" and bias is None:
            raise ValueError("the fused SiLU epilogue takes a bias")
        self.activation = activation
        self.n, self.k = weight.shape
        device = device if device is not None else weight.device
        self.weight = shard_rows(weight, self.rank, self.world).to(device).contiguous()
        self.bias = shard_rows(bias, self.rank, self.world).to(device).contiguous() if bias is not None else None

    def __call__(self, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        m = a.shape[0]
        ns = self.weight.shape[0]
        local = torch.empty((m, ns), dtype=a.dtype, device=a.device)
        kernels.linear_into(a, self.weight.t(), local, self.bias, self.activation)
        if out is None:
            out = torch.empty((m, self.n), dtype=a.dtype, device=a.device)
        return gather_columns(local, out, self.group)
