"""Multi-GPU sharding of the quantized-inference path (one process per GPU).

* DequantizeLinear -> MatMul: the weight [K, N] (with its scales / zero points)
  is split by columns into `world` contiguous slices; every rank computes its
  [M, N/world] output slice with the fused kernel and the slices are
  all-gathered (NCCL over NVLink on GPUs, gloo on CPU) into the full [M, N]
  output.  Activations are replicated.
* Attention: KV heads are split into `world` contiguous groups; each rank holds
  the KV cache of its heads and the matching query heads (GQA groups never
  straddle ranks), and the per-head outputs are all-gathered.

The gather writes the rank-major buffer [world, M, N/world]; for M == 1 that is
already the [M, N] layout, otherwise one transpose copy restores it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int):
    """Contiguous [begin, end) of `n` items owned by `rank` (equal shards)."""
    if n % world:
        raise ValueError(f"{n} columns do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def column_slice(t: torch.Tensor, world: int, rank: int, axis: int = -1) -> torch.Tensor:
    b, e = shard_range(t.shape[axis], world, rank)
    return t.narrow(axis, b, e - b).contiguous()


def gather_columns(local: torch.Tensor, world: int, group=None,
                   out: Optional[torch.Tensor] = None,
                   staging: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gathers [M, n_loc] slices into [M, world * n_loc] (rank order)."""
    M, n_loc = local.shape
    if staging is None:
        staging = torch.empty((world, M, n_loc), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(staging.view(-1), local.contiguous().view(-1), group=group)
    if out is None:
        out = torch.empty((M, world * n_loc), dtype=local.dtype, device=local.device)
    if M == 1:
        out.view(-1).copy_(staging.view(-1))
    else:
        out.copy_(staging.permute(1, 0, 2).reshape(M, world * n_loc))
    return out


@dataclass
class ShardedLinear:
    """A column-sharded weight-only quantized projection.

    `compute(a, w, scale, zp)` runs the local fused DequantizeLinear -> MatMul
    (the CUDA kernel on GPUs); `__call__` returns the gathered full output.
    """

    w: object
    scale: torch.Tensor
    zp: object
    n_total: int
    world: int
    compute: Callable
    group: object = None

    def __call__(self, a: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        local = self.compute(a, self.w, self.scale, self.zp)
        local = local.reshape(-1, local.shape[-1])
        full = gather_columns(local, self.world, self.group)
        shape = tuple(a.shape[:-1]) + (self.n_total,)
        if out is not None:
            out.view(-1, self.n_total).copy_(full)
            return out
        return full.reshape(shape)


def kv_head_range(kv_heads: int, q_heads: int, world: int, rank: int):
    """(kv_begin, kv_end, q_begin, q_end) of the heads a rank owns."""
    kb, ke = shard_range(kv_heads, world, rank)
    group = q_heads // kv_heads
    return kb, ke, kb * group, ke * group


def gather_heads(local_y: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gathers rank-4 [B, Hq/world, S, D] head slices into [B, Hq, S, D]."""
    B, h, S, D = local_y.shape
    staging = torch.empty((world, B, h, S, D), dtype=local_y.dtype, device=local_y.device)
    dist.all_gather_into_tensor(staging.view(-1), local_y.contiguous().view(-1), group=group)
    return staging.permute(1, 0, 2, 3, 4).reshape(B, world * h, S, D)
