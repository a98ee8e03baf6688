"""N-column split of a quantized Linear across ranks (tensor parallel over outputs).

Rank r of P owns the contiguous weight rows [r*N/P, (r+1)*N/P) of the packed
codes, scales and bias; each rank computes its output columns for all tokens
and one all-gather assembles [..., N]. The reference is single-device; this is
the B200 build's column-parallel variant for the largest layers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import convrot_w4a4_linear


def shard_rows(qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None, rank: int, world: int):
    """This rank's (qweight, wscales, bias) slice; N must be divisible by world."""
    n = qweight.shape[0]
    if n % world:
        raise ValueError(f"N={n} is not divisible by the world size {world}")
    lo, hi = rank * n // world, (rank + 1) * n // world
    return (qweight[lo:hi].contiguous(), wscales[lo:hi].contiguous(),
            None if bias is None else bias[lo:hi].contiguous())


def convrot_w4a4_linear_nsplit(x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                               bias_shard: torch.Tensor | None, convrot_groupsize: int = 256,
                               group=None, local_fn=None) -> torch.Tensor:
    """Local column block through the int4 path, then an all-gather over `group`.

    Every rank passes the same full activation x [..., K]; the result [..., N] is
    identical (bit for bit) on every rank and equal to the unsplit layer's output.
    ``local_fn`` (defaults to ``convrot_w4a4_linear``) computes the local block.
    """
    fn = local_fn or convrot_w4a4_linear
    local = fn(x, qweight_shard, wscales_shard, bias_shard, convrot_groupsize)
    world = dist.get_world_size(group)
    lead, nl = local.shape[:-1], local.shape[-1]
    flat = local.reshape(-1, nl).contiguous()
    gathered = torch.empty((world,) + tuple(flat.shape), dtype=flat.dtype, device=flat.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, flat, group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), flat, group=group)
    out = gathered.permute(1, 0, 2).reshape(*lead, world * nl)
    return out
