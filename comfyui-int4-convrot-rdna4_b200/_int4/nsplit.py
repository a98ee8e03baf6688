"""N-column split of a quantized Linear across ranks (tensor parallel over outputs).

Rank r of P owns the contiguous weight rows [r*N/P, (r+1)*N/P) of the packed
codes, scales and bias (and of a Dynamic-LoRA up matrix); each rank computes its
output columns for all tokens and an all-gather assembles [..., N] on every
rank. The reference is single-device; this is the B200 build's column-parallel
variant for the largest layers.

With ``chunks`` > 1 (CUDA tensors) the tokens go in row blocks: block i's
all-gather (NCCL over NVLink, on a side stream) and its placement into the
[M, N] output run while block i+1's columns are computed. The default is one
block: the local GEMM is persistent over every SM, so an all-gather running
beside it takes SMs from it, and the overlapped form measured slower than
computing all local columns first and gathering once.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import convrot_w4a4_linear, convrot_w4a4_linear_lora

_COMM_STREAMS: dict = {}
_ROW_ALIGN = 256          # row blocks are whole GEMM tiles


def shard_rows(qweight: torch.Tensor, wscales: torch.Tensor, bias: torch.Tensor | None, rank: int, world: int):
    """This rank's (qweight, wscales, bias) slice; N must be divisible by world."""
    n = qweight.shape[0]
    if n % world:
        raise ValueError(f"N={n} is not divisible by the world size {world}")
    lo, hi = rank * n // world, (rank + 1) * n // world
    return (qweight[lo:hi].contiguous(), wscales[lo:hi].contiguous(),
            None if bias is None else bias[lo:hi].contiguous())


def shard_adapters(adapters, rank: int, world: int):
    """Each adapter's (down, up rows of this rank, scale): the down projection is shared."""
    out = []
    for down, up, scale in adapters:
        n = up.shape[0]
        if n % world:
            raise ValueError(f"LoRA up rows {n} not divisible by the world size {world}")
        out.append((down, up[rank * n // world:(rank + 1) * n // world].contiguous(), scale))
    return out


def _row_blocks(m: int, world: int, chunks: int | None):
    if chunks is None:
        chunks = 1
    step = max(_ROW_ALIGN, ((m + chunks - 1) // chunks + _ROW_ALIGN - 1) // _ROW_ALIGN * _ROW_ALIGN)
    return [(lo, min(m, lo + step)) for lo in range(0, m, step)]


def _gather_into(out_rows: torch.Tensor, local: torch.Tensor, world: int, group) -> None:
    """out_rows [rows, world * nl] <- the world ranks' local [rows, nl] blocks in rank order."""
    rows, nl = local.shape
    gathered = torch.empty((world, rows, nl), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local, group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), local, group=group)
    out_rows.view(rows, world, nl).copy_(gathered.permute(1, 0, 2))


def _nsplit(x: torch.Tensor, local_fn, nl: int, group, chunks):
    world = dist.get_world_size(group)
    lead = x.shape[:-1]
    x2d = x.reshape(-1, x.shape[-1])
    m = x2d.shape[0]
    if not x.is_cuda or m == 0 or len(_row_blocks(m, world, chunks)) == 1:
        local = local_fn(x2d).contiguous()
        out = torch.empty((m, world * nl), dtype=local.dtype, device=local.device)
        _gather_into(out, local, world, group)
        return out.reshape(*lead, world * nl)
    x2d = x2d.contiguous()
    compute = torch.cuda.current_stream(x.device)
    comm = _COMM_STREAMS.setdefault(x.device, torch.cuda.Stream(x.device))
    out = None
    for lo, hi in _row_blocks(m, world, chunks):
        local = local_fn(x2d[lo:hi]).contiguous()
        if out is None:
            out = torch.empty((m, world * nl), dtype=local.dtype, device=x.device)
        comm.wait_stream(compute)
        with torch.cuda.stream(comm):
            local.record_stream(comm)
            _gather_into(out[lo:hi], local, world, group)
    compute.wait_stream(comm)
    out.record_stream(comm)
    return out.reshape(*lead, world * nl)


def convrot_w4a4_linear_nsplit(x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                               bias_shard: torch.Tensor | None, convrot_groupsize: int = 256,
                               group=None, local_fn=None, chunks: int | None = None) -> torch.Tensor:
    """Local column block through the int4 path, gathered over `group`.

    Every rank passes the same full activation x [..., K]; the result [..., N] is
    identical (bit for bit) on every rank and equal to the unsplit layer's output.
    ``local_fn`` (defaults to ``convrot_w4a4_linear``) computes the local block;
    ``chunks`` row blocks overlap the gather with the compute (CUDA only).
    """
    fn = local_fn or convrot_w4a4_linear
    return _nsplit(x, lambda xx: fn(xx, qweight_shard, wscales_shard, bias_shard, convrot_groupsize),
                   qweight_shard.shape[0], group, chunks)


def convrot_w4a4_linear_lora_nsplit(x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                                    bias_shard: torch.Tensor | None, adapters_shard, convrot_groupsize: int = 256,
                                    group=None, chunks: int | None = None) -> torch.Tensor:
    """As ``convrot_w4a4_linear_nsplit`` with the Dynamic-LoRA side path fused into each
    rank's GEMM: ``adapters_shard`` from ``shard_adapters`` (this rank's up rows)."""
    return _nsplit(x, lambda xx: convrot_w4a4_linear_lora(xx, qweight_shard, wscales_shard, bias_shard,
                                                         adapters_shard, convrot_groupsize),
                   qweight_shard.shape[0], group, chunks)
