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

``PeerColumnSplit`` (CUDA, NCCL group, bf16 activations of whole 256-column
tiles) replaces the gather: every rank's GEMM writes its column block into its
own [M, N] buffer in row chunks, and the copy engines carry each finished
chunk to every peer's buffer over NVLink (peer mappings by CUDA IPC, no
multicast) while the next chunk computes; a flag barrier with a bounded wait
then tells each rank that all blocks have landed. No NCCL kernel runs and no
permute copy is needed; the result is bit-identical. (Stores to the peers
straight from the GEMM epilogue measured slower: the remote stores hold up the
epilogue, and with it the MMAs, 540 against 291 us on 2 GPUs.)
"""
from __future__ import annotations

import contextlib
import os

import torch
import torch.distributed as dist

from . import _lora_operands, convrot_w4a4_linear, convrot_w4a4_linear_lora, cuda_loader

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


class _HostArrayView:
    """A [rows, cols] view of device memory this module allocated (CUDA array interface)."""

    def __init__(self, ptr: int, rows: int, cols: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


_VIEW_TYPES = {torch.bfloat16: ("<i2", torch.int16), torch.float32: ("<f4", torch.float32)}


class PeerSplitUnavailable(RuntimeError):
    """Raised on every rank when some rank cannot map a peer's buffer."""


def _all_ranks_ok(ok: bool, group, device) -> bool:
    """True on every rank exactly when ``ok`` holds on every rank of ``group`` (MIN all-reduce)."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(int(flag.item()))


def _on_device(device: torch.device):
    """The CUDA device context for ``device`` (none needed for a CPU device)."""
    return torch.cuda.device(device) if device.type == "cuda" else contextlib.nullcontext()


class PeerColumnSplit:
    """Peer-memory resources of the column-split linear for one process group.

    Per rank: a flag page (int32 slots written by the peers, plus this rank's
    epoch counter) and, per output shape, two [M, N] buffers used in turn; all
    mapped into every rank by CUDA IPC. Creating it and the first call for a
    shape are collective: every rank makes the same calls in the same order.
    Two buffers in turn are enough: rank r writes buffer b of call i + 2 only
    after passing the barrier of call i + 1, which rank p enters only after
    copying out call i.
    """

    TIMEOUT_NS = 2_000_000_000
    CHUNK_MIN_ROWS = 4096     # two row chunks from 8192 rows on (measured: 2 beat 1, 4 and 8)

    def __init__(self, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer column split supports up to 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._own: list[int] = []
        self._opened: list[int] = []
        flags = self._alloc(256)
        try:
            self.flag_ptrs = self._exchange(flags)
        except PeerSplitUnavailable:
            self.close()                 # every rank is on this path: the barriers in close() match
            raise
        self.counter = flags[0] + 128
        self._outs: dict = {}
        self.copy_stream = torch.cuda.Stream(self.device)

    def _alloc(self, nbytes: int):
        with _on_device(self.device):
            ptr, handle = cuda_loader.peer_buffer_alloc(nbytes)
        self._own.append(ptr)
        return ptr, handle

    def _exchange(self, own) -> list[int]:
        """Every rank's pointer to its buffer (this rank's own, the others' opened). The
        ranks agree on the outcome: if any rank fails to map a peer's buffer, every
        rank raises PeerSplitUnavailable (so none is left waiting in a collective)."""
        handles = [None] * self.world
        dist.all_gather_object(handles, own[1], group=self.group)
        ptrs = []
        err = None
        with _on_device(self.device):
            for p, h in enumerate(handles):
                if p == self.rank:
                    ptrs.append(own[0])
                    continue
                try:
                    q = cuda_loader.peer_buffer_open(h)
                except RuntimeError as e:          # no peer mapping between these devices
                    err = e
                    break
                self._opened.append(q)
                ptrs.append(q)
        if not _all_ranks_ok(err is None, self.group, self.device):
            raise PeerSplitUnavailable(f"a rank could not map a peer's buffer ({err or 'on another rank'})")
        return ptrs

    def output(self, m: int, n: int, dtype: torch.dtype):
        """(every rank's pointer to this call's [m, n] buffer, this rank's buffer as a tensor)."""
        key = (m, n, dtype)
        if key not in self._outs:
            typestr, view_dtype = _VIEW_TYPES[dtype]
            bufs = []
            for _ in range(2):
                own = self._alloc(m * n * torch.empty((), dtype=dtype).element_size())
                ptrs = self._exchange(own)
                local = torch.as_tensor(_HostArrayView(own[0], m, n, typestr), device=self.device).view(dtype)
                bufs.append((ptrs, local))
            self._outs[key] = [bufs, 0]
        entry = self._outs[key]
        bufs, i = entry
        entry[1] = 1 - i
        return bufs[i]

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with _on_device(self.device):
            for q in self._opened:
                cuda_loader.peer_buffer_close(q)
            dist.barrier(group=self.group)
            for p in self._own:
                cuda_loader.peer_buffer_free(p)
        self._opened, self._own, self._outs = [], [], {}


def peer_split_supported(x: torch.Tensor, n_local: int, convrot_groupsize: int, group=None) -> bool:
    """The peer form applies: CUDA bf16 rows of whole tiles, an NCCL group of <= 8
    ranks, local column blocks of whole 16-byte chunks (CONVROT_NSPLIT_PEER=0 turns
    it off)."""
    if os.environ.get("CONVROT_NSPLIT_PEER", "1") == "0" or not x.is_cuda:
        return False
    if dist.get_backend(group) != "nccl" or dist.get_world_size(group) > 8 or n_local % 8:
        return False
    return cuda_loader.unpacked_path_supported(x.reshape(-1, x.shape[-1]), convrot_groupsize)


def convrot_w4a4_linear_peer_split(x: torch.Tensor, qweight_shard: torch.Tensor, wscales_shard: torch.Tensor,
                                   bias_shard: torch.Tensor | None, adapters_shard, split: PeerColumnSplit,
                                   convrot_groupsize: int = 256) -> torch.Tensor:
    """The column-split int4 linear (optional Dynamic-LoRA side path) over peer memory.

    Every rank passes the full x; quantization (and the LoRA down projection)
    run on each rank. The A8 GEMM on this rank's N/P weight rows writes its
    columns into this rank's [M, N] buffer, in row chunks; each chunk goes on
    to every peer's buffer by copy-engine 2D copies on a side stream while the
    next chunk computes (no SM time taken from the GEMM); the flag barrier
    completes the exchange. Returns a fresh [..., N] tensor equal (bit for bit)
    to the unsplit layer's output on every rank.
    """
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).contiguous()
    m = x2d.shape[0]
    nl = qweight_shard.shape[0]
    n = nl * split.world
    esize = x.element_size()
    qact, x_scale = cuda_loader.convrot_quant_int4_unpacked(x2d, convrot_groupsize)
    lora_t = lora_b = None
    lora_scale = 0.0
    adapters_shard = list(adapters_shard or ())
    if adapters_shard:
        lora_t, lora_b, lora_scale = _lora_operands(x2d, adapters_shard, nl)
    ptrs, local = split.output(m, n, x.dtype)
    own = ptrs[split.rank]
    peers = [p for r, p in enumerate(ptrs) if r != split.rank]
    main = torch.cuda.current_stream(x.device)
    side = split.copy_stream
    rows = m if m < split.CHUNK_MIN_ROWS * 2 else (m + 1) // 2
    for lo in range(0, m, rows):
        hi = min(m, lo + rows)
        cuda_loader.int4_convrot_gemm_a8_peers(
            qact[lo:hi], qweight_shard, x_scale[lo:hi], wscales_shard, bias_shard, x.dtype, [own + lo * n * esize],
            n, split.rank * nl, None if lora_t is None else lora_t[lo:hi], lora_b, lora_scale)
        if peers:
            done = torch.cuda.Event()
            done.record(main)
            side.wait_event(done)
            cuda_loader.peer_copy_columns([p + lo * n * esize for p in peers], own + lo * n * esize, n * esize,
                                          split.rank * nl * esize, nl * esize, hi - lo, side)
    if peers:
        sent = torch.cuda.Event()
        sent.record(side)
        main.wait_event(sent)
    cuda_loader.peer_barrier(split.flag_ptrs, split.rank, split.counter, split.TIMEOUT_NS, x.device)
    return local.clone().reshape(*shape[:-1], n)
