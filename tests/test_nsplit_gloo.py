"""Host logic of the N-column split on 2 CPU ranks (gloo): sharding, all-gather
and column order give exactly the unsplit layer's output. The local block is
computed by the CPU oracle here (the product path itself needs a GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_linear(x, qw, ws, bias, g):
    from oracle import convrot_oracle as orc
    lead = x.shape[:-1]
    xb = x.reshape(-1, x.shape[-1]).contiguous().view(torch.int16).numpy().view(np.uint16)
    out = orc.convrot_w4a4_linear(xb, qw.numpy(), ws.numpy(), None if bias is None else bias.float().numpy(), g)
    return torch.from_numpy(out.view(np.int16).copy()).view(torch.bfloat16).reshape(*lead, qw.shape[0])


def _worker(rank, world, port, path, result_q):
    import sys
    sys.path[:0] = path
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from _int4.nsplit import convrot_w4a4_linear_nsplit, shard_rows
        g = torch.Generator().manual_seed(0)
        m, k, n = 7, 512, 96
        x = torch.randn(2, m, k, generator=g).to(torch.bfloat16)
        from oracle import convrot_oracle as orc
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)
        qw, ws = orc.quantize_weight(w.numpy(), 256, "f16")
        qw, ws = torch.from_numpy(qw), torch.from_numpy(ws)
        bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
        q_s, w_s, b_s = shard_rows(qw, ws, bias, rank, world)
        out = convrot_w4a4_linear_nsplit(x, q_s, w_s, b_s, 256, local_fn=_oracle_linear)
        full = _oracle_linear(x.reshape(-1, k), qw, ws, bias, 256).reshape(2, m, n)
        result_q.put((rank, tuple(out.shape), bool(torch.equal(out.view(torch.int16), full.view(torch.int16)))))
    except Exception as e:  # report instead of leaving the peer waiting for the queue
        result_q.put((rank, repr(e), False))
        raise
    finally:
        dist.destroy_process_group()


def test_nsplit_two_ranks_matches_unsplit():
    import sys
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, list(sys.path), q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, shape, equal in results:
        assert shape == (2, 7, 96)
        assert equal, f"rank {rank} differs from the unsplit output"


def test_shard_rows_rejects_uneven():
    from _int4.nsplit import shard_rows
    with pytest.raises(ValueError):
        shard_rows(torch.zeros(10, 4, dtype=torch.int8), torch.ones(10), None, 0, 3)


def _peer_exchange_worker(rank, world, port, path, fail_rank, result_q):
    """The peer split's buffer exchange on CPU ranks with the device calls faked: the
    handles go round, one rank's mapping may fail, and the ranks must agree."""
    import sys
    sys.path[:0] = path
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from _int4 import cuda_loader, nsplit
        calls = []

        def alloc(nbytes):
            ptr = 0x1000 * (rank + 1) + len(calls)
            calls.append(("alloc", ptr))
            return ptr, bytes([rank]) * 64

        def open_(handle):
            if rank == fail_rank:
                raise RuntimeError("ck_peer_buffer_open: peer access unsupported (fake)")
            calls.append(("open", handle[0]))
            return 0x9000 + handle[0]

        cuda_loader.peer_buffer_alloc = alloc
        cuda_loader.peer_buffer_open = open_
        cuda_loader.peer_buffer_close = lambda p: calls.append(("close", p))
        cuda_loader.peer_buffer_free = lambda p: calls.append(("free", p))
        if fail_rank >= 0:
            try:
                nsplit.PeerColumnSplit(device="cpu")
                outcome = "constructed"
            except nsplit.PeerSplitUnavailable:
                outcome = "unavailable"
            result_q.put((rank, outcome, calls))
        else:
            split = object.__new__(nsplit.PeerColumnSplit)
            split.group, split.world, split.rank = None, world, rank
            split.device, split._own, split._opened = torch.device("cpu"), [], []
            ptrs = split._exchange(split._alloc(64))
            result_q.put((rank, ptrs, calls))
    except Exception as e:  # report instead of leaving the peer waiting for the queue
        result_q.put((rank, repr(e), []))
        raise
    finally:
        dist.destroy_process_group()


def _run_two(target, *args):
    import sys
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, list(sys.path), *args, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return results


def test_peer_split_exchange_pointers_in_rank_order():
    (_, p0, c0), (_, p1, c1) = _run_two(_peer_exchange_worker, -1)
    assert p0 == [0x1000, 0x9001] and p1 == [0x9000, 0x2000]
    assert ("open", 1) in c0 and ("open", 0) in c1


def test_peer_split_mapping_failure_raises_on_every_rank_and_releases():
    """Rank 1 cannot map rank 0's buffer: both ranks raise PeerSplitUnavailable (none
    is left in a collective), rank 0 unmaps what it opened, both free their own."""
    (_, o0, c0), (_, o1, c1) = _run_two(_peer_exchange_worker, 1)
    assert o0 == "unavailable" and o1 == "unavailable"
    assert c0 == [("alloc", 0x1000), ("open", 1), ("close", 0x9001), ("free", 0x1000)]
    assert c1 == [("alloc", 0x2000), ("free", 0x2000)]
