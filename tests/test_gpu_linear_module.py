"""GPU tests of the node-style quantized Linear (int4_ops.py:366-383 contract) and of the
N-column split on real GPUs (NCCL, skipped with fewer than 2 GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import convrot_oracle as orc

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_linear_module_matches_oracle_and_float(need_gpu):
    from _int4.linear import Int4ConvRotLinear
    torch.manual_seed(0)
    lin = torch.nn.Linear(768, 320).to(torch.bfloat16)
    mod = Int4ConvRotLinear.from_linear(lin, device="cuda")
    x = torch.randn(3, 40, 768).to(torch.bfloat16).cuda()
    out = mod(x)
    assert out.shape == (3, 40, 320) and out.dtype == torch.bfloat16
    ref = orc.convrot_w4a4_linear(bits(x.reshape(-1, 768)), mod._q.cpu().numpy(), mod._qs.cpu().numpy(),
                                  mod.bias.float().cpu().numpy(), 256)
    assert np.array_equal(bits(out.reshape(-1, 320)), ref)
    fl = (x.float() @ lin.weight.float().cuda().t() + lin.bias.float().cuda())
    # W4A4 quantization error against the unquantized layer (sanity bound only)
    assert (out.float() - fl).norm() / fl.norm() < 0.35


def test_linear_module_dynamic_lora(need_gpu):
    from _int4.linear import Int4ConvRotLinear
    torch.manual_seed(1)
    lin = torch.nn.Linear(512, 256).to(torch.bfloat16)
    mod = Int4ConvRotLinear.from_linear(lin, device="cuda")
    x = torch.randn(64, 512).to(torch.bfloat16).cuda()
    base = mod(x).float()
    down, up = torch.randn(16, 512) * 0.05, torch.randn(256, 16) * 0.05
    mod.set_dynamic_lora([(down, up, 16.0, 0.8)])
    out = mod(x).float()
    side = 0.8 * ((x.float() @ down.cuda().bfloat16().float().t()) @ up.cuda().bfloat16().float().t())
    assert ((out - base) - side).norm() / side.norm() < 2e-2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank, world, port, path, q):
    import sys
    sys.path[:0] = path
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import _int4
        from _int4.nsplit import convrot_w4a4_linear_nsplit, shard_rows
        g = torch.Generator().manual_seed(5)
        x = torch.randn(300, 1024, generator=g).to(torch.bfloat16).cuda()
        w = (torch.randn(512, 1024, generator=g) * 0.02).to(torch.float16).cuda()
        b = (torch.randn(512, generator=g) * 0.01).to(torch.float16).cuda()
        qw, ws = _int4.quantize_convrot_w4a4_weight(w, 256)
        full = _int4.convrot_w4a4_linear(x, qw, ws, b)
        out = convrot_w4a4_linear_nsplit(x, *shard_rows(qw, ws, b, rank, world), 256)
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(out, full))))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_nsplit_nccl_two_gpus_bit_identical(need_gpu):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import sys
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, list(sys.path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is True for r in res), res
