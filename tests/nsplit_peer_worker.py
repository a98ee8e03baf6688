"""Worker of tests/test_gpu_nsplit_peers.py (one process per GPU, launched by torchrun).

Checks the peer-memory column split against the unsplit layer, bit for bit, on
every rank: config-4-shaped layers with and without the Dynamic-LoRA side path,
ragged token counts (one and two row chunks), several calls in a row (the two
output buffers in turn)
and chained calls in a CUDA graph; then the device status word must be clear.
Prints one line "ok <rank>" per rank on success.
"""
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "comfyui-int4-convrot-rdna4_b200"))

import _int4  # noqa: E402
from _int4 import cuda_loader  # noqa: E402
from _int4.nsplit import (PeerColumnSplit, convrot_w4a4_linear_peer_split, peer_split_supported,  # noqa: E402
                          shard_adapters, shard_rows)


def layer(m, k, n, r, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: k // 100]] *= 20
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16)
    adapters = []
    if r:
        adapters = [((torch.randn(r, k, generator=g) * 0.01).to(torch.float16).to(device),
                     (torch.randn(n, r, generator=g) * 0.01).to(torch.float16).to(device), 64.0 / r)]
    qw, ws = _int4.quantize_convrot_w4a4_weight(w.to(device), 256)
    return x.to(torch.bfloat16).to(device), qw, ws, bias.to(device), adapters


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=device)
    split = PeerColumnSplit(device=device)
    for m, k, n, r in ((4608, 12288, 3072, 64), (9001, 3072, 3072, 64), (1000, 3072, 12288, 0),
                       (333, 3072, 1024, 16)):
        x, qw, ws, bias, adapters = layer(m, k, n, r, seed=m + k + n, device=device)
        ref = _int4.convrot_w4a4_linear_lora(x, qw, ws, bias, adapters, 256) if adapters else \
            _int4.convrot_w4a4_linear(x, qw, ws, bias=bias, convrot_groupsize=256)
        q, w, b = shard_rows(qw, ws, bias, rank, world)
        ad = shard_adapters(adapters, rank, world)
        assert peer_split_supported(x, q.shape[0], 256)
        outs = [convrot_w4a4_linear_peer_split(x, q, w, b, ad, split) for _ in range(3)]
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), f"rank {rank}: {(m, k, n, r)} differs"
    # chained in a CUDA graph: each call's input is the previous call's output
    x, qw, ws, bias, _ = layer(256, 3072, 3072, 0, seed=7, device=device)
    q, w, b = shard_rows(qw, ws, bias, rank, world)
    chain_ref = [x]
    for _ in range(4):
        chain_ref.append(_int4.convrot_w4a4_linear(chain_ref[-1], qw, ws, bias=bias, convrot_groupsize=256))
    for _ in range(2):                              # warm: the shape's buffers exist before capture
        convrot_w4a4_linear_peer_split(x, q, w, b, (), split)
    torch.cuda.synchronize()
    dist.barrier()
    static_x = x.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = static_x
        ys = []
        for _ in range(4):
            y = convrot_w4a4_linear_peer_split(y, q, w, b, (), split)
            ys.append(y)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        for got, want in zip(ys, chain_ref[1:]):
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"rank {rank}: graph chain differs"
    del graph
    assert cuda_loader.device_status(device) == 0
    split.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"ok {rank}", flush=True)


if __name__ == "__main__":
    main()
