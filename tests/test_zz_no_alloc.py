"""The no-allocation linear entry, ck_convrot_w4a4_linear_noalloc.

It must give exactly what ck_convrot_w4a4_linear gives with a caller
workspace, on consecutive calls that reuse its static scratch, and refuse
sizes beyond the scratch before touching CUDA. This file is collected last so
it also runs after every other GPU test in one process (and passes alone).
"""
import os

import numpy as np
import pytest
import torch

from _int4 import build as libbuild
from _int4 import cuda_loader

SCRATCH = 128 << 20


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(libbuild.lib_path()):
        libbuild.build()
    return cuda_loader.library()


def test_noalloc_rejects_sizes_beyond_the_scratch(lib):
    """Checked on the host before any CUDA call (runs without a GPU)."""
    f = lib.ck_convrot_w4a4_linear_noalloc
    m, k = 32768, 8192                     # 128 MiB of codes + scales: over the limit
    assert lib.ck_convrot_w4a4_linear_workspace_size(m, k) > SCRATCH
    assert f(256, 1, 256, 256, 0, 0, 256, 1, m, 64, k, 256, None) == -1
    assert b"128 MiB" in lib.ck_convrot_last_error()
    assert lib.ck_convrot_w4a4_linear_workspace_size(18432, 12288) <= SCRATCH
    assert f(256, 1, 256, 256, 0, 0, 256, 1, 0, 64, k, 256, None) == 0      # empty: no launch
    assert f(256, 1, 256, 256, 0, 7, 256, 1, 4, 64, 256, 256, None) == -1   # bad bias dtype


def _case(m, k, n, seed, bias_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(m, k, generator=g) * 3).to(torch.bfloat16).cuda()
    wq = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8).cuda()
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).to(bias_dtype).cuda()
    return x, wq, ws, bias


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n", [(1, 3072, 3072), (4, 768, 520), (300, 3072, 1280), (4608, 3072, 3072)])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(lib, m, k, n):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    a = _case(m, k, n, seed=m)
    b = _case(m, k, n, seed=m + 1, bias_dtype=torch.float32)
    # two calls in a row on one stream: the second overwrites the scratch the first used
    na = cuda_loader.convrot_w4a4_linear_noalloc(*a, torch.bfloat16, 256)
    nb = cuda_loader.convrot_w4a4_linear_noalloc(*b, torch.float32, 256)
    wa = cuda_loader.convrot_w4a4_linear(*a, torch.bfloat16, 256)
    wb = cuda_loader.convrot_w4a4_linear(*b, torch.float32, 256)
    torch.cuda.synchronize()
    assert torch.equal(na, wa)
    assert torch.equal(nb, wb)
    assert not torch.equal(na.float(), nb)
    assert cuda_loader.device_status() == 0


@pytest.mark.gpu
def test_noalloc_inside_a_cuda_graph_after_first_call(lib):
    """After the first (setup) call the entry only launches kernels: capturable."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    x, wq, ws, bias = _case(96, 1024, 640, seed=3)
    first = cuda_loader.convrot_w4a4_linear_noalloc(x, wq, ws, bias, torch.bfloat16, 256)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = cuda_loader.convrot_w4a4_linear_noalloc(x, wq, ws, bias, torch.bfloat16, 256)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    ref = cuda_loader.convrot_w4a4_linear(x, wq, ws, bias, torch.bfloat16, 256)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().view(torch.int16).numpy(), ref.cpu().view(torch.int16).numpy())
