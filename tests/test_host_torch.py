"""The torch-side helpers of the drop-in ``_int4`` package against the reference goldens (CPU).

``_int4.eager.quantize_convrot_w4a4_weight`` defines the weight bytes at load
time, so on the same device it must reproduce the reference exactly
(reference: _int4/eager.py:123-135, _int4/_codec.py:19-36).
"""
import os

import numpy as np
import pytest
import torch

from _int4 import _codec, eager, int8_eager
from oracle import eager_torch

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bits_to_bf16(a):
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)


def test_codec_roundtrip_vs_reference():
    g = np.load(os.path.join(GOLD, "codec.npz"))
    vals = torch.from_numpy(g["values"])
    packed = _codec._pack_int4_row_major(vals)
    assert np.array_equal(packed.numpy(), g["packed"])
    assert np.array_equal(_codec._unpack_int4_row_major(packed).numpy(), g["unpacked"])


@pytest.mark.parametrize("g", [16, 64, 256])
def test_hadamard_vs_reference(g):
    h = np.load(os.path.join(GOLD, "hadamard.npz"))
    hm = eager._build_hadamard(g, dtype=torch.float32)
    assert np.array_equal(torch.sign(hm).to(torch.int8).numpy(), h[f"signs_{g}"])
    assert hm.abs().unique().item() == h[f"scale_{g}"]


@pytest.mark.parametrize("case", ["g256", "g64", "g16", "cfg0"])
def test_weight_quant_bytes_match_reference(case):
    lin = np.load(os.path.join(GOLD, "linear.npz"))
    grp = int(lin[f"{case}_meta"][0])
    w = bits_to_bf16(lin[f"{case}_w"]).to(torch.float16)
    qw, ws = eager.quantize_convrot_w4a4_weight(w, grp)
    assert np.array_equal(qw.numpy(), lin[f"{case}_qw"])
    assert np.array_equal(ws.numpy().view(np.uint32), lin[f"{case}_ws"].view(np.uint32))


@pytest.mark.parametrize("case", ["g256_bf16", "g64_bf16", "g256_f16"])
def test_rowwise_quant_bytes_match_reference(case):
    q = np.load(os.path.join(GOLD, "quant.npz"))
    dt = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}[int(q[f"{case}_meta"][2])]
    xr = q[f"{case}_xrot"]
    xr_t = bits_to_bf16(xr) if dt == torch.bfloat16 else torch.from_numpy(xr)
    packed, s = eager.quantize_signed_int4_rowwise(xr_t)
    assert np.array_equal(packed.numpy(), q[f"{case}_q"])
    assert np.array_equal(s.numpy().view(np.uint32), q[f"{case}_scale"].view(np.uint32))


def test_stochastic_rounding_is_seeded():
    w = torch.randn(32, 256, dtype=torch.float16)
    a = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=1234)
    b = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=1234)
    c = eager.quantize_convrot_w4a4_weight(w, 256, stochastic_rounding=0)
    assert torch.equal(a[0], b[0])
    assert not torch.equal(a[0], c[0])


def test_dequantize_inverts_quantize():
    w = torch.randn(64, 512) * 0.02
    qw, ws = eager.quantize_convrot_w4a4_weight(w, 256)
    wd = eager.dequantize_convrot_w4a4_weight(qw, ws, 256)
    assert (wd - w).norm() / w.norm() < 0.2


def test_int8_tier_roundtrip():
    w = torch.randn(48, 256) * 0.02
    q, s = int8_eager.quantize_convrot_w8a8_weight(w, 256)
    assert q.dtype == torch.int8 and q.shape == (48, 256)
    wd = int8_eager.dequantize_convrot_w8a8_weight(q, s, 256)
    assert (wd - w).norm() / w.norm() < 0.02
    x = torch.randn(5, 256)
    out = eager_torch.convrot_w8a8_linear(x, q, s)
    ref = x @ w.T
    assert (out - ref).norm() / ref.norm() < 0.05
