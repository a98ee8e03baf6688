"""Pin the CPU oracle against golden vectors made by the reference's eager code.

Golden files come from ``tests/golden/make_golden.py`` (reference functions:
``_int4/_codec.py:19-36``, ``_int4/eager.py:20-197``).
"""
import os

import numpy as np
import pytest

from oracle import convrot_oracle as orc

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DTYPES = {0: "bf16", 1: "f16", 2: "f32"}


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_codec_matches_reference():
    g = load("codec.npz")
    assert np.array_equal(orc.pack_int4(g["values"]), g["packed"])
    assert np.array_equal(orc.unpack_int4(g["packed"]), g["unpacked"])
    assert np.array_equal(orc.unpack_int4(orc.pack_int4(g["values"])), g["values"])


def test_codec_rejects_odd_width():
    with pytest.raises(ValueError):
        orc.pack_int4(np.zeros((2, 3), np.int8))


@pytest.mark.parametrize("g", [16, 64, 256])
def test_hadamard_matches_reference(g):
    h = load("hadamard.npz")
    assert np.array_equal(orc.hadamard_signs(g), h[f"signs_{g}"])
    assert np.float32(1.0 / np.sqrt(g)) == h[f"scale_{g}"]
    # orthogonal and symmetric
    hm = orc.hadamard(g)
    assert np.allclose(hm @ hm.T, np.eye(g))
    assert np.array_equal(hm, hm.T)


def test_hadamard_rejects_bad_size():
    for bad in (2, 8, 32, 100):
        with pytest.raises(ValueError):
            orc.hadamard_signs(bad)


def test_pick_groupsize():
    assert orc.pick_groupsize(3072) == 256
    assert orc.pick_groupsize(320) == 64
    assert orc.pick_groupsize(48) == 16
    assert orc.pick_groupsize(40) is None


QUANT_CASES = ["g256_bf16", "g64_bf16", "g16_bf16", "g256_f16", "g256_f32", "cfg0_bf16"]


@pytest.mark.parametrize("case", QUANT_CASES)
def test_quantizer_bit_exact_given_reference_rotation(case):
    """Codes and scales are bit-exact when fed the reference's rotated tensor."""
    g = load("quant.npz")
    dt = DTYPES[int(g[f"{case}_meta"][2])]
    q, s = orc.quantize_rowwise(g[f"{case}_xrot"], dt)
    assert np.array_equal(q, orc.unpack_int4(g[f"{case}_q"]))
    assert np.array_equal(s.view(np.uint32), g[f"{case}_scale"].view(np.uint32))


@pytest.mark.parametrize("case", QUANT_CASES)
def test_rotation_matches_reference(case):
    """Kernel-order fp32 butterflies vs the reference's library matmul.

    Both round once to the activation dtype; they may disagree only where the
    exact value sits within fp32 noise of a rounding tie.
    """
    g = load("quant.npz")
    grp, _, dti = (int(v) for v in g[f"{case}_meta"])
    dt = DTYPES[dti]
    xr = orc.to_f32(orc.rotate(g[f"{case}_x"], grp, dt), dt)
    ref = orc.to_f32(g[f"{case}_xrot"], dt)
    if dt == "f32":
        tol = 1e-5 * np.abs(ref).max(axis=1, keepdims=True)
        assert np.all(np.abs(xr - ref) <= tol)
    else:
        mism = np.count_nonzero(xr != ref)
        assert mism <= max(2, xr.size // 50000), mism


@pytest.mark.parametrize("case", QUANT_CASES)
def test_fused_quant_codes_vs_reference(case):
    """End-to-end codes: rotation ties may move a code by at most one step."""
    g = load("quant.npz")
    grp, _, dti = (int(v) for v in g[f"{case}_meta"])
    dt = DTYPES[dti]
    xp, s = orc.convrot_quant_int4(g[f"{case}_x"], grp, dt)
    q = orc.unpack_int4(xp).astype(np.int32)
    ref = orc.unpack_int4(g[f"{case}_q"]).astype(np.int32)
    diff = np.abs(q - ref)
    assert diff.max() <= 1
    assert np.count_nonzero(diff) <= max(1, q.size // 100000)


LIN_CASES = ["g256", "g64", "g16", "cfg0"]


@pytest.mark.parametrize("case", LIN_CASES)
def test_exact_accumulator_and_output_vs_reference(case):
    lin = load("linear.npz")
    grp, k, n, m = (int(v) for v in lin[f"{case}_meta"])
    x, qw, ws = lin[f"{case}_x"], lin[f"{case}_qw"], lin[f"{case}_ws"]
    bias = orc.bf16_bits_to_f32(lin[f"{case}_bias"])
    xp, xs = orc.convrot_quant_int4(x, grp, "bf16")
    acc = orc.int4_gemm_acc(xp, qw)
    exact = orc.unpack_int4(xp).astype(np.int64) @ orc.unpack_int4(qw).astype(np.int64).T
    assert np.array_equal(acc, exact)
    out = orc.bf16_bits_to_f32(orc.convrot_w4a4_linear(x, qw, ws, bias, grp))
    ref = orc.bf16_bits_to_f32(lin[f"{case}_out"])
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-2, rel


@pytest.mark.parametrize("case", LIN_CASES)
def test_weight_quant_vs_reference(case):
    """Oracle weight quant (fp16, kernel butterfly order) vs the reference fp16 matmul."""
    lin = load("linear.npz")
    grp = int(lin[f"{case}_meta"][0])
    w16 = orc.bf16_bits_to_f32(lin[f"{case}_w"]).astype(np.float16)
    qw, ws = orc.quantize_weight(w16, grp, "f16")
    q = orc.unpack_int4(qw).astype(np.int32)
    ref = orc.unpack_int4(lin[f"{case}_qw"]).astype(np.int32)
    assert np.abs(q - ref).max() <= 1
    assert np.count_nonzero(q != ref) <= max(2, q.size // 20000)
    assert np.allclose(ws, lin[f"{case}_ws"], rtol=1e-3)


def test_dequantize_roundtrip():
    lin = load("linear.npz")
    grp = int(lin["g256_meta"][0])
    w = orc.bf16_bits_to_f32(lin["g256_w"]).astype(np.float64)
    wd = orc.dequantize_weight(lin["g256_qw"], lin["g256_ws"], grp)
    rel = np.linalg.norm(wd - w) / np.linalg.norm(w)
    assert rel < 0.2, rel


def test_bf16_rounding_helpers():
    vals = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, 1e-40, 0.0], np.float32)
    r = orc.round_to_bf16(vals)
    assert r[0] == 1.0 and r[1] == 1.0          # tie -> even
    assert r[2] == np.float32(1.0078125)
    assert r[3] == -2.5
    assert np.isnan(orc.round_to_bf16(np.array([np.nan], np.float32)))[0]


def test_reciprocal_quant_identity_bf16():
    """bf16(fp32(x * fp32(1/s))) == bf16(fp32(x / s)) for bf16 x, s.

    The CUDA quantizer multiplies by the reciprocal of the row scale; this
    checks the identity on every bf16 x in [-8s, 8s] for a sweep of scales.
    """
    rng = np.random.default_rng(0)
    pos = np.arange(0x0080, 0x7F80, dtype=np.uint16)            # all positive normal bf16
    scales = orc.bf16_bits_to_f32(np.concatenate([
        rng.choice(pos, 400, replace=False), np.array([0x3F80, 0x3E12, 0x2EDC, 0x0080], np.uint16)]))
    allx = orc.bf16_bits_to_f32(pos)
    for s in scales:
        with np.errstate(over="ignore"):                          # 8 * s is inf for the largest s
            x = allx[allx <= 8 * s]
        x = np.concatenate([x, -x])
        a = orc.round_to_bf16(x / s)
        b = orc.round_to_bf16(x * (np.float32(1.0) / s))
        assert np.array_equal(a, b), s


def test_scale_multiply_identity_bf16():
    """bf16(fp32(a / 7)) == bf16(fp32(a * fp32(1/7))) for every positive bf16 a."""
    a = orc.bf16_bits_to_f32(np.arange(0x0001, 0x7F80, dtype=np.uint16))
    assert np.array_equal(orc.round_to_bf16(a / np.float32(7)),
                          orc.round_to_bf16(a * (np.float32(1) / np.float32(7))))


# ------------------------------------------------------------------ W8A8 tier (int8.npz)

I8_QUANT = ["g256_bf16", "g64_bf16", "g16_bf16", "g256_f16", "cfg0_bf16"]


@pytest.mark.parametrize("case", I8_QUANT)
def test_int8_quantizer_bit_exact_given_reference_rotation(case):
    """The int8 quantizer (_int4/int8_eager.py:22-27) on the reference's rotated tensor."""
    g = load("int8.npz")
    dt = DTYPES[int(g[f"q_{case}_meta"][2])]
    q, s = orc.quantize_rowwise_int8(g[f"q_{case}_xrot"], dt)
    assert np.array_equal(q, g[f"q_{case}_q"])
    assert np.array_equal(s.view(np.uint32), g[f"q_{case}_scale"].view(np.uint32))


@pytest.mark.parametrize("case", I8_QUANT)
def test_int8_codes_vs_reference_end_to_end(case):
    """Kernel-order rotation + int8 quantizer: rotation ties move a code by at most one."""
    g = load("int8.npz")
    grp, _, dti = (int(v) for v in g[f"q_{case}_meta"])
    dt = DTYPES[dti]
    q, s = orc.convrot_quant_int8(g[f"q_{case}_x"], grp, dt)
    diff = np.abs(q.astype(np.int32) - g[f"q_{case}_q"].astype(np.int32))
    assert diff.max() <= 1
    assert np.count_nonzero(diff) <= max(2, q.size // 20000)


@pytest.mark.parametrize("case", ["g256", "g64", "cfg0"])
def test_int8_linear_vs_reference(case):
    """Exact int32 accumulator + fp32 epilogue vs the reference's eager W8A8 linear
    (fp32 matmul of int8 values, then bf16): within 1e-2 relative L2."""
    g = load("int8.npz")
    grp, k, n, m = (int(v) for v in g[f"l_{case}_meta"])
    x, qw, ws = g[f"l_{case}_x"], g[f"l_{case}_qw"], g[f"l_{case}_ws"]
    bias = orc.bf16_bits_to_f32(g[f"l_{case}_bias"])
    xq, xs = orc.convrot_quant_int8(x, grp, "bf16")
    acc = orc.int8_gemm_acc(xq, qw)
    assert np.array_equal(acc, xq.astype(np.int64) @ qw.astype(np.int64).T)
    out = orc.bf16_bits_to_f32(orc.convrot_w8a8_linear(x, qw, ws, bias, grp))
    ref = orc.bf16_bits_to_f32(g[f"l_{case}_out"])
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 1e-2, rel


@pytest.mark.parametrize("case", ["g256", "g64", "cfg0"])
def test_int8_weight_quant_torch_matches_reference_bytes(case):
    """_int4.int8_eager.quantize_convrot_w8a8_weight gives the reference's bytes."""
    import torch
    from _int4 import int8_eager
    g = load("int8.npz")
    grp = int(g[f"l_{case}_meta"][0])
    w = torch.from_numpy(g[f"l_{case}_w"].view(np.int16)).view(torch.bfloat16).to(torch.float16)
    qw, ws = int8_eager.quantize_convrot_w8a8_weight(w, grp)
    assert np.array_equal(qw.numpy(), g[f"l_{case}_qw"])
    assert np.array_equal(ws.numpy().view(np.uint32), g[f"l_{case}_ws"].view(np.uint32))


def _bf16(a):
    import torch
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)


@pytest.mark.parametrize("case", LIN_CASES)
def test_eager_torch_port_matches_reference_linear_bits(case):
    """oracle.eager_torch (the CPU baseline's fallback) reproduces the reference's
    eager W4A4 linear bit for bit on the CPU."""
    from oracle import eager_torch
    lin = load("linear.npz")
    grp = int(lin[f"{case}_meta"][0])
    import torch
    out = eager_torch.convrot_w4a4_linear(_bf16(lin[f"{case}_x"]), torch.from_numpy(lin[f"{case}_qw"]),
                                          torch.from_numpy(lin[f"{case}_ws"]), _bf16(lin[f"{case}_bias"]), grp)
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), lin[f"{case}_out"])


@pytest.mark.parametrize("case", ["g256", "g64", "cfg0"])
def test_eager_torch_port_matches_reference_w8a8_linear_bits(case):
    from oracle import eager_torch
    import torch
    g = load("int8.npz")
    grp = int(g[f"l_{case}_meta"][0])
    out = eager_torch.convrot_w8a8_linear(_bf16(g[f"l_{case}_x"]), torch.from_numpy(g[f"l_{case}_qw"]),
                                          torch.from_numpy(g[f"l_{case}_ws"]), _bf16(g[f"l_{case}_bias"]), grp)
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), g[f"l_{case}_out"])
