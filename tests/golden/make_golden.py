"""Generate the golden vectors in this folder from the reference's own eager code.

Run where the reference checkout is available::

    python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

It imports the reference package ``_int4`` (eager.py, _codec.py) directly from
its source tree under a private module name and runs its CPU torch functions on
seeded inputs. The outputs are written as ``.npz`` files next to this script;
the tests read only those files, so the reference is not needed to run them.

Reference functions exercised (paths relative to the reference project):
  _int4/_codec.py:19-36   _pack_int4_row_major / _unpack_int4_row_major
  _int4/eager.py:20-46    _build_hadamard
  _int4/eager.py:65-79    _rotate_activation
  _int4/eager.py:112-120  quantize_signed_int4_rowwise
  _int4/eager.py:123-135  quantize_convrot_w4a4_weight (fp16 weight, as int4_ops.py:342-349)
  _int4/eager.py:154-169  int4_linear
  _int4/eager.py:172-197  convrot_w4a4_linear
  _int4/int8_eager.py:22-27  quantize_signed_int8_rowwise (W8A8 tier)
  _int4/int8_eager.py:30-47  quantize_convrot_w8a8_weight (fp16 weight, as int4_ops.py:339-342)
  _int4/int8_eager.py:60-89  convrot_w8a8_linear

``--only int8`` rewrites int8.npz alone.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(path: str):
    pkg = os.path.join(path, "_int4")
    spec = importlib.util.spec_from_file_location(
        "convrot_reference_int4", os.path.join(pkg, "__init__.py"),
        submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["convrot_reference_int4"] = mod
    spec.loader.exec_module(mod)
    return mod


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def store(t: torch.Tensor) -> np.ndarray:
    """Activation storage form: bf16 as uint16 bits, others as numpy floats."""
    if t.dtype == torch.bfloat16:
        return bf16_bits(t)
    return t.numpy().copy()


def activation(gen: torch.Generator, m: int, k: int, outlier_frac: float = 0.01) -> torch.Tensor:
    """N(0,1) activations with a seeded 1% of channels scaled x20 (config-0 recipe)."""
    x = torch.randn(m, k, generator=gen)
    n_out = max(1, int(k * outlier_frac))
    idx = torch.randperm(k, generator=gen)[:n_out]
    x[:, idx] *= 20.0
    return x


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference project checkout")
    ap.add_argument("--only", choices=["int8"], default=None, help="write one file only")
    args = ap.parse_args()
    ref = load_reference(args.reference)
    eager, codec = ref.eager, ref._codec
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if args.only == "int8":
        write_int8(ref)
        return

    # 1. codec: every nibble value at every position parity
    gen = torch.Generator().manual_seed(11)
    vals = torch.randint(-8, 8, (6, 64), generator=gen, dtype=torch.int8)
    vals[0, :16] = torch.arange(-8, 8, dtype=torch.int8)
    vals[1, :16] = torch.arange(7, -9, -1, dtype=torch.int8)
    packed = codec._pack_int4_row_major(vals)
    np.savez_compressed(os.path.join(HERE, "codec.npz"), values=vals.numpy(),
                        packed=packed.numpy(), unpacked=codec._unpack_int4_row_major(packed).numpy())

    # 2. Hadamard sign patterns (entries are exactly +-1/sqrt(G) in fp32)
    had = {}
    for g in (16, 64, 256):
        h = eager._build_hadamard(g, dtype=torch.float32)
        had[f"signs_{g}"] = torch.sign(h).to(torch.int8).numpy()
        had[f"scale_{g}"] = np.float32(h[0, 0].abs().item())
    np.savez_compressed(os.path.join(HERE, "hadamard.npz"), **had)

    # 3. activation rotation + quantization, per group size and dtype
    cases = {}
    specs = [
        ("g256_bf16", 256, 768, torch.bfloat16),
        ("g64_bf16", 64, 320, torch.bfloat16),
        ("g16_bf16", 16, 160, torch.bfloat16),
        ("g256_f16", 256, 512, torch.float16),
        ("g256_f32", 256, 512, torch.float32),
        ("cfg0_bf16", 256, 3072, torch.bfloat16),
    ]
    for name, g, k, dt in specs:
        gen = torch.Generator().manual_seed(100 + k + g)
        m = 40 if name != "cfg0_bf16" else 64
        x = activation(gen, m, k).to(dt)
        if dt != torch.float16:
            x[3] = 0                      # all-zero row -> absmax clamp
        x[5] = 0
        x[5, 7] = 3.0                     # single spike
        x[6] = x[6] * 1e-30 if dt != torch.float16 else x[6]   # tiny magnitudes
        h = eager._build_hadamard(g, device="cpu", dtype=dt)
        xr = eager._rotate_activation(x, h, g).contiguous()
        q, s = eager.quantize_signed_int4_rowwise(xr)
        cases[f"{name}_x"] = store(x)
        cases[f"{name}_xrot"] = store(xr)
        cases[f"{name}_q"] = q.numpy()
        cases[f"{name}_scale"] = s.numpy()
        cases[f"{name}_meta"] = np.array([g, k, {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[dt]])
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **cases)

    # 4. weights (fp16 quantization like the reference loader) + full eager linear
    lin = {}
    for name, g, k, n, m in [("g256", 256, 768, 96, 48), ("g64", 64, 320, 64, 33),
                             ("g16", 16, 192, 48, 17), ("cfg0", 256, 3072, 128, 64)]:
        gen = torch.Generator().manual_seed(7 + k + n)
        w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(n, generator=gen) * 0.01).to(torch.bfloat16)
        x = activation(gen, m, k).to(torch.bfloat16)
        qw, ws = eager.quantize_convrot_w4a4_weight(w.to(torch.float16), g)
        out = eager.convrot_w4a4_linear(x, qw, ws, bias=bias.to(torch.float16), convrot_groupsize=g)
        lin[f"{name}_w"] = bf16_bits(w)
        lin[f"{name}_bias"] = bf16_bits(bias)
        lin[f"{name}_x"] = bf16_bits(x)
        lin[f"{name}_qw"] = qw.numpy()
        lin[f"{name}_ws"] = ws.numpy()
        lin[f"{name}_out"] = bf16_bits(out)
        lin[f"{name}_meta"] = np.array([g, k, n, m])
    np.savez_compressed(os.path.join(HERE, "linear.npz"), **lin)
    write_int8(ref)
    print("golden vectors written to", HERE)


def write_int8(ref) -> None:
    """5. the W8A8 tier (_int4/int8_eager.py): activation int8 quantization of the
    rotated tensor, fp16 weight quantization and the eager W8A8 linear."""
    eager, i8 = ref.eager, ref.int8_eager
    out = {}
    for name, g, k, dt in [("g256_bf16", 256, 768, torch.bfloat16), ("g64_bf16", 64, 512, torch.bfloat16),
                           ("g16_bf16", 16, 160, torch.bfloat16), ("g256_f16", 256, 512, torch.float16),
                           ("cfg0_bf16", 256, 3072, torch.bfloat16)]:
        gen = torch.Generator().manual_seed(300 + k + g)
        m = 40 if name != "cfg0_bf16" else 64
        x = activation(gen, m, k).to(dt)
        x[3] = 0                          # all-zero row -> absmax clamp
        x[5] = 0
        x[5, 7] = 3.0                     # single spike
        h = eager._build_hadamard(g, device="cpu", dtype=dt)
        xr = eager._rotate_activation(x, h, g).contiguous()
        q, sc = i8.quantize_signed_int8_rowwise(xr)
        out[f"q_{name}_x"] = store(x)
        out[f"q_{name}_xrot"] = store(xr)
        out[f"q_{name}_q"] = q.numpy()
        out[f"q_{name}_scale"] = sc.numpy()
        out[f"q_{name}_meta"] = np.array([g, k, {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}[dt]])
    for name, g, k, n, m in [("g256", 256, 768, 96, 48), ("g64", 64, 512, 64, 33), ("cfg0", 256, 3072, 128, 64)]:
        gen = torch.Generator().manual_seed(400 + k + n)
        w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(n, generator=gen) * 0.01).to(torch.bfloat16)
        x = activation(gen, m, k).to(torch.bfloat16)
        qw, ws = i8.quantize_convrot_w8a8_weight(w.to(torch.float16), g)
        y = i8.convrot_w8a8_linear(x, qw, ws, bias=bias.to(torch.float16), convrot_groupsize=g)
        out[f"l_{name}_w"] = bf16_bits(w)
        out[f"l_{name}_bias"] = bf16_bits(bias)
        out[f"l_{name}_x"] = bf16_bits(x)
        out[f"l_{name}_qw"] = qw.numpy()
        out[f"l_{name}_ws"] = ws.numpy()
        out[f"l_{name}_out"] = bf16_bits(y)
        out[f"l_{name}_meta"] = np.array([g, k, n, m])
    np.savez_compressed(os.path.join(HERE, "int8.npz"), **out)


if __name__ == "__main__":
    main()
