"""Prequantized checkpoints: files written by the reference's own save node
(tests/golden/ckpt_*.safetensors, from make_checkpoint_golden.py) load into
Int4ConvRotLinear and save back byte for byte (int4_ops.py:223-284,
int4_save.py:78-158). CPU only; the GPU forward of the loaded layers is in
test_gpu_checkpoint.py.
"""
import json
import os
import struct

import pytest
import torch

from _int4 import checkpoint
from _int4.linear import Int4ConvRotLinear

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYERS = [("double_blocks.0.img_attn.qkv", 512, 192, True),
          ("double_blocks.0.img_mlp.0", 320, 256, False),
          ("single_blocks.0.linear2", 256, 128, True)]


def fixture(fmt):
    return os.path.join(GOLD, f"ckpt_{fmt}.safetensors")


def file_content(path):
    """(header, data bytes) of a safetensors file. The header is compared as parsed
    JSON: safetensors writes the ``__metadata__`` entries in hash-map order, which
    changes from one process to the next even for the same writer and model. The
    tensor entries (names, dtypes, shapes, offsets) and every data byte must match."""
    raw = open(path, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    return json.loads(raw[8:8 + n]), raw[8 + n:]


def build_model(device="cpu"):
    """The fixture's module tree, quantized layers built before the loader knows their precision."""
    dm = torch.nn.Module()
    for name, k, n, has_bias in LAYERS:
        parent = dm
        parts = name.split(".")
        for p in parts[:-1]:
            if not hasattr(parent, p):
                parent.add_module(p, torch.nn.Module())
            parent = getattr(parent, p)
        parent.add_module(parts[-1], Int4ConvRotLinear(k, n, bias=has_bias, device=device))
    dm.add_module("img_in", torch.nn.Linear(64, 128, dtype=torch.bfloat16, device=device))
    dm.register_buffer("final_norm_scale", torch.zeros(192, dtype=torch.bfloat16, device=device))
    return dm


def load_fixture(fmt, device="cpu"):
    sd, meta = checkpoint.load_checkpoint(fixture(fmt))
    model = build_model(device)
    result = model.load_state_dict(sd, strict=True)
    assert not result.missing_keys and not result.unexpected_keys
    return model, meta


@pytest.mark.parametrize("fmt", ["native", "legacy"])
def test_reference_file_round_trips_byte_identical(tmp_path, fmt):
    model, meta = load_fixture(fmt)
    out = tmp_path / "resaved.safetensors"
    checkpoint.save_checkpoint(model, str(out), native=fmt == "native", source_metadata=meta)
    assert file_content(str(out)) == file_content(fixture(fmt))


def test_format_conversion_matches_the_reference_writer(tmp_path):
    """native -> legacy and legacy -> native give the reference's file of the other format."""
    model, meta = load_fixture("native")
    out = tmp_path / "as_legacy.safetensors"
    checkpoint.save_checkpoint(model, str(out), native=False, source_metadata=meta)
    assert file_content(str(out)) == file_content(fixture("legacy"))
    model, meta = load_fixture("legacy")
    meta = {k: v for k, v in meta.items() if k not in (checkpoint.FORMAT_TAG, checkpoint.PRECISION_TAG)}
    out = tmp_path / "as_native.safetensors"
    checkpoint.save_checkpoint(model, str(out), native=True, source_metadata=meta)
    assert file_content(str(out)) == file_content(fixture("native"))


def test_loaded_layers_take_precision_and_groupsize_from_the_file():
    for fmt in ("native", "legacy"):
        model, meta = load_fixture(fmt)
        qkv = model.get_submodule("double_blocks.0.img_attn.qkv")
        mlp = model.get_submodule("double_blocks.0.img_mlp.0")
        l2 = model.get_submodule("single_blocks.0.linear2")
        assert (qkv._qmode, qkv._qgs, tuple(qkv._q.shape)) == ("int4", 256, (192, 256))
        assert (mlp._qmode, mlp._qgs, tuple(mlp._q.shape), mlp.bias) == ("int4", 64, (256, 160), None)
        assert (l2._qmode, l2._qgs, tuple(l2._q.shape), tuple(l2._qs.shape)) == ("int8", 256, (128, 256), (128,))
        assert qkv.bias.dtype == torch.float16 and qkv._qs.dtype == torch.float32
    assert json.loads(meta[checkpoint.PRECISION_TAG]) == {
        "double_blocks.0.img_attn.qkv": "int4", "double_blocks.0.img_mlp.0": "int4",
        "single_blocks.0.linear2": "int8"}
    assert meta[checkpoint.FORMAT_TAG] == "2"


def test_take_prequantized_rules():
    q = torch.zeros(8, 128, dtype=torch.int8)
    sd = {"l.weight": q, "l.weight_scale": torch.ones(8, 1, dtype=torch.float16), "l.bias": torch.ones(8)}
    pw = checkpoint.take_prequantized(sd, "l.", 256)
    assert pw.mode == "int4" and pw.groupsize == 256 and pw.scale.shape == (8,) and pw.scale.dtype == torch.float32
    assert pw.bias.dtype == torch.float16 and sd == {}                     # keys consumed
    sd = {"l.weight": torch.zeros(8, 320, dtype=torch.int8), "l.weight_scale": torch.ones(8)}
    assert checkpoint.take_prequantized(sd, "l.", 320).mode == "int8"        # K columns: int8
    assert checkpoint.take_prequantized({"l.weight": q, "l.weight_scale": torch.ones(8)}, "l.", 200) is None
    tag = checkpoint.quant_tag("int4", 64)
    assert bytes(tag.tolist()) == b'{"format": "convrot_w4a4", "convrot_groupsize": 64}'
    sd = {"l.weight": q, "l.weight_scale": torch.ones(8), "l.comfy_quant": tag}
    assert checkpoint.take_prequantized(sd, "l.", 256).groupsize == 64       # the tag wins
    for conf in ({"format": "float8_e4m3fn"}, {"format": "int8_tensorwise", "convrot_groupsize": 256}):
        bad = torch.tensor(list(json.dumps(conf).encode()), dtype=torch.uint8)
        sd = {"l.weight": torch.zeros(8, 256, dtype=torch.int8), "l.weight_scale": torch.ones(8), "l.comfy_quant": bad}
        assert checkpoint.take_prequantized(sd, "l.", 256) is None and len(sd) == 3   # left for a plain load
    garbled = torch.tensor([0xFF, 0x00], dtype=torch.uint8)                  # unreadable tag: pick_groupsize
    sd = {"l.weight": q, "l.weight_scale": torch.ones(8), "l.comfy_quant": garbled}
    assert checkpoint.take_prequantized(sd, "l.", 256).groupsize == 256


def test_module_rejects_foreign_layouts():
    m = Int4ConvRotLinear(256, 8)
    with pytest.raises(RuntimeError, match="not a ConvRot"):
        m.load_state_dict({"weight": torch.zeros(8, 100, dtype=torch.int8), "weight_scale": torch.ones(8),
                           "bias": torch.zeros(8)})
    with pytest.raises(RuntimeError, match="Missing key"):
        m.load_state_dict({"bias": torch.zeros(8)})
    with pytest.raises(RuntimeError, match="Unexpected key"):
        m.load_state_dict({"weight": torch.zeros(8, 128, dtype=torch.int8), "weight_scale": torch.ones(8),
                           "bias": torch.zeros(8), "extra": torch.zeros(1)})


def test_single_layer_model_saves_unprefixed_keys(tmp_path):
    m = Int4ConvRotLinear(256, 8, bias=False, mode="int8")
    sd, meta = checkpoint.checkpoint_state(m, native=False)
    assert sorted(sd) == ["weight", "weight_scale"] and sd["weight"].shape == (8, 256)
    assert json.loads(meta[checkpoint.PRECISION_TAG]) == {"": "int8"}
