"""Prequantized ConvRot checkpoints, in the node's on-disk format.

The node saves a quantized model with ``INT4ConvRotModelSave.save``
(int4_save.py:78-158) and loads it back without re-quantizing through
``Int4ConvRotOps.Linear._load_prequantized`` (int4_ops.py:223-284). This module
restates both for models built from :class:`_int4.linear.Int4ConvRotLinear`, so
a file written by the node loads here, and a file saved from here is the file
the node would have written: same tensor names, dtypes, shapes and bytes, same
header metadata (safetensors writes the metadata entries in hash-map order, so
their byte order in the header differs from one write to the next, for the
node's writer as for this one).

Per quantized Linear ``<key>`` (the module's name in the diffusion model):

* ``<key>.weight``: int8, ``[N, K/2]`` for int4 (two nibbles per byte,
  ``_int4/_codec.py``) or ``[N, K]`` for int8;
* ``<key>.weight_scale``: f32 per-row scale, ``[N]``; the native format stores
  the int8 scale as ``[N, 1]``;
* ``<key>.comfy_quant`` (native format only): uint8 bytes of the JSON tag
  ``{"format": "convrot_w4a4", "convrot_groupsize": G}`` or
  ``{"format": "int8_tensorwise", "convrot": true, "convrot_groupsize": G}``;
* ``<key>.bias``: fp16 (the load path casts it, int4_ops.py:268-271).

The legacy format has no tags; its header carries ``{"convrot_w4a4": "2",
"convrot_precision": JSON {key: "int4"|"int8"}}``. Both formats keep the source
file's str->str metadata. On load, int4 and int8 are told apart by the stored
column count, and the group size comes from the tag or, without one, from
``pick_groupsize(in_features)``.
"""
from __future__ import annotations

import json
from typing import NamedTuple

import torch

# Header markers of the legacy format (int4_save.py:27-29); the strings are the format.
FORMAT_TAG = "convrot_w4a4"
FORMAT_VERSION = "2"
PRECISION_TAG = "convrot_precision"


class PrequantizedWeight(NamedTuple):
    q: torch.Tensor            # int8 [N, K/2] (int4) or [N, K] (int8)
    scale: torch.Tensor        # f32 [N]
    groupsize: int
    mode: str                  # "int4" or "int8"
    bias: torch.Tensor | None  # fp16 [N]


def quant_tag(mode: str, groupsize: int) -> torch.Tensor:
    """The per-layer ``comfy_quant`` tag of the native format (int4_save.py:119-127)."""
    if mode == "int8":
        conf = {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": int(groupsize)}
    else:
        conf = {"format": "convrot_w4a4", "convrot_groupsize": int(groupsize)}
    return torch.tensor(list(json.dumps(conf).encode("utf-8")), dtype=torch.uint8)


def _tag_groupsize(tag: torch.Tensor):
    """Group size from a ``comfy_quant`` tag; False if the tag names a layout the
    ConvRot kernels cannot run; None if it gives no usable group size."""
    try:
        conf = json.loads(bytes(tag.cpu().numpy().tolist()).decode("utf-8"))
        fmt = conf.get("format")
        if fmt not in ("convrot_w4a4", "int8_tensorwise"):
            return False
        if fmt == "int8_tensorwise" and not conf.get("convrot", False):
            return False                      # plain (unrotated) int8
        return int(conf.get("convrot_groupsize", 0)) or None
    except Exception:
        return None


def take_prequantized(state_dict: dict, prefix: str, in_features: int,
                      device=None) -> PrequantizedWeight | None:
    """Consume ``prefix``'s quantized weight from ``state_dict`` (int4_ops.py:223-271).

    Returns None, leaving ``state_dict`` untouched, when the stored layout is not
    one of the two ConvRot forms. Otherwise pops the weight, scale, tag and bias
    keys and returns them on ``device`` (scale f32 flattened, bias fp16).
    """
    from . import pick_groupsize
    wkey, skey, tkey, bkey = (prefix + s for s in ("weight", "weight_scale", "comfy_quant", "bias"))
    w = state_dict.get(wkey)
    if w is None or w.dim() != 2 or skey not in state_dict:
        return None
    cols = w.shape[-1]
    if cols == in_features:
        mode = "int8"
    elif cols * 2 == in_features:
        mode = "int4"
    else:
        return None
    gs = None
    tag = state_dict.get(tkey)
    if tag is not None:
        gs = _tag_groupsize(tag)
        if gs is False:
            return None
    if gs is None:
        gs = pick_groupsize(in_features)
    if gs is None:
        return None
    device = torch.device(device) if device is not None else w.device
    q = w.to(device).contiguous()
    scale = state_dict[skey].to(device, torch.float32).reshape(-1).contiguous()
    for k in (wkey, skey, tkey):
        state_dict.pop(k, None)
    bias = state_dict.pop(bkey).to(device, torch.float16) if bkey in state_dict else None
    return PrequantizedWeight(q, scale, gs, mode, bias)


def put_quantized(sd: dict, prefix: str, q: torch.Tensor, scale: torch.Tensor, mode: str,
                  groupsize: int, native: bool = True) -> None:
    """Write one quantized layer's tensors into ``sd`` under ``prefix`` (the
    layer's name and a dot) (int4_save.py:110-133)."""
    scale = scale.detach().float().to("cpu").contiguous()
    sd[prefix + "weight"] = q.detach().to("cpu").contiguous()
    if native:
        if mode == "int8":
            scale = scale.reshape(-1, 1).contiguous()
        sd[prefix + "comfy_quant"] = quant_tag(mode, groupsize)
    sd[prefix + "weight_scale"] = scale


def header_metadata(precision: dict, native: bool, source_metadata: dict | None = None) -> dict:
    """Header of the saved file (int4_save.py:146-155): the source file's str->str
    entries, plus the legacy markers when not native."""
    meta = {k: v for k, v in (source_metadata or {}).items() if isinstance(k, str) and isinstance(v, str)}
    if not native:
        meta[FORMAT_TAG] = FORMAT_VERSION
        meta[PRECISION_TAG] = json.dumps(precision)
    return meta


def checkpoint_state(model: torch.nn.Module, native: bool = True,
                     source_metadata: dict | None = None) -> tuple[dict, dict]:
    """(tensors, metadata) of ``model`` as the save node writes them: every other
    parameter and buffer as is, each Int4ConvRotLinear in the quantized form."""
    from .linear import Int4ConvRotLinear
    sd = {}
    for k, v in model.state_dict().items():
        if isinstance(v, torch.Tensor):
            sd[k] = v.detach().to("cpu").contiguous()
    precision = {}
    for name, module in model.named_modules():
        if isinstance(module, Int4ConvRotLinear):
            prefix = name + "." if name else ""
            for k in ("weight", "weight_scale", "comfy_quant"):
                sd.pop(prefix + k, None)
            put_quantized(sd, prefix, module._q, module._qs, module._qmode, module._qgs, native)
            precision[name] = module._qmode
    return sd, header_metadata(precision, native, source_metadata)


def save_checkpoint(model: torch.nn.Module, path: str, native: bool = True,
                    source_metadata: dict | None = None) -> None:
    """Write ``model`` to ``path`` as a prequantized ConvRot safetensors file."""
    from safetensors.torch import save_file
    sd, meta = checkpoint_state(model, native, source_metadata)
    save_file(sd, path, metadata=meta)


def load_checkpoint(path: str) -> tuple[dict, dict]:
    """(state_dict, header metadata) of a safetensors file; pass the metadata back
    to :func:`save_checkpoint` to keep it on a round trip."""
    from safetensors import safe_open
    from safetensors.torch import load_file
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
    return load_file(path), meta
