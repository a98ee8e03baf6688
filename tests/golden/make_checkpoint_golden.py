"""Generate the prequantized-checkpoint fixtures in this folder with the reference's
own save node.

Run where the reference checkout is available::

    python tests/golden/make_checkpoint_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

It imports the reference's ``int4_save.py`` (``INT4ConvRotModelSave.save``,
int4_save.py:78-158) and its ``_int4`` package (weight quantizers,
_int4/eager.py:123-135 and _int4/int8_eager.py:30-47) from the source tree, and
saves a small synthetic diffusion model in both formats:

* ``ckpt_native.safetensors`` -- per-layer ``comfy_quant`` tags;
* ``ckpt_legacy.safetensors`` -- header markers, no tags.

The model holds the three quantized layer kinds the loader accepts (int4 at
G = 256 and at G = 64, int8), one unquantized bf16 Linear and a norm weight, in
the node's loaded-layer form (``_q``, ``_qs``, ``_qmode``, ``_qgs``, fp16 bias,
no ``weight``). ComfyUI itself is not installed, so its three modules that
int4_save.py imports are stand-ins here: ``comfy.model_management.load_models_gpu``
does nothing (the model is already on the CPU), ``folder_paths`` points at this
folder, and ``comfy.utils.save_torch_file`` is ComfyUI's (unpinned) behaviour:
``safetensors.torch.save_file(sd, path, metadata=metadata)``.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE_METADATA = {"modelspec.title": "synthetic convrot fixture", "modelspec.architecture": "flux-like"}
# (name, in_features, out_features, mode, bias)
LAYERS = [("double_blocks.0.img_attn.qkv", 512, 192, "int4", True),
          ("double_blocks.0.img_mlp.0", 320, 256, "int4", False),
          ("single_blocks.0.linear2", 256, 128, "int8", True)]


def install_comfy_stand_ins(out_dir: str) -> None:
    comfy = types.ModuleType("comfy")
    mm = types.ModuleType("comfy.model_management")
    mm.load_models_gpu = lambda models, force_full_load=False: None
    utils = types.ModuleType("comfy.utils")

    def save_torch_file(sd, path, metadata=None):
        if metadata is not None:
            save_file(sd, path, metadata=metadata)
        else:
            save_file(sd, path)
    utils.save_torch_file = save_torch_file
    comfy.model_management, comfy.utils = mm, utils
    fp = types.ModuleType("folder_paths")
    fp.get_output_directory = lambda: out_dir
    fp.get_save_image_path = lambda prefix, output_dir: (output_dir, prefix, 0, "", prefix)
    sys.modules.update({"comfy": comfy, "comfy.model_management": mm, "comfy.utils": utils,
                        "folder_paths": fp})


def load_module(name: str, path: str, package_dir: str | None = None):
    spec = importlib.util.spec_from_file_location(
        name, path, submodule_search_locations=[package_dir] if package_dir else None)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


class QuantizedLinear(torch.nn.Module):
    """The node's Linear after an on-the-fly quantization: weight None, codes in plain attributes."""

    def __init__(self, q, qs, mode, gs, bias):
        super().__init__()
        self.weight = None
        self.bias = torch.nn.Parameter(bias, requires_grad=False) if bias is not None else None
        self._q, self._qs, self._qmode, self._qgs = q, qs, mode, gs


def build_model(ref_int4):
    g = torch.Generator().manual_seed(7)
    dm = torch.nn.Module()
    for name, k, n, mode, has_bias in LAYERS:
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.float16)
        gs = ref_int4.pick_groupsize(k) if hasattr(ref_int4, "pick_groupsize") else (256 if k % 256 == 0 else 64)
        if mode == "int4":
            q, qs = ref_int4.eager.quantize_convrot_w4a4_weight(w, gs)
        else:
            q, qs = ref_int4.int8_eager.quantize_convrot_w8a8_weight(w, gs)
        bias = (torch.randn(n, generator=g) * 0.01).to(torch.float16) if has_bias else None
        parent = dm
        parts = name.split(".")
        for p in parts[:-1]:
            if not hasattr(parent, p):
                parent.add_module(p, torch.nn.Module())
            parent = getattr(parent, p)
        parent.add_module(parts[-1], QuantizedLinear(q.contiguous(), qs.float().contiguous(), mode, gs, bias))
    dm.add_module("img_in", torch.nn.Linear(64, 128, dtype=torch.bfloat16))
    with torch.no_grad():
        dm.img_in.weight.copy_(torch.randn(128, 64, generator=g).to(torch.bfloat16))
        dm.img_in.bias.copy_(torch.randn(128, generator=g).to(torch.bfloat16))
    dm.register_buffer("final_norm_scale", torch.randn(192, generator=g).to(torch.bfloat16))
    model = types.SimpleNamespace(model=types.SimpleNamespace(diffusion_model=dm),
                                  _safetensors_metadata=dict(SOURCE_METADATA))
    return model


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    ref = os.path.abspath(args.reference)
    install_comfy_stand_ins(HERE)
    ref_int4 = load_module("convrot_reference_int4", os.path.join(ref, "_int4", "__init__.py"),
                           os.path.join(ref, "_int4"))
    saver = load_module("convrot_reference_int4_save", os.path.join(ref, "int4_save.py"))
    model = build_model(ref_int4)
    node = saver.INT4ConvRotModelSave()
    for fmt in ("native", "legacy"):
        node.save(model, f"ckpt_{fmt}", save_format=fmt)
        written = os.path.join(HERE, f"ckpt_{fmt}_00000_.safetensors")
        os.replace(written, os.path.join(HERE, f"ckpt_{fmt}.safetensors"))
        print("wrote", os.path.join(HERE, f"ckpt_{fmt}.safetensors"))


if __name__ == "__main__":
    main()
