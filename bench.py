"""Benchmark of the B200 ConvRot W4A4 linear path.

One step = the Flux-class double-block linear set at M = 4608 tokens:
QKV 3072->9216, attention-out 3072->3072, MLP-up 3072->12288 and MLP-down
12288->3072, each a full W4A4 forward through the public API
(``_int4.convrot_w4a4_linear``: fused rotate+quantize kernel, then the tcgen05
GEMM with the dequant + bias epilogue). Metric: W4A4 linear TOPS (2*M*N*K ops
per layer; integer MACs count as two ops).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU: the step's 4608 tokens are
split over the ranks (4608/N rows each, weights replicated, no collective on
the data path), strong scaling; the step time is the max over ranks. Extra
keys of the same line: ``replicas`` (every rank runs all 4608 tokens: weak
scaling), ``nsplit`` (config 4's 12288->3072 layer with its LoRA side path,
split by output columns over the ranks and gathered over NVLink), and at
N = 1 ``dit_step`` (one denoising step of a synthetic Flux-architecture DiT,
config 2) plus the per-kernel roofline probes.

``--impl reference`` times the reference's own CPU implementation of the path,
``_int4.eager.convrot_w4a4_linear`` imported from ``baseline/_ref`` (installed
by ``oracle/ref_install.py``; its torch restatement ``oracle/eager_torch.py``
when that is absent), on every host core, rank 0 only, on the same 4608-token
step.

Timing: inputs are resident in HBM; L2 is flushed (a 256 MiB write) before
every timed step; each step is bracketed by CUDA events on the launching
stream and the K durations are summed.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "comfyui-int4-convrot-rdna4_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

M_TOKENS = 4608
HIDDEN = 3072
LAYERS = [("qkv", 3072, 9216), ("attn_out", 3072, 3072), ("mlp_up", 3072, 12288), ("mlp_down", 12288, 3072)]
GROUP = 256
LORA_RANK = 64
REF_BUDGET_S = 150.0          # bound on the reference arm's whole --steps/--warmup run


def flux_dit_layers():
    """Every int4 Linear of one forward of a Flux-architecture DiT (config 2): 19 double
    blocks (image stream at 4096 tokens, text stream at 512) and 38 single blocks at
    4608 tokens, hidden 3072, MLP x4; the modulation Linears and vector_in run at M = 1.
    The embedders and the final layer stay bf16 (the reference loader's skip list)."""
    layers = [("vector_in.in_layer", 1, 768, 3072, 0), ("vector_in.out_layer", 1, 3072, 3072, 0)]
    for d in range(19):
        for stream, m in (("img", 4096), ("txt", 512)):
            layers += [(f"d{d}.{stream}_attn.qkv", m, 3072, 9216, 0), (f"d{d}.{stream}_attn.proj", m, 3072, 3072, 0),
                       (f"d{d}.{stream}_mlp.0", m, 3072, 12288, 0), (f"d{d}.{stream}_mlp.2", m, 12288, 3072, 0),
                       (f"d{d}.{stream}_mod.lin", 1, 3072, 18432, 0)]
    for b in range(38):
        layers += [(f"s{b}.linear1", 4608, 3072, 21504, 0), (f"s{b}.linear2", 4608, 15360, 3072, 0),
                   (f"s{b}.modulation.lin", 1, 3072, 9216, 0)]
    return layers


# Per-config step: (name, M, K, N, lora_rank). Config 1 is the default (the
# BASELINE metric's configuration); the others are the BASELINE parity configs.
WORKLOADS = {
    2: ("config2_flux_dit_linears", flux_dit_layers()),
    0: ("config0_single_linear", [("linear", 512, 3072, 3072, 0)]),
    1: ("config1_flux_double_block_linears", [(name, M_TOKENS, k, n, 0) for name, k, n in LAYERS]),
    3: ("config3_zimage_mlp_token_sweep", [(f"{nm}_m{m}", m, k, n, 0) for m in (1024, 4096, 16384)
                                           for nm, k, n in (("mlp_up", 3840, 15360), ("mlp_down", 15360, 3840))]),
    4: ("config4_dynamic_lora_m18432", [("mlp_up", 18432, 3072, 12288, LORA_RANK),
                                        ("mlp_down", 18432, 12288, 3072, LORA_RANK)]),
}
METRIC = "w4a4_linear_tops"
UNIT = "TOPS"
L2_FLUSH_BYTES = 256 << 20


def step_ops(m: int) -> int:
    """Config-1 ops for m tokens (used by the CPU arm)."""
    return sum(2 * m * n * k for _, k, n in LAYERS)


def layer_ops(m, k, n, r) -> int:
    """int4 GEMM ops, plus the LoRA side path's 2*M*r*(K+N) when present."""
    return 2 * m * n * k + (2 * m * r * (k + n) if r else 0)


def shard_range(m: int, rank: int, world: int):
    """Rows [lo, hi) of m tokens that `rank` of `world` runs (token split)."""
    return rank * m // world, (rank + 1) * m // world


def workload_config(cfg_id=1, world=1, extra=None):
    name, layers = WORKLOADS[cfg_id]
    if cfg_id == 2:
        shapes = sorted({(m, k, n) for _, m, k, n, _ in layers}, reverse=True)
        desc = {"linears": len(layers), "blocks": "19 double (img M=4096, txt M=512) + 38 single (M=4608)",
                "shapes": [f"M={m} {k}->{n}" for m, k, n in shapes],
                "weights": "random packed int4 codes and scales (the kernels' work does not depend on the values)"}
    else:
        desc = {"layers": {lname: f"M={m} {k}->{n}" + (f" +LoRA r={r}" if r else "") for lname, m, k, n, r in layers}}
    cfg = {"workload": name, **desc, "convrot_groupsize": GROUP,
           "l2": "flushed before every timed step (256 MiB write)"}
    if cfg_id == 2 or world == 1:
        cfg["parallelism"] = "single GPU"
    else:
        cfg["parallelism"] = f"token split x{world}: each rank runs 1/{world} of every layer's rows, weights replicated"
    if cfg_id == 1:
        cfg.update({"tokens": M_TOKENS, "tokens_per_gpu": M_TOKENS // world, "hidden": HIDDEN})
    if extra:
        cfg.update(extra)
    return cfg


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic():
    """Per-launch DRAM bytes (read + write) of the dominant GEMM, from the committed
    summary of one ncu capture of it (profiles/roofline_traffic.json)."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if not os.path.exists(path):
        return {}
    with open(path) as f:
        return json.load(f)


def synth_activation(m, k, gen, device):
    x = torch.randn(m, k, generator=gen)
    idx = torch.randperm(k, generator=gen)[: max(1, k // 100)]
    x[:, idx] *= 20.0
    return x.to(torch.bfloat16).to(device)


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []            # (host time the line arrived, line)
        self.window = None

    def start(self):
        """Start sampling every 20 ms; returns once the first sample has arrived."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._drain, daemon=True).start()
        except OSError:
            self.proc = None
            return
        deadline = time.time() + 10.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.01)

    def _drain(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, t0: float, t1: float):
        """Host-time window of the timed region: only samples inside it count."""
        self.window = (t0, t1)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.05)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        lines = list(self.lines)
        if self.window is not None:
            inside = [(t, l) for t, l in lines if self.window[0] <= t <= self.window[1] + 0.03]
            lines = inside if inside else lines[-1:]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU arm

def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_impl():
    """The reference's own CPU implementation of the path: (weight quantizer, linear,
    kind, description). The reference package from baseline/_ref when installed,
    else the torch restatement of the same eager code (bit-identical on the CPU)."""
    root = os.path.join(ROOT, "baseline", "_ref", "_int4")
    if os.path.exists(os.path.join(root, "eager.py")):
        import importlib.util
        spec = importlib.util.spec_from_file_location("convrot_reference_int4", os.path.join(root, "__init__.py"),
                                                      submodule_search_locations=[root])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        return (mod.quantize_convrot_w4a4_weight, mod.eager.convrot_w4a4_linear, "reference",
                "the reference's _int4.eager.convrot_w4a4_linear (baseline/_ref), torch CPU")
    from _int4.eager import quantize_convrot_w4a4_weight
    from oracle import eager_torch
    return (quantize_convrot_w4a4_weight, eager_torch.convrot_w4a4_linear, "port",
            "oracle/eager_torch.convrot_w4a4_linear (torch restatement of _int4/eager.py:172-197), torch CPU")


class CpuWorkload:
    """Config 1's four layers on the host through `linear`, inputs built once."""

    def __init__(self, quant_weight, linear, seed: int = 0):
        self.linear = linear
        gen = torch.Generator().manual_seed(seed)
        self.layers = []
        for _, k, n in LAYERS:
            w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.float16)
            qw, ws = quant_weight(w, GROUP)
            bias = (torch.randn(n, generator=gen) * 0.01).to(torch.bfloat16).to(torch.float16)
            self.layers.append((synth_activation(M_TOKENS, k, gen, "cpu"), qw, ws, bias))

    def step(self, rows: int = M_TOKENS) -> float:
        t0 = time.perf_counter()
        for x, qw, ws, bias in self.layers:
            self.linear(x[:rows], qw, ws, bias, GROUP)
        return time.perf_counter() - t0


def cpu_sample(budget_s: float):
    """CPU baseline of the default run: full 4608-token steps through the reference's
    CPU path for about `budget_s` seconds (at least 3), median."""
    quant_weight, linear, kind, what = reference_impl()
    torch.set_num_threads(host_cores())
    wl = CpuWorkload(quant_weight, linear)
    wl.step()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or time.perf_counter() < t_end:
        times.append(wl.step())
    t = statistics.median(times)
    return {"value": step_ops(M_TOKENS) / t / 1e12, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
            "ms_per_step": t * 1e3,
            "sample": f"all {M_TOKENS} tokens through the four layers, median of {len(times)} steps: {what}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    quant_weight, linear, kind, what = reference_impl()
    torch.set_num_threads(host_cores())
    wl = CpuWorkload(quant_weight, linear)
    t_first = wl.step()                              # first warm-up step, also sizes the sample
    rows = M_TOKENS
    runs = args.steps + args.warmup - 1
    if t_first * runs > REF_BUDGET_S:                # keep the whole run within a few minutes
        rows = max(256, int(M_TOKENS * REF_BUDGET_S / (t_first * runs)) // 256 * 256)
    for _ in range(args.warmup - 1):
        wl.step(rows)
    times = [wl.step(rows) for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = step_ops(rows) / t / 1e12
    cfg = workload_config(1, world)
    if rows != M_TOKENS:
        cfg["cpu_tokens_per_step"] = rows
    sample = f"{rows} of {M_TOKENS} tokens per step through all four layers: {what}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int4", "data": "synthetic (seeded; config-1 shapes and value distributions)",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm

def build_layers(device, seed, cfg_id=1):
    """Quantized layers (the same weights on every rank) and device-resident inputs of
    one step of config `cfg_id`."""
    import _int4
    gen = torch.Generator().manual_seed(seed)
    layers = []
    xs = {}
    dgen = torch.Generator(device=device).manual_seed(seed)
    for name, m, k, n, r in WORKLOADS[cfg_id][1]:
        if cfg_id == 2:
            # 304 layers, 5.9 GB of int4 weights: random packed codes and scales
            w = None
            qw = torch.randint(-128, 128, (n, k // 2), generator=dgen, dtype=torch.int8, device=device)
            ws = torch.rand(n, generator=dgen, device=device) * 1e-3 + 1e-5
        else:
            w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).to(device)
            qw, ws = _int4.quantize_convrot_w4a4_weight(w.to(torch.float16), GROUP)
        bias = (torch.randn(n, generator=gen) * 0.01).to(torch.bfloat16).to(torch.float16).to(device)
        layer = {"name": name, "m": m, "k": k, "n": n, "r": r, "qw": qw, "ws": ws, "bias": bias,
                 "bias32": bias.float().contiguous()}
        if r:
            down = (torch.randn(r, k, generator=gen) * 0.01).to(torch.bfloat16).to(device)
            up = (torch.randn(n, r, generator=gen) * 0.01).to(torch.bfloat16).to(device)
            layer["adapters"] = [(down, up, 64.0 / r)]            # alpha = 64
        layers.append(layer)
        del w
        if (m, k) not in xs:
            xs[(m, k)] = synth_activation(m, k, gen, device)
        layer["key"] = (m, k)
    return layers, xs


def run_layer(l, x):
    import _int4
    if l["r"]:
        return _int4.convrot_w4a4_linear_lora(x, l["qw"], l["ws"], l["bias"], l["adapters"], GROUP)
    return _int4.convrot_w4a4_linear(x, l["qw"], l["ws"], l["bias"], GROUP)


def device_step(layers, xs):
    """One step through the public API on device-resident inputs."""
    return [run_layer(l, xs[l["key"]]) for l in layers]


def time_kernel_batch(fns, iters, flush, stream):
    """Average device time (ms) per launch of back-to-back launches over distinct
    inputs (together larger than L2), captured in one CUDA graph: the launch
    latency of a single short kernel stays out of the figure."""
    for fn in fns:
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for fn in fns:
            fn()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(iters):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        b.synchronize()
        best = min(best, a.elapsed_time(b) / len(fns))
    del graph
    return best


def time_kernel(fn, iters, flush, stream):
    """Average device time (ms) of the work fn() launches, L2 flushed before each run.

    fn is captured once in a CUDA graph and replayed between two events on the
    launching stream, so host-side launch work stays out of the measurement.
    """
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.replay()
        b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    del graph
    return total / iters


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def timed_steps(step_fn, steps, flush, stream, world, device):
    """Device ms per step (max over ranks) of `steps` steps, L2 flushed before each,
    barrier + synchronize on both sides."""
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    events = []
    for _ in range(steps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step_fn()
        b.record(stream)
        events.append((a, b))
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = sum(a.elapsed_time(b) for a, b in events) / steps
    return max_over_ranks(ms, world, device)


def graphed(step_fn, flush):
    """Capture one call of step_fn in a CUDA graph (after one eager call, which builds any
    per-weight state outside the graph); returns a replaying callable and the graph."""
    step_fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = step_fn()
    torch.cuda.synchronize()

    def replay():
        graph.replay()
        return outs
    for _ in range(2):
        flush()
        replay()
    torch.cuda.synchronize()
    return replay, graph


def roofline_probes(layers, xs, device, flush, stream):
    """Per-kernel roofline figures of config 1 on this GPU (rank 0, N = 1)."""
    import _int4
    from _int4 import cuda_loader as ck
    from _int4 import weight_cache
    extras = {}
    peaks, peak_src = load_peaks()
    up = next(l for l in layers if l["name"] == "mlp_up")
    m, k, n = up["m"], up["k"], up["n"]
    iters = 10
    # time the kernels the public linear runs for this layer: by default (packed
    # weights, M > 128) the A8 form -- unpacked activation codes, packed weights
    # expanded in the kernel; with the opt-in unpacked-weight cache the int8 pair
    # GEMM on sign-extended codes of both operands; for few rows the packed GEMM
    x = xs[up["key"]]
    if _int4._use_unpacked(x, up["qw"], GROUP):
        quant = ck.convrot_quant_int4_unpacked
        wq = weight_cache.unpacked(up["qw"])
        xq, xsc = quant(x, GROUP)
        gemm = lambda: ck.int8_convrot_gemm(xq, wq, xsc, up["ws"], up["bias32"], torch.bfloat16)
        gemm_name, code_bytes, form = "int8 pair GEMM on cached unpacked weight codes", (1, 1), "unpacked"
    elif _int4._use_a8(x, GROUP):
        quant = ck.convrot_quant_int4_unpacked
        xq, xsc = quant(x, GROUP)
        gemm = lambda: ck.int4_convrot_gemm_a8(xq, up["qw"], xsc, up["ws"], up["bias"], torch.bfloat16)
        gemm_name, code_bytes, form = ("A8T GEMM (int8 activation codes by TMA, packed int4 weights expanded into "
                                       "tensor memory)", (1, 0.5), "a8")
    else:
        quant = ck.convrot_quant_int4
        xq, xsc = quant(x, GROUP)
        gemm = lambda: ck.int4_convrot_gemm(xq, up["qw"], xsc, up["ws"], up["bias32"], torch.bfloat16)
        gemm_name, code_bytes, form = "int4 pair GEMM on packed codes", (0.5, 0.5), "packed"
    gemm_ms = time_kernel(gemm, iters, flush, stream)
    # 8 distinct activations (8 x 28 MB, well beyond L2), launched back to back
    xq_in = [synth_activation(m, k, torch.Generator().manual_seed(100 + i), device) for i in range(8)]
    quant_ms = time_kernel_batch([lambda x=x: quant(x, GROUP) for x in xq_in], iters, flush, stream)
    del xq_in
    gemm_ops = 2 * m * n * k
    int8_peak = 2.0 * peaks["bf16_tflops"]           # dense int8 rate = 2x bf16 on B200
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    extras["roofline"] = {
        "kernel": f"{'int4_gemm_a8t_kernel' if form == 'a8' else 'int4_gemm_pair_kernel'}, {gemm_name} "
                  f"(MLP up 3072->12288, M=4608)",
        "bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
        "frac": achieved / int8_peak,
        "peak_source": f"2 x {peak_src} bf16 burst ({peaks['bf16_tflops']} TFLOP/s): B200 dense int8 rate",
        "ms_per_launch": gemm_ms,
        "traffic": load_traffic().get({"a8": "a8t_bytes_per_launch", "unpacked": "int8_pair_unpacked_bytes_per_launch",
                                       "packed": "int4_gemm_kernel_bytes_per_launch"}[form]),
        "traffic_note": "ncu dram read + write of one launch at this shape; the output fits in L2, so part of "
                        "its write-back lands after the kernel (profiles/a8t_mlp_up_m4608.md)",
        "algorithmic_bytes": (m * k + n * k) // 2 + 4 * m + 4 * n + 2 * n + 2 * m * n,
        "bytes_read_as_launched": int(code_bytes[0] * m * k + code_bytes[1] * n * k) + 4 * m + 4 * n + 2 * n
                                  + 2 * m * n,
    }
    qbytes = 2 * m * k + m * k // 2 + 4 * m          # W4A4 activation bytes (packed codes)
    extras["quant_kernel"] = {
        "kernel": f"convrot_quant_bf16_kernel{' (unpacked codes)' if form != 'packed' else ''} (K=3072, M=4608)",
        "bound": "hbm",
        "achieved": qbytes / (quant_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": qbytes / (quant_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "ms_per_launch": quant_ms,
        "bytes": "2MK read + MK/2 + 4M written (packed-code bytes, whatever form the codes take)",
        "timing": "8 launches back to back over distinct 28 MB inputs in one CUDA graph, per launch",
    }
    # small-M (weight-bound) layers at M = 1 / 16 / 64 / 128
    sm = {}
    for mm, kk, nn in ((1, 3072, 18432), (16, 3072, 18432), (64, 3072, 18432), (128, 3072, 18432),
                       (1, 12288, 3072), (64, 12288, 3072)):
        wsm = (torch.randn(nn, kk, device=device) * 0.02).to(torch.float16)
        qsm, wssm = _int4.quantize_convrot_w4a4_weight(wsm, GROUP)
        del wsm
        copies = max(2, math.ceil(400e6 / qsm.numel()))          # distinct weight copies beyond L2
        qsms = [qsm] + [qsm.roll(i, 0).contiguous() for i in range(1, copies)]
        xsm = synth_activation(mm, kk, torch.Generator().manual_seed(5), device)
        ms = time_kernel_batch([lambda q=q: _int4.convrot_w4a4_linear(xsm, q, wssm, None, GROUP) for q in qsms],
                               iters, flush, stream)
        del qsms
        wbytes = nn * kk // 2 + 4 * nn + mm * kk * 2 + 2 * mm * nn
        sm[f"M={mm} {kk}->{nn}"] = {"ms_per_call": ms, "achieved_gbs": wbytes / (ms * 1e-3) / 1e9,
                                    "frac": wbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]}
    first = sm["M=1 3072->18432"]
    extras["small_m"] = {
        "kernel": "public linear at M <= 128 (quantizer + int4 GEMV / swapped-tile GEMM), headline M=1 3072->18432",
        "bound": "hbm", "achieved": first["achieved_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": first["frac"], "ms_per_launch": first["ms_per_call"],
        "bytes": "packed weights + scales + bf16 activations + bf16 output",
        "timing": "calls back to back over distinct weight copies (>= 400 MB) in one CUDA graph, per call",
        "cases": sm,
    }
    return extras


# ---------------------------------------------------------------- config 2: a Flux DiT step

FLUX_SKIP = ("img_in", "time_in", "guidance_in", "txt_in", "final_layer")   # int4_loader.py:25-27 (flux2 list)


class FluxDiT:
    """Synthetic Flux-architecture DiT, random init.

    19 double-stream and 38 single-stream blocks, hidden 3072, 24 heads x 128,
    MLP ratio 4, RoPE over (t, h, w) axes of 16/56/56 dims. Every Linear with
    in_features >= 512 whose name matches no entry of the reference loader's
    flux skip list is an ``Int4ConvRotLinear`` (random packed codes and scales);
    the others are bf16. Attention is torch SDPA; norms, modulation, GELU and
    RoPE are torch ops in bf16 (fp32 inside the norms and RoPE).
    """

    def __init__(self, device, seed=0, double=19, single=38, hidden=3072, heads=24):
        from _int4.linear import Int4ConvRotLinear
        self.device, self.hidden, self.heads = device, hidden, heads
        self.gen = torch.Generator(device=device).manual_seed(seed)
        self.int4_layers = 0
        self.Q = Int4ConvRotLinear
        self.fused_ln = True

        def lin(name, k, n):
            if k >= 512 and not any(s in name for s in FLUX_SKIP):
                mod = Int4ConvRotLinear(k, n, True, device=device)
                lo = torch.randint(-7, 8, (n, k // 2), generator=self.gen, device=device, dtype=torch.int16)
                hi = torch.randint(-7, 8, (n, k // 2), generator=self.gen, device=device, dtype=torch.int16)
                mod._q.copy_(((lo & 0xF) | ((hi & 0xF) << 4)).to(torch.uint8).view(torch.int8))
                mod._qs.copy_(torch.rand(n, generator=self.gen, device=device) * 2e-3 + 4e-3)
                mod.bias.copy_(torch.randn(n, generator=self.gen, device=device) * 0.01)
                self.int4_layers += 1
                return mod
            w = (torch.randn(n, k, generator=self.gen, device=device) * (1.0 / math.sqrt(k))).to(torch.bfloat16)
            b = torch.zeros(n, device=device, dtype=torch.bfloat16)
            return lambda x: torch.nn.functional.linear(x, w, b)

        h = hidden
        self.img_in, self.txt_in = lin("img_in", 64, h), lin("txt_in", 4096, h)
        self.time_in = (lin("time_in.in_layer", 256, h), lin("time_in.out_layer", h, h))
        self.guidance_in = (lin("guidance_in.in_layer", 256, h), lin("guidance_in.out_layer", h, h))
        self.vector_in = (lin("vector_in.in_layer", 768, h), lin("vector_in.out_layer", h, h))
        self.double = []
        for i in range(double):
            blk = {}
            for s in ("img", "txt"):
                blk[s] = {"mod": lin(f"double_blocks.{i}.{s}_mod.lin", h, 6 * h),
                          "qkv": lin(f"double_blocks.{i}.{s}_attn.qkv", h, 3 * h),
                          "proj": lin(f"double_blocks.{i}.{s}_attn.proj", h, h),
                          "mlp0": lin(f"double_blocks.{i}.{s}_mlp.0", h, 4 * h),
                          "mlp2": lin(f"double_blocks.{i}.{s}_mlp.2", 4 * h, h),
                          "qn": torch.ones(128, device=device), "kn": torch.ones(128, device=device)}
            self.double.append(blk)
        self.single = [{"mod": lin(f"single_blocks.{i}.modulation.lin", h, 3 * h),
                        "linear1": lin(f"single_blocks.{i}.linear1", h, 3 * h + 4 * h),
                        "linear2": lin(f"single_blocks.{i}.linear2", h + 4 * h, h),
                        "qn": torch.ones(128, device=device), "kn": torch.ones(128, device=device)}
                       for i in range(single)]
        self.final_mod = lin("final_layer.adaLN_modulation.1", h, 2 * h)
        self.final = lin("final_layer.linear", h, 64)

    @staticmethod
    def _mlp_embed(pair, x):
        return pair[1](torch.nn.functional.silu(pair[0](x)))

    @staticmethod
    def _timestep_embedding(t, dim=256, max_period=10000.0):
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        args = (t.float() * 1000.0)[:, None] * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1).to(torch.bfloat16)

    def _rope(self, ids):
        """cos/sin [L, 64] of the (t, h, w) position axes, 16/56/56 dims, theta 10000."""
        parts = []
        for axis, d in enumerate((16, 56, 56)):
            freqs = 1.0 / (10000.0 ** (torch.arange(0, d, 2, dtype=torch.float64, device=ids.device) / d))
            parts.append(ids[:, axis:axis + 1].double() * freqs[None])
        ang = torch.cat(parts, dim=-1).float()
        return torch.cos(ang), torch.sin(ang)

    @staticmethod
    def _apply_rope(x, cos, sin):
        xf = x.float().reshape(*x.shape[:-1], -1, 2)
        x0, x1 = xf[..., 0], xf[..., 1]
        out = torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], dim=-1)
        return out.reshape(x.shape).to(x.dtype)

    @staticmethod
    def _rms(x, scale):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * scale).to(x.dtype)

    def _ln_mod(self, x, shift, scale):
        return torch.nn.functional.layer_norm(x, (self.hidden,), eps=1e-6) * (1 + scale) + shift

    def _ln_mod_lin(self, lin, x, shift, scale):
        """lin((1 + scale) * LayerNorm(x) + shift): int4 layers take the normalisation into their
        rotate + quantize pass (fused_ln), otherwise torch normalises first."""
        if self.fused_ln and isinstance(lin, self.Q):
            return lin.forward_lnmod(x, shift, scale, eps=1e-6)
        return lin(self._ln_mod(x, shift, scale))

    def _heads(self, qkv, qn, kn):
        L = qkv.shape[0]
        q, k, v = qkv.view(L, 3, self.heads, 128).permute(1, 2, 0, 3)
        return self._rms(q, qn), self._rms(k, kn), v

    def _attend(self, q, k, v, cos, sin):
        q, k = self._apply_rope(q, cos, sin), self._apply_rope(k, cos, sin)
        o = torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None])[0]
        return o.permute(1, 0, 2).reshape(q.shape[1], self.hidden)

    def forward(self, latent, txt, y, t, guidance):
        h = self.hidden
        c, hh, ww = latent.shape[1], latent.shape[2] // 2, latent.shape[3] // 2
        img = latent[0].view(c, hh, 2, ww, 2).permute(1, 3, 0, 2, 4).reshape(hh * ww, c * 4)
        img = self.img_in(img)
        txt = self.txt_in(txt[0])
        vec = (self._mlp_embed(self.time_in, self._timestep_embedding(t))
               + self._mlp_embed(self.guidance_in, self._timestep_embedding(guidance))
               + self._mlp_embed(self.vector_in, y))
        svec = torch.nn.functional.silu(vec)
        n_txt = txt.shape[0]
        ids = torch.zeros(n_txt + hh * ww, 3, device=latent.device)
        ids[n_txt:, 1] = torch.arange(hh, device=latent.device).repeat_interleave(ww).float()
        ids[n_txt:, 2] = torch.arange(ww, device=latent.device).repeat(hh).float()
        cos, sin = self._rope(ids)
        for blk in self.double:
            mods = {s: blk[s]["mod"](svec).chunk(6, dim=-1) for s in ("img", "txt")}
            streams = {"img": img, "txt": txt}
            qkv = {}
            for s in ("txt", "img"):
                sh, sc, _, _, _, _ = mods[s]
                qkv[s] = self._heads(self._ln_mod_lin(blk[s]["qkv"], streams[s], sh, sc), blk[s]["qn"], blk[s]["kn"])
            q, k, v = (torch.cat([qkv["txt"][i], qkv["img"][i]], dim=1) for i in range(3))
            attn = self._attend(q, k, v, cos, sin)
            outs = {"txt": attn[:n_txt], "img": attn[n_txt:]}
            for s in ("txt", "img"):
                _, _, g1, sh2, sc2, g2 = mods[s]
                x = streams[s] + g1 * blk[s]["proj"](outs[s])
                mlp = blk[s]["mlp2"](torch.nn.functional.gelu(self._ln_mod_lin(blk[s]["mlp0"], x, sh2, sc2),
                                                              approximate="tanh"))
                streams[s] = x + g2 * mlp
            img, txt = streams["img"], streams["txt"]
        x = torch.cat([txt, img], dim=0)
        for blk in self.single:
            sh, sc, g = blk["mod"](svec).chunk(3, dim=-1)
            lin1 = self._ln_mod_lin(blk["linear1"], x, sh, sc)
            q, k, v = self._heads(lin1[:, :3 * h], blk["qn"], blk["kn"])
            attn = self._attend(q, k, v, cos, sin)
            mlp = torch.nn.functional.gelu(lin1[:, 3 * h:], approximate="tanh")
            x = x + g * blk["linear2"](torch.cat([attn, mlp], dim=-1))
        img = x[n_txt:]
        sh, sc = self.final_mod(svec).chunk(2, dim=-1)
        out = self._ln_mod_lin(self.final, img, sh, sc)
        return out.view(hh, ww, c, 2, 2).permute(2, 0, 3, 1, 4).reshape(1, c, hh * 2, ww * 2)


def dit_step_leg(device, flush, stream, steps):
    """Config 2: one denoising step (the DiT forward) at 1024^2, batch 1, CUDA graph."""
    model = FluxDiT(device)
    gen = torch.Generator(device=device).manual_seed(2)
    latent = torch.randn(1, 16, 128, 128, generator=gen, device=device).to(torch.bfloat16)
    txt = torch.randn(1, 512, 4096, generator=gen, device=device).to(torch.bfloat16)
    y = torch.randn(1, 768, generator=gen, device=device).to(torch.bfloat16)
    t = torch.full((1,), 0.5, device=device)
    guidance = torch.full((1,), 3.5, device=device)
    fwd = lambda: model.forward(latent, txt, y, t, guidance)
    for _ in range(3):
        out = fwd()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all(), "DiT step produced non-finite values"
    replay, graph = graphed(fwd, flush)
    ms = timed_steps(replay, steps, flush, stream, 1, device)
    del graph
    # the same step with torch normalising before every int4 projection (no fused producer)
    model.fused_ln = False
    for _ in range(2):
        fwd()
    replay, graph = graphed(fwd, flush)
    ms_unfused = timed_steps(replay, steps, flush, stream, 1, device)
    del graph
    model.fused_ln = True
    return {"ms": ms, "unfused_ln_ms": ms_unfused, "int4_linears": model.int4_layers, "tokens": 4096 + 512,
            "fused_ln": "LayerNorm + modulation before QKV / MLP-up / linear1 inside the int4 quantizer "
                        "(ck_convrot_w4a4_linear_lnmod); unfused_ln_ms: torch normalises first",
            "inputs": "latent [1,16,128,128], text [1,512,4096] ~ N(0,1), pooled [1,768] ~ N(0,1), t=0.5, "
                      "guidance=3.5 (seeded)",
            "launch": "CUDA graph replay, L2 flushed before each step"}


# ---------------------------------------------------------------- config 4's layer, N-column split

def nsplit_leg(device, rank, world, flush, stream, steps):
    """Config 4's 12288->3072 layer (M = 18432, rank-64 LoRA) split by output columns:
    each rank owns N/world weight rows, computes its columns for every token and the
    all-gather assembles [M, N] on every rank. world = 1: the unsplit layer."""
    import _int4
    from _int4.nsplit import convrot_w4a4_linear_lora_nsplit, shard_adapters, shard_rows
    layers, xs = build_layers(device, seed=4321, cfg_id=4)
    down = next(l for l in layers if l["k"] == 12288)
    x = xs[down["key"]]
    ops = layer_ops(down["m"], down["k"], down["n"], down["r"])
    one_gpu = None
    if rank == 0:
        fn1, g1 = graphed(lambda: run_layer(down, x), flush)
        one_gpu = timed_steps(fn1, steps, flush, stream, 1, device)
        del g1
    if world == 1:
        return {"value": ops / (one_gpu * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": one_gpu,
                "layer": "M=18432 12288->3072 +LoRA r=64, unsplit"}
    from _int4.nsplit import PeerColumnSplit, convrot_w4a4_linear_peer_split, peer_split_supported
    q, w, b = shard_rows(down["qw"], down["ws"], down["bias"], rank, world)
    adapters = shard_adapters(down["adapters"], rank, world)
    gather = lambda: convrot_w4a4_linear_lora_nsplit(x, q, w, b, adapters, GROUP)
    res = {}
    from _int4.nsplit import PeerSplitUnavailable
    split = None
    if peer_split_supported(x, q.shape[0], GROUP):
        try:
            split = PeerColumnSplit(device=device)
        except PeerSplitUnavailable:     # every rank sees the same outcome
            split = None
    legs = [("nccl_all_gather", gather)]
    if split is not None:
        legs.insert(0, ("peer_stores", lambda: convrot_w4a4_linear_peer_split(x, q, w, b, adapters, split, GROUP)))
    for name, step in legs:
        for _ in range(3):
            out = step()
        torch.cuda.synchronize()
        res[name] = timed_steps(step, steps, flush, stream, world, device)
        del out
    if split is not None:
        split.close()
    name = "peer_stores" if split is not None else "nccl_all_gather"
    ms = res[name]
    return {"value": ops / (ms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": ms, "one_gpu_ms": one_gpu,
            "speedup_vs_one_gpu": one_gpu / ms if one_gpu else None,
            "exchange": ("each rank's GEMM writes its column block into its own [M, N] buffer in row chunks; "
                         "copy engines carry each chunk to every peer over NVLink (CUDA IPC peer mappings) "
                         "while the next chunk computes; bounded flag barrier" if split is not None
                         else "NCCL all-gather, then a permute copy into [M, N]"),
            "nccl_all_gather_ms": res["nccl_all_gather"],
            "layer": f"M=18432 12288->3072 +LoRA r=64, N split x{world}"}


# ---------------------------------------------------------------- the GPU arm

def run_ours(args, rank, world, local_rank):
    import _int4
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    assert _int4.is_available(), "libconvrot_b200.so must load on an sm_100 device"
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def flush():
        flush_buf.fill_(1.0)

    cfg_id = args.config
    split = world > 1 and cfg_id != 2
    layers, xs = _build_split(device, cfg_id, rank, world, split)
    ops_total = sum(layer_ops(m, k, n, r) for _, m, k, n, r in WORKLOADS[cfg_id][1])
    step_fn = lambda inputs=None: device_step(layers, xs if inputs is None else inputs)
    for _ in range(args.warmup):
        flush()
        step_fn()
    torch.cuda.synchronize()
    graph = None
    timed_fn = step_fn
    if args.graph:
        # One step (the kernels of every layer) as a CUDA graph: per-launch host
        # work (argument checks, tensor-map encoding) leaves the timed region.
        timed_fn, graph = graphed(step_fn, flush)

    # ---------------- timed region: K steps, barrier + sync on both sides
    sampler = ClockSampler(local_rank)
    sampler.start()
    t_region = time.time()
    ms_per_step = timed_steps(timed_fn, args.steps, flush, stream, world, device)
    sampler.mark(t_region, time.time())
    clocks = sampler.stop()
    value = ops_total / (ms_per_step * 1e-3) / 1e12
    del graph

    # ---------------- each layer of the step on its own (graph, L2 flushed, max over ranks):
    # which layer limits the step at this N
    layers_ms = {}
    if args.extras and args.graph:
        for l in layers:
            fn, g = graphed(lambda l=l: run_layer(l, xs[l["key"]]), flush)
            layers_ms[f"{l['name']} M={l['m']} {l['k']}->{l['n']}"] = timed_steps(fn, min(args.steps, 20), flush,
                                                                                 stream, world, device)
            del g

    # ---------------- end to end: host buffers in, host buffers out, through the public API
    e2e = e2e_leg(layers, xs, device, stream, world, args.steps)
    e2e_value = ops_total / (e2e["ms_per_step"] * 1e-3) / 1e12

    extras = {}
    if world == 1 and cfg_id == 1 and args.extras:
        extras.update(roofline_probes(layers, xs, device, flush, stream))
        # the same step with the opt-in unpacked-weight cache (int8 form, 2x weight bytes)
        from _int4 import weight_cache
        weight_cache.enable(True)
        try:
            fn, g = graphed(lambda: device_step(layers, xs), flush)
            cms = timed_steps(fn, args.steps, flush, stream, 1, device)
            del g
        finally:
            weight_cache.enable(False)
        extras["unpacked_cache"] = {"value": ops_total / (cms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": cms,
                                    "what": "same step with the opt-in unpacked-weight cache (int8 pair GEMM on "
                                            "sign-extended codes of both operands; twice the weight bytes)"}
    # ---------------- weak replicas: every rank runs all tokens
    if world > 1 and cfg_id != 2 and args.extras:
        full_layers, full_xs = build_layers(device, seed=1234, cfg_id=cfg_id)
        fn, g = graphed(lambda: device_step(full_layers, full_xs), flush)
        rms = timed_steps(fn, args.steps, flush, stream, world, device)
        extras["replicas"] = {"value": world * ops_total / (rms * 1e-3) / 1e12, "unit": UNIT, "ms_per_step": rms,
                              "scaling": "weak", "what": f"every rank runs all tokens of the step (x{world} work)"}
        del g, full_layers, full_xs
    # ---------------- config 4's 12288->3072 layer split by columns
    if cfg_id == 1 and args.extras:
        extras["nsplit"] = nsplit_leg(device, rank, world, flush, stream, min(args.steps, 50))
    # ---------------- config 2: a full DiT denoising step (one GPU)
    if world == 1 and cfg_id == 1 and args.extras:
        dit = dit_step_leg(device, flush, stream, min(args.steps, 10))
        lin_layers, lin_xs = build_layers(device, seed=7, cfg_id=2)
        fn, g = graphed(lambda: device_step(lin_layers, lin_xs), flush)
        lin_ms = timed_steps(fn, min(args.steps, 10), flush, stream, 1, device)
        del g, lin_layers, lin_xs
        dit.update({"linears_ms": lin_ms, "linears_share": lin_ms / dit["ms"],
                    "linears_tops": sum(layer_ops(m, k, n, r) for _, m, k, n, r in WORKLOADS[2][1])
                    / (lin_ms * 1e-3) / 1e12})
        extras["dit_step_ms"] = dit["ms"]
        extras["dit_step"] = dit


    if rank == 0:
        cpu = None
        if world == 1 and cfg_id == 1 and args.cpu_seconds > 0:
            cpu = cpu_sample(args.cpu_seconds)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if split else "weak",
            "vs_baseline": None, "dtype": "int4",
            "data": "synthetic (seeded N(0,1) activations with 1% x20 outlier channels, N(0,0.02) weights)",
            "config": workload_config(cfg_id, world if split else 1,
                                      {"launch": "CUDA graph replay" if args.graph else "eager launches"}),
            "gpu_launches": 2 * len(layers) * args.steps,
            **({"layers_ms": layers_ms} if layers_ms else {}),
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, **e2e},
            **extras,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def _build_split(device, cfg_id, rank, world, split):
    """Layers (replicated weights) and this rank's rows of every activation."""
    if not split:
        return build_layers(device, seed=1234, cfg_id=cfg_id)
    layers, xs = build_layers(device, seed=1234, cfg_id=cfg_id)
    shard = {}
    for key, x in xs.items():
        lo, hi = shard_range(x.shape[0], rank, world)
        shard[key] = x[lo:hi].contiguous()
    for l in layers:
        l["m"] = shard[l["key"]].shape[0]
    return layers, shard


def e2e_leg(layers, xs, device, stream, world, steps):
    """The step end to end through the public API: this rank's inputs from pinned host
    buffers, outputs back to pinned host buffers, on three event-ordered streams."""
    host_in = {k: v.cpu().pin_memory() for k, v in xs.items()}
    out_shapes = [(xs[l["key"]].shape[0], l["n"]) for l in layers]
    # one pinned buffer per output shape; every layer's output still crosses PCIe each step
    host_buf = {sh: torch.empty(sh, dtype=torch.bfloat16).pin_memory() for sh in set(out_shapes)}
    host_out = [host_buf[sh] for sh in out_shapes]
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = sum(v.numel() * v.element_size() for v in host_out)
    h2d_stream = torch.cuda.Stream(device)
    d2h_stream = torch.cuda.Stream(device)
    first_use = []
    for l in layers:
        if l["key"] not in first_use:
            first_use.append(l["key"])

    # Uploads, the layers and the downloads run on three streams, ordered by events:
    # a layer starts when its input has landed, its output leaves while the next
    # layers compute, and host<->device copies use both PCIe directions at once.
    def e2e_step():
        dev_in, ready = {}, {}
        with torch.cuda.stream(h2d_stream):
            for key in first_use:
                dev_in[key] = host_in[key].to(device, non_blocking=True)
                ready[key] = torch.cuda.Event()
                ready[key].record(h2d_stream)
        for l, h in zip(layers, host_out):
            stream.wait_event(ready[l["key"]])
            x = dev_in[l["key"]]
            x.record_stream(stream)
            o = run_layer(l, x)
            done = torch.cuda.Event()
            done.record(stream)
            d2h_stream.wait_event(done)
            with torch.cuda.stream(d2h_stream):
                o.record_stream(d2h_stream)
                h.copy_(o, non_blocking=True)
        stream.wait_stream(d2h_stream)          # the step ends when its results are on the host

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    n = max(3, min(steps, 10))
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / n, world, device)
    return {"ms_per_step": ms, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "bytes": "whole job (all ranks)",
            "overlap": "uploads, layers and downloads on three streams (event-ordered)"}


def run_case(args):
    """A few launches of one kernel on its own, for ncu captures (no timing, no flush)."""
    import _int4
    from _int4 import cuda_loader as ck
    device = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(0)
    if args.case == "small_m":
        m, k, n = 1, 3072, 18432
    elif args.case == "lora_down":
        m, k, n = M_TOKENS, 12288, 3072          # config 4's MLP-down input, rank 64
    else:
        m, k, n = M_TOKENS, 3072, 12288
    if args.m:
        m = args.m
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.float16).to(device)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, GROUP)
    bias = torch.zeros(n, device=device)
    x = synth_activation(m, k, gen, device)
    wpacked = qw
    if args.case.endswith("_unpacked") or args.case.endswith("_a8"):   # the captured kernel is the first launch
        xq, xsc = ck.convrot_quant_int4_unpacked(x, GROUP)
        if args.case.endswith("_unpacked"):
            qw = ck.int4_unpack(qw)
    else:
        xq, xsc = ck.convrot_quant_int4(x, GROUP)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    down = (torch.randn(64, k, generator=gen) * 0.01).to(torch.float16).to(device)
    mod_scale = (torch.randn(k, generator=gen) * 0.2).to(torch.bfloat16).to(device)
    mod_shift = (torch.randn(k, generator=gen) * 0.2).to(torch.bfloat16).to(device)
    for _ in range(args.iters):
        if args.case == "lora_down":
            ck.lora_down(x, down)
        elif args.case == "lnmod_quant":
            ck.convrot_quant_int4_lnmod(x, mod_scale, mod_shift, 1e-6, GROUP, True)
        elif args.case == "quant":
            ck.convrot_quant_int4(x, GROUP)
        elif args.case == "quant_unpacked":
            ck.convrot_quant_int4_unpacked(x, GROUP)
        elif args.case == "mlp_up_unpacked":
            ck.int8_convrot_gemm(xq, qw, xsc, ws, bias, torch.bfloat16)
        elif args.case == "mlp_up_a8":
            ck.int4_convrot_gemm_a8(xq, wpacked, xsc, ws, bias, torch.bfloat16)
        else:
            ck.int4_convrot_gemm(xq, qw, xsc, ws, bias, torch.bfloat16)
        flush_buf.fill_(1.0)          # evicts the output from L2: the launch's writes reach DRAM
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "m": m, "k": k, "n": n, "iters": args.iters}))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU-baseline time budget")
    ap.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=1,
                    help="BASELINE config whose linear set is one step (default 1, the metric's config)")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="only the main step (no probes, replicas, N-split or DiT legs)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every kernel from the host each step instead of replaying a CUDA graph")
    ap.add_argument("--case", choices=["mlp_up", "small_m", "quant", "mlp_up_unpacked", "quant_unpacked", "mlp_up_a8",
                                       "lora_down", "lnmod_quant"],
                    default=None,
                    help="run one kernel --iters times (profiling helper) instead of the benchmark")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--m", type=int, default=0, help="token rows of the --case kernel (default: the case's own)")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference" and args.config != 1:
        ap.error("the reference arm times config 1 (the metric's config) only")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)          # rank 0 only; no process group needed
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
