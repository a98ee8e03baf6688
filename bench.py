"""Benchmark of the B200 ConvRot W4A4 linear path.

One step = the Flux-class double-block linear set at M = 4608 tokens:
QKV 3072->9216, attention-out 3072->3072, MLP-up 3072->12288 and MLP-down
12288->3072, each a full W4A4 forward (fused rotate+quantize kernel, then the
tcgen05 int4 GEMM with the dequant + bias epilogue). Metric: W4A4 linear TOPS
(2*M*N*K ops per layer; integer MACs count as two ops).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one process per GPU: token-parallel replicas (each
rank runs its own 4608-token step with replicated weights, no collective on
the data path), weak scaling; the step time is the max over ranks.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/convrot_oracle.py, the port of _int4/eager.py + the HIP epilogue) on
the host cores, rank 0 only.

Timing: inputs are resident in HBM; L2 is flushed (a 256 MiB write) before
every timed step; each step is bracketed by CUDA events on the launching
stream and the K durations are summed.
"""
from __future__ import annotations

import argparse
import json
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

def flux_dit_layers():
    """Every int4 Linear of one forward of a Flux-architecture DiT (config 2): 19 double
    blocks (image stream at 4096 tokens, text stream at 512) and 38 single blocks at
    4608 tokens, hidden 3072, MLP x4; the modulation Linears run at M = 1. The
    embedders and the final layer stay bf16 in the reference loader (EXCLUDED list)."""
    layers = []
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


def workload_config(cfg_id=1, extra=None):
    name, layers = WORKLOADS[cfg_id]
    if cfg_id == 2:
        shapes = sorted({(m, k, n) for _, m, k, n, _ in layers}, reverse=True)
        desc = {"linears": len(layers), "blocks": "19 double (img M=4096, txt M=512) + 38 single (M=4608)",
                "shapes": [f"M={m} {k}->{n}" for m, k, n in shapes],
                "weights": "random packed int4 codes and scales (the kernels' work does not depend on the values)"}
    else:
        desc = {"layers": {lname: f"M={m} {k}->{n}" + (f" +LoRA r={r}" if r else "") for lname, m, k, n, r in layers}}
    cfg = {"workload": name, **desc,
           "convrot_groupsize": GROUP, "l2": "flushed before every timed step (256 MiB write)"}
    if cfg_id == 1:
        cfg.update({"tokens_per_gpu": M_TOKENS, "hidden": HIDDEN})
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
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if not os.path.exists(path):
        return None
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

class CpuWorkload:
    """The oracle port of the reference path (all four layers) on `rows` tokens."""

    def __init__(self, rows: int, seed: int = 0):
        from oracle import convrot_oracle as orc
        self.orc = orc
        self.rows = rows
        rng = np.random.default_rng(seed)
        self.layers = []
        for _, k, n in LAYERS:
            w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02).astype(np.float16)
            wp, ws = orc.quantize_weight(w, GROUP, "f16")
            bias = (rng.standard_normal(n, dtype=np.float32) * 0.01).astype(np.float16).astype(np.float32)
            x = rng.standard_normal((rows, k), dtype=np.float32)
            x[:, rng.permutation(k)[: k // 100]] *= 20
            # weights stay decoded across steps, like resident device weights
            self.layers.append((orc.f32_to_bf16_bits(x), orc.decode_weight(wp), ws, bias))

    def step(self) -> float:
        t0 = time.perf_counter()
        for x, wcodes, ws, bias in self.layers:
            self.orc.convrot_w4a4_linear_decoded(x, wcodes, ws, bias, GROUP)
        return time.perf_counter() - t0


def cpu_sample(rows: int, budget_s: float, seed: int = 0):
    """Median step time of the oracle port over about `budget_s` seconds: (TOPS, s, steps)."""
    wl = CpuWorkload(rows, seed)
    wl.step()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 2 or time.perf_counter() < t_end:
        times.append(wl.step())
    t = statistics.median(times)
    return step_ops(rows) / t / 1e12, t, len(times)


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def run_reference(args, rank):
    if rank != 0:
        return
    rows = args.cpu_rows
    wl = CpuWorkload(rows)
    for _ in range(args.warmup):
        wl.step()
    times = [wl.step() for _ in range(args.steps)]
    t = statistics.median(times)
    value = step_ops(rows) / t / 1e12
    sample = f"{rows} of {M_TOKENS} tokens per step through all four layers (oracle port, numpy + BLAS)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3 * M_TOKENS / rows,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4",
        "data": "synthetic (seeded; config-1 shapes and value distributions)",
        "config": workload_config(1, {"cpu_rows_per_step": rows}),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm

def build_layers(device, seed, cfg_id=1):
    """Quantized layers and device-resident inputs of one step of config `cfg_id`."""
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
    return layers, xs


def device_step(layers, xs):
    """One step through the public API on device-resident inputs."""
    import _int4
    outs = []
    for l in layers:
        x = xs[(l["m"], l["k"])]
        if l["r"]:
            outs.append(_int4.convrot_w4a4_linear_lora(x, l["qw"], l["ws"], l["bias"], l["adapters"], GROUP))
        else:
            outs.append(_int4.convrot_w4a4_linear(x, l["qw"], l["ws"], l["bias"], GROUP))
    return outs


def nsplit_step(layers, xs, rank, world):
    """Config 4's 12288->3072 layer (with its LoRA side path unfused: the split
    applies to the int4 product) column-split over the ranks: each rank owns N/P
    weight rows, all ranks see the same M=18432 tokens, an NCCL all-gather
    assembles [M, N]. Returns (step_fn, ops of the whole layer, layer list)."""
    from _int4.nsplit import convrot_w4a4_linear_nsplit, shard_rows
    down = next(l for l in layers if l["k"] == 12288)
    q, w, b = shard_rows(down["qw"], down["ws"], down["bias"], rank, world)
    ops = 2 * down["m"] * down["n"] * down["k"]
    lay = [dict(down, n_out=down["n"])]

    def step(inputs=None):
        src = xs if inputs is None else inputs
        return [convrot_w4a4_linear_nsplit(src[(down["m"], down["k"])], q, w, b, GROUP)]
    return step, ops, lay


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


def run_ours(args, rank, world, local_rank):
    import _int4
    from _int4 import cuda_loader as ck
    from _int4 import weight_cache
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    assert _int4.is_available(), "libconvrot_b200.so must load on an sm_100 device"
    stream = torch.cuda.current_stream(device)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def flush():
        flush_buf.fill_(1.0)

    cfg_id = args.config
    layers, xs = build_layers(device, seed=1234 + rank, cfg_id=cfg_id)
    ops_per_step = sum(layer_ops(l["m"], l["k"], l["n"], l["r"]) for l in layers)
    if args.nsplit:
        step_fn, ops_per_step, layers = nsplit_step(layers, xs, rank, world)
    else:
        step_fn = lambda inputs=None: device_step(layers, xs if inputs is None else inputs)
    for _ in range(args.warmup):
        flush()
        step_fn()
    torch.cuda.synchronize()
    if args.graph and not args.nsplit:
        # Capture one step (the kernels of every layer) in a CUDA graph and
        # replay it: per-launch host work (argument checks, tensor-map
        # encoding) leaves the timed region, the device work is unchanged.
        eager_fn = step_fn
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_outs = eager_fn()
        torch.cuda.synchronize()

        def step_fn(inputs=None):
            if inputs is not None:
                return eager_fn(inputs)
            graph.replay()
            return graph_outs
        for _ in range(2):
            flush()
            step_fn()
        torch.cuda.synchronize()

    # ---------------- timed region: K steps, barrier + sync on both sides
    sampler = ClockSampler(local_rank)
    sampler.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    t_region = time.time()
    events = []
    for _ in range(args.steps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step_fn()
        b.record(stream)
        events.append((a, b))
    torch.cuda.synchronize()
    sampler.mark(t_region, time.time())
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    elapsed_ms = sum(a.elapsed_time(b) for a, b in events)
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    # weak scaling: every rank ran a full step; N-split: the ranks shared one step
    value = (1 if args.nsplit else world) * ops_per_step / (ms_per_step * 1e-3) / 1e12

    # ---------------- per-kernel roofline (dominant GEMM = MLP up), rank 0, config 1
    extras = {}
    if rank == 0 and cfg_id == 1 and not args.nsplit:
        peaks, peak_src = load_peaks()
        up = next(l for l in layers if l["name"] == "mlp_up")
        m, k, n = up["m"], up["k"], up["n"]
        iters = 10
        # time the kernels the public linear runs for this layer: with the
        # unpacked-weight cache on (default) and M > 128 that is the int8 pair GEMM
        # on sign-extended codes, else the int4 pair GEMM on packed codes
        unpacked = _int4._use_unpacked(xs[(m, k)], up["qw"], GROUP)
        if unpacked:
            quant = ck.convrot_quant_int4_unpacked
            wq = weight_cache.unpacked(up["qw"])
            xq, xsc = quant(xs[(m, k)], GROUP)
            gemm = lambda: ck.int8_convrot_gemm(xq, wq, xsc, up["ws"], up["bias32"], torch.bfloat16)
            gemm_name, code_bytes = "int8 pair GEMM on unpacked int4 codes", 1
            traffic_key = "int8_pair_unpacked_bytes_per_launch"
        else:
            quant = ck.convrot_quant_int4
            xq, xsc = quant(xs[(m, k)], GROUP)
            gemm = lambda: ck.int4_convrot_gemm(xq, up["qw"], xsc, up["ws"], up["bias32"], torch.bfloat16)
            gemm_name, code_bytes = "int4_gemm_pair_kernel", 0.5
            traffic_key = "int4_gemm_kernel_bytes_per_launch"
        gemm_ms = time_kernel(gemm, iters, flush, stream)
        # 8 distinct activations (8 x 28 MB, well beyond L2), launched back to back
        xq_in = [synth_activation(m, k, torch.Generator().manual_seed(100 + i), device) for i in range(8)]
        quant_ms = time_kernel_batch([lambda x=x: quant(x, GROUP) for x in xq_in], iters, flush, stream)
        del xq_in
        gemm_ops = 2 * m * n * k
        int8_peak = 2.0 * peaks["bf16_tflops"]           # dense int8 rate = 2x bf16 on B200
        achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
        traffic = load_traffic()
        extras["roofline"] = {
            "kernel": f"int4_gemm_pair_kernel, {gemm_name} (MLP up 3072->12288, M=4608)",
            "bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
            "frac": achieved / int8_peak,
            "peak_source": f"2 x {peak_src} bf16 burst ({peaks['bf16_tflops']} TFLOP/s): B200 dense int8 rate",
            "ms_per_launch": gemm_ms,
            "traffic": traffic.get(traffic_key) if traffic else None,
            "algorithmic_bytes": int(code_bytes * (m * k + n * k)) + 4 * m + 4 * n + 4 * n + 2 * m * n,
        }
        qbytes = 2 * m * k + int(code_bytes * m * k) + 4 * m
        extras["quant_kernel"] = {
            "kernel": f"convrot_quant_bf16_kernel{' (unpacked codes)' if unpacked else ''} (K=3072, M=4608)",
            "bound": "hbm",
            "achieved": qbytes / (quant_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": qbytes / (quant_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "ms_per_launch": quant_ms,
            "timing": "8 launches back to back over distinct 28 MB inputs in one CUDA graph, per launch",
            "traffic": traffic.get("convrot_quant_unpacked_bytes_per_launch" if unpacked else
                                   "convrot_quant_bf16_kernel_bytes_per_launch") if traffic else None,
        }
        # small-M (weight-bound) layer: Flux modulation 3072 -> 18432 at M = 1
        wsm = (torch.randn(18432, 3072, device=device) * 0.02).to(torch.float16)
        qsm, wssm = _int4.quantize_convrot_w4a4_weight(wsm, GROUP)
        del wsm
        # 16 distinct weight copies (16 x 28 MB, beyond L2), launched back to back
        qsms = [qsm] + [qsm.roll(i, 0).contiguous() for i in range(1, 16)]
        x1 = synth_activation(1, 3072, torch.Generator().manual_seed(5), device)
        x1q, x1s = ck.convrot_quant_int4(x1, GROUP)
        sm_ms = time_kernel_batch([lambda q=q: ck.int4_convrot_gemm(x1q, q, x1s, wssm, None, torch.bfloat16)
                                   for q in qsms], iters, flush, stream)
        del qsms
        sm_bytes = 3072 // 2 + 18432 * 3072 // 2 + 4 + 4 * 18432 + 2 * 18432
        extras["small_m"] = {
            "kernel": "int4_gemv_kernel (modulation 3072->18432, M=1)", "bound": "hbm",
            "achieved": sm_bytes / (sm_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": sm_bytes / (sm_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "ms_per_launch": sm_ms,
            "timing": "16 launches back to back over distinct 28 MB weight copies in one CUDA graph, per launch",
            "traffic": traffic.get("int4_gemv_kernel_bytes_per_launch") if traffic else None,
        }

    # ---------------- end to end: host buffers in, host buffers out, through the public API
    host_in = {k: v.cpu().pin_memory() for k, v in xs.items()}
    # one pinned buffer per output shape (config 2 has 304 outputs of 9 shapes); every
    # layer's output still crosses PCIe each step
    out_shapes = [(l["m"], l["n_out"] if "n_out" in l else l["n"]) for l in layers]
    host_buf = {sh: torch.empty(sh, dtype=torch.bfloat16).pin_memory() for sh in set(out_shapes)}
    host_out = [host_buf[sh] for sh in out_shapes]
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = sum(v.numel() * v.element_size() for v in host_out)

    # Uploads, the layers and the downloads run on three streams, ordered by events:
    # a layer starts when its input has landed, its output leaves while the next
    # layers compute, and host<->device copies use both PCIe directions at once.
    h2d_stream = torch.cuda.Stream(device)
    d2h_stream = torch.cuda.Stream(device)
    first_use = []
    for l in layers:
        if (l["m"], l["k"]) not in first_use:
            first_use.append((l["m"], l["k"]))

    def e2e_step_serial():
        dev_in = {k: v.to(device, non_blocking=True) for k, v in host_in.items()}
        outs = step_fn(dev_in)
        for o, h in zip(outs, host_out):
            h.copy_(o, non_blocking=True)

    def e2e_step_pipelined():
        import _int4
        dev_in, ready = {}, {}
        with torch.cuda.stream(h2d_stream):
            for key in first_use:
                dev_in[key] = host_in[key].to(device, non_blocking=True)
                ready[key] = torch.cuda.Event()
                ready[key].record(h2d_stream)
        for l, h in zip(layers, host_out):
            key = (l["m"], l["k"])
            stream.wait_event(ready[key])
            x = dev_in[key]
            x.record_stream(stream)
            if l["r"]:
                o = _int4.convrot_w4a4_linear_lora(x, l["qw"], l["ws"], l["bias"], l["adapters"], GROUP)
            else:
                o = _int4.convrot_w4a4_linear(x, l["qw"], l["ws"], l["bias"], GROUP)
            done = torch.cuda.Event()
            done.record(stream)
            d2h_stream.wait_event(done)
            with torch.cuda.stream(d2h_stream):
                o.record_stream(d2h_stream)
                h.copy_(o, non_blocking=True)
        stream.wait_stream(d2h_stream)          # the step ends when its results are on the host

    e2e_step = e2e_step_serial if args.nsplit else e2e_step_pipelined

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = (1 if args.nsplit else world) * ops_per_step / (e2e_ms * 1e-3) / 1e12

    if rank == 0:
        cpu_tops = None
        if world == 1 and cfg_id == 1 and args.cpu_seconds > 0:
            cpu_tops, _, _ = cpu_sample(args.cpu_rows, args.cpu_seconds)
        par = (f"N-column split x{world} of the 12288->3072 layer, NCCL all-gather" if args.nsplit
               else f"token-parallel replicas x{world}")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if args.nsplit else "weak",
            "vs_baseline": None, "dtype": "int4",
            "data": "synthetic (seeded N(0,1) activations with 1% x20 outlier channels, N(0,0.02) weights)",
            "config": workload_config(cfg_id, {"parallelism": par,
                                               "launch": "CUDA graph replay" if args.graph and not args.nsplit
                                               else "eager launches"}),
            "gpu_launches": 2 * len(layers) * args.steps,
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "overlap": "serial" if args.nsplit else
                               "uploads, layers and downloads on three streams (event-ordered)"},
            **extras,
        }
        if cpu_tops is not None:
            line["cpu_baseline"] = {"value": cpu_tops, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                                    "sample": f"{args.cpu_rows} tokens through all four layers, "
                                              f"median over ~{args.cpu_seconds:.0f} s (oracle port)"}
        print(json.dumps(line), flush=True)


def run_case(args):
    """A few launches of one kernel on its own, for ncu captures (no timing, no flush)."""
    import _int4
    from _int4 import cuda_loader as ck
    device = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(0)
    if args.case == "small_m":
        m, k, n = 1, 3072, 18432
    else:
        m, k, n = M_TOKENS, 3072, 12288
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.float16).to(device)
    qw, ws = _int4.quantize_convrot_w4a4_weight(w, GROUP)
    bias = torch.zeros(n, device=device)
    x = synth_activation(m, k, gen, device)
    if args.case.endswith("_unpacked"):                # the captured kernel is the first launch
        xq, xsc = ck.convrot_quant_int4_unpacked(x, GROUP)
        qw = ck.int4_unpack(qw)
    else:
        xq, xsc = ck.convrot_quant_int4(x, GROUP)
    for _ in range(args.iters):
        if args.case == "quant":
            ck.convrot_quant_int4(x, GROUP)
        elif args.case == "quant_unpacked":
            ck.convrot_quant_int4_unpacked(x, GROUP)
        elif args.case == "mlp_up_unpacked":
            ck.int8_convrot_gemm(xq, qw, xsc, ws, bias, torch.bfloat16)
        else:
            ck.int4_convrot_gemm(xq, qw, xsc, ws, bias, torch.bfloat16)
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "m": m, "k": k, "n": n, "iters": args.iters}))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-rows", type=int, default=256, help="tokens per CPU-baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline time budget")
    ap.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=1,
                    help="BASELINE config whose linear set is one step (default 1, the metric's config)")
    ap.add_argument("--nsplit", action="store_true",
                    help="config 4's 12288->3072 layer split by output columns over the ranks (strong scaling)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every kernel from the host each step instead of replaying a CUDA graph")
    ap.add_argument("--case", choices=["mlp_up", "small_m", "quant", "mlp_up_unpacked", "quant_unpacked"], default=None,
                    help="run one kernel --iters times (profiling helper) instead of the benchmark")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.nsplit:
        args.config = 4

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)          # rank 0 only; no process group needed
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
