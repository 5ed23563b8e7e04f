"""Benchmark of the W4A4 quantized-linear hot path on B200.

Headline workload (BASELINE config 1 at batch 32, Qwen3-8B shapes): one *step*
is the chained forward of the four W4A4 projections of all 36 decoder layers
at M=32 tokens -- QKV (K=4096 -> N=6144), O (4096 -> 4096), gate/up
(4096 -> 24576), down (12288 -> 4096) -- each one activation-prep launch
(block128 RHT + per-group INT4 quantisation, codes in [-8, 7]) and one grouped
INT4 GEMM launch, with distinct random weights per layer (3.58 GB, larger than
L2, so no flush is needed).  The projections are chained as in a Qwen3 decoder
layer with attention left out (it is not on the quantized-linear path): QKV's
prep applies the residual add + input RMSNorm, O reads the first M*K elements
of the QKV output viewed as [M, K] (no copy kernel), gate/up's prep applies
the residual add + post-attention RMSNorm, and down's prep reads the whole
gate/up output and applies the MLP's SiluAndMul -- each producer fused into
the prep kernel, as in the model.  The step is captured in a CUDA graph and
replayed, as the reference's model runner does for decode.

``--gpus N`` (torchrun, one rank per GPU):
  * ``--mode tp`` (default for N > 1): tensor parallelism over the N ranks, the
    reference's partition (nanovllm/layers/linear.py:54-155): QKV and gate/up
    sharded along N, O and down along group-aligned K with the row-parallel
    sum over NVLink peer memory.  The batch stays 32 tokens (strong scaling);
    ``value`` is the step's algorithmic bytes over the slowest rank's time.
  * ``--mode dp``: N independent replicas, each with its own batch of 32 (weak
    scaling); ``value`` is all ranks' bytes over the slowest rank's time.

Every run (1 GPU, and TP at N > 1) also carries ``model_decode``: BASELINE
config 4, a random-init Qwen3-8B through the engine's public API (32 requests
of 4096 tokens, then 256 batch-32 greedy decode steps, CUDA graphs), with W4A4
and with BF16 cuBLAS linears: decode tokens/s of both and their ratio.

At one GPU the line also carries ``configs``: every configuration BASELINE
names, measured in the same run -- config 1 per projection at M in {1, 8, 32}
(GEMM launches over 36 distinct weight sets, and the prep launch), config 2
prefill TOPS at M in {512, 2048, 4096} against a same-run dense INT8 peak
(torch._int_mm, 8192^3), config 3 W4A16 at M in {1, 16, 128, 2048}, and the
same-box BF16 cuBLAS chain (torch F.linear with the same 36 layers, chaining
and producers) as the comparator the north_star's end-to-end target names.

``--impl reference`` times the reference's own PyTorch CPU path (restated in
oracle/torch_ref.py) on one decoder layer of the same chained workload per
step, with every host core.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-int4_b200"))

import torch  # noqa: E402

from nanovllm.utils import synthetic  # noqa: E402

M_TOKENS = 32
LAYERS = 36
SHAPES = [("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 24576, 4096), ("down", 4096, 12288)]
METRIC = "W4A4 decode linears HBM GB/s (Qwen3-8B shapes, batch 32, 36 layers)"
NORM_EPS = 1e-6

# Published A6000 figures of the reference (benchmarks/README.md:126-133), microseconds.
REF_A6000_US = {
    32: {"qkv": 21.25, "o": 14.97, "gate_up": 79.86, "down": 46.06},
    4096: {"qkv": 861.77, "o": 505.62, "gate_up": 3293.68, "down": 1550.64},
}


def linear_bytes(m: int, n: int, k: int, silu: bool = False, norm: int = 0) -> int:
    """Algorithmic HBM bytes of one prep + GEMM chain: X read (the [M, 2K]
    gate/up output when the prep applies SiluAndMul; with a fused RMSNorm
    (`norm` = 1) also its BF16 weight, and with the residual add (`norm` = 2)
    the residual read and the new residual written), codes (INT8 layout) and
    scales written then read, weights and weight scales read, BF16 output
    written, signs."""
    prep = 2 * m * k * (2 if silu else 1) + k + (m * k + 2 * m * k // 128)
    prep += (2 * k if norm else 0) + (4 * m * k if norm == 2 else 0)
    return prep + gemm_bytes(m, n, k)


def gemm_bytes(m: int, n: int, k: int) -> int:
    """Algorithmic bytes of one GEMM launch: packed weights + weight scales, INT8
    activation codes + scales, BF16 output."""
    return n * k // 2 + 2 * n * k // 128 + m * k + 2 * m * k // 128 + 2 * m * n


def prep_bytes(m: int, k: int) -> int:
    """Algorithmic bytes of one plain prep launch: BF16 X, signs, INT8 codes, scales."""
    return 2 * m * k + k + m * k + 2 * m * k // 128


def w4a16_bytes(m: int, n: int, k: int) -> int:
    """qweight (N*K/2) + FP16 scales + qzeros + BF16 X + BF16 out."""
    return n * k // 2 + 2 * n * k // 128 + 4 * n * k // 1024 + 2 * m * k + 2 * m * n


def layer_bytes(m: int, first: bool, tp: int = 1) -> int:
    """One decoder layer of the chain: QKV (RMSNorm, plus the residual add after
    the first layer), O, gate/up (residual add + RMSNorm), down (SiluAndMul).
    With tensor parallelism every rank reads its weight shard and the
    replicated activations; the bytes counted are the whole job's weights
    plus one rank's activations (the algorithmic minimum of the partition)."""
    norms = {"qkv": 1 if first else 2, "o": 0, "gate_up": 2, "down": 0}
    return sum(linear_bytes(m, n, k, silu=name == "down", norm=norms[name]) for name, n, k in SHAPES)


def step_bytes(m: int, layers: int) -> int:
    return layer_bytes(m, True) + (layers - 1) * layer_bytes(m, False)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


TRAFFIC_PROFILE = os.path.join(ROOT, "profiles", "w4a4_stream_gemm_m32.md")


def profiled_traffic():
    """DRAM bytes (read + write) of one gate/up GEMM launch from the committed
    ncu capture of this kernel, or None when the summary is absent."""
    import re
    if not os.path.exists(TRAFFIC_PROFILE):
        return None
    with open(TRAFFIC_PROFILE) as f:
        m = re.search(r"gate/up traffic per launch \(dram read \+ write\): (\d+) bytes", f.read())
    return int(m.group(1)) if m else None


# ---------------------------------------------------------------- clocks (NVML, read-only)
class ClockSampler(threading.Thread):
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.005):
        super().__init__(daemon=True)
        self.samples, self.reasons, self.period = [], set(), period_s
        self._halt = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = getattr(torch.cuda.get_device_properties(device_index), "uuid", None)
            if uuid is not None:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
            else:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - depends on the box
            self.error = repr(e)

    def run(self):
        if not self.ok:
            return
        while not self._halt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self):
        self._halt.set()
        self.join(timeout=2)
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": getattr(self, "error", "nvml")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------- model of the workload
def build_layers(device, layers, tp_rank, tp_size):
    from nanovllm.layers.linear_w4a4 import (W4A4MergedColumnParallelLinear, W4A4QKVParallelLinear,
                                             W4A4RowParallelLinear)
    gen = torch.Generator(device=device)
    mods = []
    for i in range(layers):
        layer = {}
        for name, n, k in SHAPES:
            if name == "qkv":
                mod = W4A4QKVParallelLinear(k, 128, 32, 8, tp_rank=tp_rank, tp_size=tp_size)
            elif name == "gate_up":
                mod = W4A4MergedColumnParallelLinear(k, [n // 2, n // 2], tp_rank=tp_rank, tp_size=tp_size)
            else:
                mod = W4A4RowParallelLinear(k, n, tp_rank=tp_rank, tp_size=tp_size)
            mod = mod.to(device)
            # every rank draws the same full matrices and keeps its shard
            gen.manual_seed(1000 * i + n + k)
            packed = torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=device, generator=gen)
            scale = (torch.randn(n, k // 128, device=device, generator=gen).abs() * (0.02 / 7)).bfloat16()
            signs = (torch.randint(0, 2, (k,), device=device, generator=gen, dtype=torch.int8) * 2 - 1)
            mod.load_full(packed, scale, signs)
            del packed, scale
            layer[name] = mod
        # input / post-attention RMSNorm weights (around 1, as in trained models)
        gen.manual_seed(1000 * i + 7)
        layer["norm_in"] = (1.0 + 0.1 * torch.randn(4096, device=device, generator=gen)).bfloat16()
        layer["norm_post"] = (1.0 + 0.1 * torch.randn(4096, device=device, generator=gen)).bfloat16()
        mods.append(layer)
    return mods


def head_view(t, k):
    """The first M*K elements of a contiguous [M, N >= K] output as a contiguous
    [M, K] input: keeps the data dependency between projections without a copy
    kernel (a column slice would need one, outside the quantized-linear path)."""
    m = t.shape[0]
    return t.reshape(-1)[: m * k].view(m, k)


def forward(mods, x):
    """Chained decode forward through the linears and their fused producers (a
    Qwen3 decoder layer without attention); x: [32, 4096] BF16 (replicated)."""
    h, res = x, None
    for layer in mods:
        qkv, res = layer["qkv"].forward_add_rmsnorm(h, res, layer["norm_in"], NORM_EPS)
        o = layer["o"](head_view(qkv, layer["o"].in_features))
        gu, res = layer["gate_up"].forward_add_rmsnorm(o, res, layer["norm_post"], NORM_EPS)
        h = layer["down"].forward_silu_mul(gu)  # SiluAndMul fused into down's prep
    return h


# ---------------------------------------------------------------- CPU: the reference's PyTorch path
def cpu_layer_sample(seed=0):
    """One layer of the chained workload on the host, through the reference's
    PyTorch CPU path (oracle/torch_ref.py).  Returns (run, bytes)."""
    sys.path.insert(0, ROOT)
    from oracle import torch_ref
    x = synthetic.activations(M_TOKENS, 4096, seed)
    weights = []
    for name, n, k in SHAPES:
        codes, _, scale = synthetic.w4a4_weights(n, k, seed + n)
        weights.append((codes, scale, synthetic.make_signs(k, seed + k)))
    norm_w = torch.ones(4096, dtype=torch.bfloat16)

    def run():
        h, res = x, x
        for (name, n, k), (codes, scale, signs) in zip(SHAPES, weights):
            if name == "down":
                inp = torch_ref.silu_mul(h)
            elif name in ("qkv", "gate_up"):
                inp, res = torch_ref.add_rmsnorm(h, res, norm_w, NORM_EPS)
            else:
                inp = h.reshape(-1)[: h.shape[0] * k].reshape(h.shape[0], k)
            h = torch_ref.w4a4_linear(inp, signs, codes, scale, clamp_lo=-8)
        return h
    return run, layer_bytes(M_TOKENS, False)


CPU_SAMPLE = ("one decoder layer (4 W4A4 linears, M=32, with their add+RMSNorm / SiluAndMul producers) of the "
              "chained workload: the reference's PyTorch CPU path (rht_reference.fwht per 128-group, "
              "a4_group_quant.quantize_rotated with clamp -8, pack_int4, verify_w4a4_aw_grouped.reference, "
              ".bfloat16()) restated in oracle/torch_ref.py")


def cpu_baseline(target_s=12.0):
    torch.set_num_threads(os.cpu_count() or 1)
    run, nbytes = cpu_layer_sample()
    run()  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        run()
        reps += 1
        if time.perf_counter() - t0 >= target_s:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{reps} x {CPU_SAMPLE}, {dt * 1e3:.0f} ms each"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    run, nbytes = cpu_layer_sample()
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    cb = {"value": value, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
          "sample": f"{CPU_SAMPLE}, per step"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xint4->fp32",
        "data": "synthetic", "config": {"workload": "config1-decode-chain-1layer-cpu", "m_tokens": M_TOKENS,
                                        "layers": 1, "layout": "block128", "clamp_lo": -8},
        "cpu_baseline": cb, "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0}}), flush=True)


# ---------------------------------------------------------------- GPU timing helpers
def time_graph(graph, steps, stream):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / 1e3


def graph_of(fn, warm=2):
    """Capture fn() in a CUDA graph after `warm` eager calls (kernel attributes)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_launches(fn, launches_per_call, stream, reps):
    """Seconds per launch of fn (captured in a graph, replayed `reps` times)."""
    g = graph_of(fn)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    t = time_graph(g, reps, stream) / (reps * launches_per_call)
    del g
    return t


# ---------------------------------------------------------------- extra configurations (1 GPU)
def measure_decode(mods, device, stream, peak_hbm):
    """Config 1 per projection: the GEMM over the 36 layers' distinct weights
    (one graph, 36 launches) and the activation prep, at M in {1, 8, 32}."""
    from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
    out = {}
    for m in (1, 8, 32):
        row = {}
        for name, n, k in SHAPES:
            mod0 = mods[0][name]
            x = synthetic.activations(m, k, seed=11 + m).to(device)
            codes, sa = mod0.quantize_input(x)
            outs = [torch.empty(m, n, dtype=torch.bfloat16, device=device) for _ in mods]

            def gemms():
                for layer, o_ in zip(mods, outs):
                    w4a4_grouped_gemm_i8(codes, layer[name].packed_weight, sa, layer[name].weight_scale, out=o_)
            t_gemm = time_launches(gemms, len(mods), stream, 20)

            def preps():
                for layer in mods:
                    layer[name].quantize_input(x)
            t_prep = time_launches(preps, len(mods), stream, 20)
            gb = gemm_bytes(m, n, k)
            row[name] = {"gemm_us": t_gemm * 1e6, "gemm_gbs": gb / t_gemm / 1e9,
                         "gemm_frac": gb / t_gemm / 1e9 / peak_hbm, "gemm_bytes": gb,
                         "prep_us": t_prep * 1e6, "prep_gbs": prep_bytes(m, k) / t_prep / 1e9}
            if m in REF_A6000_US:
                row[name]["ref_a6000_gemm_us"] = REF_A6000_US[m][name]
        out[f"m{m}"] = row
    return out


def int8_peak(device, stream):
    """Dense INT8 tensor throughput of cuBLASLt on this GPU: torch._int_mm on
    8192^3 (2*N^3 ops), best of 10 launches timed with CUDA events."""
    n = 8192
    try:
        a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device)
        b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=device).t()
        c = torch._int_mm(a, b)
        best = None
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            c = torch._int_mm(a, b)
            e.record(stream)
            e.synchronize()
            t = s.elapsed_time(e) / 1e3
            best = t if best is None else min(best, t)
        del a, b, c
        return {"tops": 2 * n ** 3 / best / 1e12, "how": "torch._int_mm int8 8192^3, best of 10, CUDA events"}
    except Exception as e:  # pragma: no cover - depends on the torch build
        return {"tops": None, "error": repr(e)[:200]}


def measure_prefill(mods, device, stream, int8):
    """Config 2: the tcgen05 GEMM and the prep at M in {512, 2048, 4096}."""
    from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
    peak = int8.get("tops") or 4500.0
    out = {}
    for m in (512, 2048, 4096):
        row = {}
        for name, n, k in SHAPES:
            g = torch.Generator(device=device).manual_seed(m + n + k)
            x = torch.randn(m, k, device=device, generator=g).bfloat16()
            mod0 = mods[0][name]
            codes, sa = mod0.quantize_input(x)
            o_ = torch.empty(m, n, dtype=torch.bfloat16, device=device)
            layers = mods[:3]

            def gemms():
                for layer in layers:
                    w4a4_grouped_gemm_i8(codes, layer[name].packed_weight, sa, layer[name].weight_scale, out=o_)
            t_gemm = time_launches(gemms, len(layers), stream, 5)

            def preps():
                mod0.quantize_input(x)
            t_prep = time_launches(preps, 1, stream, 10)
            ops = 2 * m * n * k
            row[name] = {"gemm_us": t_gemm * 1e6, "tops": ops / t_gemm / 1e12,
                         "frac_int8_peak": ops / t_gemm / 1e12 / peak, "prep_us": t_prep * 1e6,
                         "prep_gbs": prep_bytes(m, k) / t_prep / 1e9}
            if m in REF_A6000_US:
                row[name]["ref_a6000_gemm_us"] = REF_A6000_US[m][name]
            del x, codes, sa, o_
        out[f"m{m}"] = row
    return out


def measure_w4a16(device, stream, peaks):
    """Config 3: W4A16Linear at M in {1, 16, 128, 2048}, plus 32 (the decode
    batch of the end-to-end model).  Small M streams
    distinct weight copies (more than 256 MB in total, larger than L2)."""
    from nanovllm import _native
    from nanovllm.layers.linear_w4a16 import W4A16Linear
    out = {}
    shapes = [("qkv", 6144, 4096), ("gate_up", 24576, 4096), ("down", 4096, 12288)]
    for name, n, k in shapes:
        g = torch.Generator(device=device).manual_seed(n + k)
        wb = n * k // 2
        copies = max(1, -(-256 * 2 ** 20 // wb))
        mods = []
        for _ in range(copies):
            lin = W4A16Linear(k, n).to(device)
            with torch.no_grad():
                lin.qweight.copy_(torch.randint(-2 ** 31, 2 ** 31 - 1, lin.qweight.shape, dtype=torch.int64,
                                                device=device, generator=g).to(torch.int32))
                lin.qzeros.copy_(torch.randint(-2 ** 31, 2 ** 31 - 1, lin.qzeros.shape, dtype=torch.int64,
                                               device=device, generator=g).to(torch.int32))
                lin.scales.copy_((torch.randn(lin.scales.shape, device=device, generator=g).abs() * 0.02).half())
            mods.append(lin)
        row = {}
        for m in (1, 16, 32, 128, 2048):
            x = torch.randn(m, k, device=device, generator=g).bfloat16()
            use = mods if m <= 16 else mods[:2]

            def calls():
                for lin in use:
                    lin(x)
            t = time_launches(calls, len(use), stream, 10 if m <= 128 else 3)
            r = {"us": t * 1e6, "gbs": w4a16_bytes(m, n, k) / t / 1e9, "tflops": 2 * m * n * k / t / 1e12}
            pl = _native.w4a16_plan(m, n, k, torch.cuda.get_device_properties(device).multi_processor_count)
            r["kernel"] = {0: "mma.sync", 1: "decode stream", 2: "tcgen05"}[pl["kernel"]]
            r["k_splits"] = pl["splits"]
            r["frac_hbm"] = r["gbs"] / peaks["hbm_gbs"]
            r["frac_bf16"] = r["tflops"] / peaks["bf16_tflops"]
            r["frac_bf16_sustained"] = r["tflops"] / peaks["bf16_tflops_sustained"]
            row[f"m{m}"] = r
        out[name] = row
        del mods
        torch.cuda.empty_cache()
    return out


def measure_bf16_chain(device, stream, layers, x_dev):
    """The same-box BF16 cuBLAS path: the same 36-layer chain with BF16 weights
    and torch.nn.functional.linear, the residual add + RMSNorm and SiluAndMul in
    FP32 torch ops, captured in one CUDA graph."""
    import torch.nn.functional as F
    gen = torch.Generator(device=device)
    ws = []
    for i in range(layers):
        layer = {}
        for name, n, k in SHAPES:
            gen.manual_seed(5000 + 1000 * i + n + k)
            layer[name] = (torch.randn(n, k, device=device, generator=gen) * 0.02).bfloat16()
        layer["norm_in"] = torch.ones(4096, dtype=torch.bfloat16, device=device)
        layer["norm_post"] = torch.ones(4096, dtype=torch.bfloat16, device=device)
        ws.append(layer)

    def rms(x, res, w):
        xf = x.float() if res is None else x.float() + res.float()
        r = xf.bfloat16()
        h = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + NORM_EPS)).bfloat16() * w
        return h, r

    def fwd():
        h, res = x_dev, None
        for layer in ws:
            a, res = rms(h, res, layer["norm_in"])
            qkv = F.linear(a, layer["qkv"])
            o = F.linear(head_view(qkv, 4096), layer["o"])
            a, res = rms(o, res, layer["norm_post"])
            gu = F.linear(a, layer["gate_up"])
            g_, u_ = gu.float().chunk(2, -1)
            h = F.linear((F.silu(g_) * u_).bfloat16(), layer["down"])
        return h

    with torch.no_grad():
        g = graph_of(fwd)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        steps = 20
        dt = time_graph(g, steps, stream) / steps
    wbytes = layers * sum(2 * n * k for _, n, k in SHAPES)
    del g, ws
    torch.cuda.empty_cache()
    return {"ms_per_step": dt * 1e3, "tok_s_linears": M_TOKENS / dt, "weight_bytes": wbytes,
            "weight_gbs": wbytes / dt / 1e9,
            "api": "torch.nn.functional.linear (cuBLAS) BF16, same chain and producers, CUDA graph"}


# ---------------------------------------------------------------- config 4: the end-to-end model
E2E_REQUESTS, E2E_PROMPT, E2E_DECODE = 32, 4096, 256


def measure_model(world: int, prompt_len: int = E2E_PROMPT, decode: int = E2E_DECODE):
    """Config 4: random-init Qwen3-8B through the engine's public API
    (``LLM(..., w4a4_checkpoint=..., tensor_parallel_size=world)`` then
    ``generate``): 32 requests of `prompt_len` uniform random token ids, serial
    prefill, then batch-32 greedy decode for `decode` tokens, CUDA graphs on,
    prefix reuse off; once with W4A4 linears and once with BF16 cuBLAS linears
    (the same-box comparator).  Decode tok/s = decode tokens / decode wall time
    (each step ends with the sampled token ids on the host)."""
    import gc
    import tempfile
    from nanovllm import LLM, SamplingParams
    model_dir = synthetic.write_qwen3_config(tempfile.mkdtemp(prefix="qwen3_8b_"))
    g = torch.Generator().manual_seed(2026)
    prompts = [torch.randint(0, synthetic.QWEN3_8B_CONFIG["vocab_size"], (prompt_len,), generator=g).tolist()
               for _ in range(E2E_REQUESTS)]
    params = SamplingParams(temperature=0.0, max_tokens=decode, ignore_eos=True)
    out = {"requests": E2E_REQUESTS, "prompt_tokens": prompt_len, "decode_tokens": decode,
           "model": "Qwen3-8B architecture, random init (36 layers, hidden 4096, 32/8 heads, vocab 151936)",
           "api": "nanovllm.LLM(...).generate, greedy, CUDA graphs, prefix reuse off", "tp": world}
    for arm, kw in (("w4a4", {"w4a4_checkpoint": "random"}), ("bf16", {})):
        llm = LLM(model_dir, load_format="dummy", max_model_len=prompt_len + decode + 8,
                  max_num_batched_tokens=16384, max_num_seqs=E2E_REQUESTS, tensor_parallel_size=world, **kw)
        try:
            llm.generate(prompts, params)
            st = dict(llm.stats)
        finally:
            llm.exit()
            del llm
            gc.collect()
            torch.cuda.empty_cache()
        out[arm] = {"decode_tok_s": st["decode_tokens"] / st["decode_s"],
                    "ms_per_decode_step": st["decode_s"] / st["decode_steps"] * 1e3,
                    "prefill_tok_s": st["prefill_tokens"] / st["prefill_s"], **st}
    out["decode_speedup_w4a4_vs_bf16"] = out["w4a4"]["decode_tok_s"] / out["bf16"]["decode_tok_s"]
    return out


# ---------------------------------------------------------------- one kernel (profiling)
def run_kernel(spec: str, reps: int) -> None:
    """``--kernel NAME:MxNxK``: one kernel on one shape, a few warm-up launches
    and `reps` timed ones (the small, self-contained command the ncu summaries
    in profiles/ are captured from).  NAME is w4a4 (activation prep + grouped
    GEMM; M > 64 takes the tcgen05 prefill kernel, fewer tokens the decode
    kernel) or w4a16 (W4A16Linear)."""
    name, shape = spec.split(":")
    m, n, k = (int(v) for v in shape.lower().split("x"))
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(1)
    x = torch.randn(m, k, device=device, generator=g).bfloat16()
    if name == "w4a4":
        from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
        from nanovllm.layers.linear_w4a4 import W4A4Linear
        mod = W4A4Linear(k, n, layout="block128", clamp_lo=-8).to(device)
        packed = torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=device, generator=g)
        scale = (torch.randn(n, k // 128, device=device, generator=g).abs() * (0.02 / 7)).bfloat16()
        signs = torch.randint(0, 2, (k,), device=device, generator=g, dtype=torch.int8) * 2 - 1
        mod.load_full(packed, scale, signs)
        codes, sa = mod.quantize_input(x)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=device)

        def call():
            w4a4_grouped_gemm_i8(codes, mod.packed_weight, sa, mod.weight_scale, out=out)
        work, unit = 2 * m * n * k / 1e12, "TOPS"
    elif name == "w4a16":
        from nanovllm.layers.linear_w4a16 import W4A16Linear
        lin = W4A16Linear(k, n).to(device)
        with torch.no_grad():
            lin.qweight.copy_(torch.randint(-2 ** 31, 2 ** 31 - 1, lin.qweight.shape, dtype=torch.int64,
                                            device=device, generator=g).to(torch.int32))
            lin.qzeros.copy_(torch.randint(-2 ** 31, 2 ** 31 - 1, lin.qzeros.shape, dtype=torch.int64,
                                           device=device, generator=g).to(torch.int32))
            lin.scales.copy_((torch.randn(lin.scales.shape, device=device, generator=g).abs() * 0.02).half())

        def call():
            lin(x)
        work, unit = 2 * m * n * k / 1e12, "TFLOPS"
    else:
        raise SystemExit(f"unknown kernel {name!r} (w4a4 or w4a16)")
    with torch.no_grad():
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            call()
        end.record()
        end.synchronize()
    t = start.elapsed_time(end) / 1e3 / reps
    print(json.dumps({"kernel": spec, "us_per_call": t * 1e6, unit.lower(): work / t}), flush=True)


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default=None, choices=["tp", "dp"],
                    help="multi-GPU partition: tensor parallel (default for N > 1) or data-parallel replicas")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config measurements (1 GPU)")
    ap.add_argument("--no-model", action="store_true", help="skip the end-to-end model (config 4)")
    ap.add_argument("--kernel", default=None, metavar="NAME:MxNxK",
                    help="time one kernel on one shape (w4a4 or w4a16), e.g. w4a4:4096x24576x4096; the command "
                         "the ncu summaries in profiles/ are captured from")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.kernel:
        return run_kernel(args.kernel, max(1, args.steps if args.steps != 200 else 10))
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    mode = args.mode or ("tp" if world > 1 else "single")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    tp = world if mode == "tp" else 1
    mods = build_layers(device, args.layers, rank if tp > 1 else 0, tp)
    x_host = synthetic.activations(M_TOKENS, 4096, seed=0).pin_memory()
    x_dev = x_host.to(device)
    stream = torch.cuda.current_stream(device)

    with torch.no_grad():
        y = forward(mods, x_dev)            # eager warm-up (kernel attributes, peer buffers)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = forward(mods, x_dev)
    y_host = torch.empty(y.shape, dtype=y.dtype).pin_memory()

    for _ in range(args.warmup):
        graph.replay()
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    dt = time_graph(graph, args.steps, stream)
    clocks = sampler.stop()
    barrier()
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([dt], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())

    # end to end: host input -> graph -> host output, every step
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        x_dev.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(y, non_blocking=True)
    end.record(stream)
    end.synchronize()
    dt_e2e = start.elapsed_time(end) / 1e3
    if world > 1:
        t = torch.tensor([dt_e2e], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt_e2e = float(t.item())
    from nanovllm import _native
    device_error = _native.device_error()

    # roofline of the dominant kernel: the gate/up GEMM (M=32, this rank's
    # N shard), timed over one launch per layer (distinct weights)
    from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
    gu = [layer["gate_up"] for layer in mods]
    with torch.no_grad():
        pa, sa = gu[0].quantize_input(x_dev)
        outs = [torch.empty(M_TOKENS, g.out_features, dtype=torch.bfloat16, device=device) for g in gu]

        def gu_gemms():
            for g, o_ in zip(gu, outs):
                w4a4_grouped_gemm_i8(pa, g.packed_weight, sa, g.weight_scale, out=o_)
        t_gemm = time_launches(gu_gemms, len(gu), stream, max(5, args.steps // 4))
    n_gu = gu[0].out_features
    gemm_b = gemm_bytes(M_TOKENS, n_gu, 4096)
    peaks, peak_kind = measured_peaks()
    achieved = gemm_b / t_gemm / 1e9

    total_bytes = step_bytes(M_TOKENS, args.layers)
    weight_bytes = args.layers * sum(n * k // 2 + 2 * n * k // 128 for _, n, k in SHAPES)
    replicas = world if mode == "dp" else 1
    value = replicas * total_bytes * args.steps / dt / 1e9  # whole-job bytes over the slowest rank's time
    e2e = replicas * total_bytes * args.steps / dt_e2e / 1e9
    launches_per_layer = 8 + (2 if tp > 1 else 0)  # + the tile reduce of the two row-parallel layers
    launches = launches_per_layer * args.layers * args.steps
    parallelism = {"single": "single GPU", "dp": f"dp{world} (replicas, batch 32 each)",
                   "tp": f"tp{world} (QKV, gate/up N-sharded; O, down K-sharded, NVLink peer-memory sum)"}[mode]
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak" if mode == "dp" else "strong", "vs_baseline": None,
        "dtype": "int4xint4->fp32 (bf16 in/out)",
        "data": "synthetic (random-init weights, N(0,1) activations)",
        "config": {"workload": "config1-decode-chain", "m_tokens": M_TOKENS, "layers": args.layers,
                   "shapes": {n: [nn, kk] for n, nn, kk in SHAPES}, "layout": "block128", "clamp_lo": -8,
                   "parallelism": parallelism, "global_batch": M_TOKENS * replicas,
                   "l2": f"weights {weight_bytes / 1e9:.2f} GB per step vs 126 MB L2, no flush",
                   "bytes_per_step": total_bytes},
        "tok_s_linears": replicas * M_TOKENS * args.steps / dt,
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": x_host.numel() * 2,
                "d2h_bytes_per_step": y_host.numel() * 2, "ms_per_step": dt_e2e / args.steps * 1e3,
                "api": "W4A4*ParallelLinear.forward chain captured in a CUDA graph"},
        "gpu_launches": launches,
        "device_error": device_error,
        "roofline": {"bound": "hbm", "kernel": f"w4a4 grouped GEMM gate_up M=32 N={n_gu} K=4096",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind, "bytes_per_launch": gemm_b,
                     "us_per_launch": t_gemm * 1e6,
                     "traffic": profiled_traffic() if tp == 1 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                       "profiles/w4a4_stream_gemm_m32.md"},
        "clocks": clocks,
    }
    del graph
    if world == 1 and not args.no_extras:
        with torch.no_grad():
            cfg = {"decode": measure_decode(mods, device, stream, peaks["hbm_gbs"])}
            del mods, gu, outs
            torch.cuda.empty_cache()
            mods_small = build_layers(device, 3, 0, 1)
            cfg["int8_peak"] = int8_peak(device, stream)
            cfg["prefill"] = measure_prefill(mods_small, device, stream, cfg["int8_peak"])
            del mods_small
            torch.cuda.empty_cache()
            cfg["w4a16"] = measure_w4a16(device, stream, peaks)
            cfg["bf16_chain"] = measure_bf16_chain(device, stream, args.layers, x_dev)
            cfg["bf16_chain"]["w4a4_speedup"] = cfg["bf16_chain"]["ms_per_step"] / (dt / args.steps * 1e3)
        cfg["peaks"] = {"hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"],
                        "bf16_tflops_sustained": peaks["bf16_tflops_sustained"], "kind": peak_kind}
        line["configs"] = cfg
    if not args.no_model and mode != "dp":
        mods = gu = outs = None  # the chain's weights are not needed any more
        torch.cuda.empty_cache()
        try:
            line["model_decode"] = measure_model(world)
        except Exception as e:  # the headline line still prints
            line["model_decode"] = {"error": repr(e)[:300]}
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        if tp > 1:
            from nanovllm.layers.linear_w4a4 import release_peer_buffers
            release_peer_buffers()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
