"""Benchmark of the W4A4 quantized-linear hot path on B200.

Workload (BASELINE config 1 at batch 32, Qwen3-8B shapes): one *step* is the
chained forward of the four W4A4 projections of all 36 decoder layers at M=32
tokens -- QKV (K=4096 -> N=6144), O (4096 -> 4096), gate/up (4096 -> 24576),
down (12288 -> 4096) -- each one activation-prep launch (block128 RHT +
per-group INT4 quantisation + packing, codes in [-8, 7]) and one grouped INT4
GEMM launch, with distinct random weights per layer (3.58 GB, larger than L2,
so no flush is needed).  The projections are chained as in a Qwen3 decoder
layer with attention left out (it is not on the quantized-linear path): QKV's
prep applies the residual add + input RMSNorm, O reads the first M*K elements
of the QKV output viewed as [M, K] (no copy kernel), gate/up's prep applies
the residual add + post-attention RMSNorm, and down's prep reads the whole
gate/up output and applies the MLP's SiluAndMul -- each producer fused into
the prep kernel, so the norms keep the activations in range as in the model.
The step is captured in a CUDA graph and replayed, as the reference's model
runner does for decode.

With ``--gpus N`` (torchrun, one rank per GPU) every rank runs the same chain
on its own batch of 32 with its own copy of the weights -- data-parallel
decode replicas, weak scaling, the device time taken as the maximum over
ranks.  The tensor-parallel layers (``W4A4*ParallelLinear`` with the
peer-memory row-parallel sum) are tested for parity on 2-4 GPUs, and the
36-layer TP=2 chain has run clean; they are not benchmarked here until the
TP=4 and TP=8 chains have been run end to end as well.

``--impl reference`` times the reference algorithm on the host CPU instead (the
numpy oracle port of the reference's PyTorch path), on one layer of the same
chained workload per step.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-int4_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from nanovllm.utils import synthetic  # noqa: E402

M_TOKENS = 32
LAYERS = 36
SHAPES = [("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 24576, 4096), ("down", 4096, 12288)]
METRIC = "W4A4 decode linears HBM GB/s (Qwen3-8B shapes, batch 32, 36 layers)"


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


def layer_bytes(m: int, first: bool) -> int:
    """One decoder layer of the chain: QKV (RMSNorm, plus the residual add after
    the first layer), O, gate/up (residual add + RMSNorm), down (SiluAndMul)."""
    norms = {"qkv": 1 if first else 2, "o": 0, "gate_up": 2, "down": 0}
    return sum(linear_bytes(m, n, k, silu=name == "down", norm=norms[name]) for name, n, k in SHAPES)


def step_bytes(m: int, layers: int) -> int:
    return layer_bytes(m, True) + (layers - 1) * layer_bytes(m, False)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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
NORM_EPS = 1e-6


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


# ---------------------------------------------------------------- CPU (oracle port) sample
def f32_bits(x):
    """float32 array -> BF16 bit patterns (round to nearest even)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def cpu_layer_sample(seed=0):
    """One layer of the chained workload on the host, with the oracle port of the
    reference algorithm (block128, clamp -8).  Returns (seconds, bytes)."""
    sys.path.insert(0, ROOT)
    from oracle import nv4_oracle as o
    x = synthetic.activations(M_TOKENS, 4096, seed)
    weights = []
    for name, n, k in SHAPES:
        codes, packed, scale = synthetic.w4a4_weights(n, k, seed + n)
        signs = synthetic.make_signs(k, seed + k)
        weights.append((n, k, packed.numpy().view(np.uint8), scale.view(torch.int16).numpy().view(np.uint16),
                        signs.numpy(), codes.numpy()))
    xb = x.view(torch.int16).numpy().view(np.uint16)

    norm_w = f32_bits(np.ones(4096, dtype=np.float32))
    res0 = xb.copy()

    def run():
        h, res = xb, res0
        for (name, _, _), (n, k, packed, sbits, signs, codes) in zip(SHAPES, weights):
            if name == "down":
                inp = o.silu_mul_bf16_bits(h)
            elif name in ("qkv", "gate_up"):
                inp, res = o.add_rmsnorm_bf16_bits(h, res, norm_w, NORM_EPS)
            else:
                inp = np.ascontiguousarray(h.reshape(-1)[: h.shape[0] * k].reshape(h.shape[0], k))
            h = o.w4a4_linear(inp, signs, packed, sbits, o.LAYOUT_BLOCK128, -8, w_codes=codes)
        return h
    return run, layer_bytes(M_TOKENS, False)


def cpu_baseline(target_s=12.0):
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
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{reps} x one decoder layer (4 linears, M=32) of the chained workload, numpy oracle port"
                      f" of the reference PyTorch path, {dt * 1e3:.0f} ms each"}


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
    cb = {"value": value, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
          "sample": "one decoder layer (4 linears, M=32) of the chained workload per step, numpy oracle port"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int4xint4->fp32",
        "data": "synthetic", "config": {"workload": "config1-decode-chain-1layer-cpu", "m_tokens": M_TOKENS,
                                        "layers": 1, "layout": "block128", "clamp_lo": -8},
        "cpu_baseline": cb, "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0}}), flush=True)


# ---------------------------------------------------------------- GPU arm
def time_graph(graph, steps, stream):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / 1e3


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    import datetime
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    mods = build_layers(device, args.layers, 0, 1)  # a full replica per rank
    x_host = synthetic.activations(M_TOKENS, 4096, seed=0).pin_memory()
    x_dev = x_host.to(device)
    stream = torch.cuda.current_stream(device)

    with torch.no_grad():
        y = forward(mods, x_dev)            # eager warm-up (sets kernel attributes)
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

    # roofline of the dominant kernel: the gate/up GEMM (N=24576, K=4096, M=32) on
    # this rank's shard, timed over one launch per layer (distinct weights)
    from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8 as w4a4_grouped_gemm
    gu = [layer["gate_up"] for layer in mods]
    with torch.no_grad():
        pa, sa = gu[0].quantize_input(x_dev)
        outs = [torch.empty(M_TOKENS, g.out_features, dtype=torch.bfloat16, device=device) for g in gu]
        for g, o_ in zip(gu, outs):
            w4a4_grouped_gemm(pa, g.packed_weight, sa, g.weight_scale, out=o_)
        g_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_graph):
            for g, o_ in zip(gu, outs):
                w4a4_grouped_gemm(pa, g.packed_weight, sa, g.weight_scale, out=o_)
    for _ in range(3):
        g_graph.replay()
    torch.cuda.synchronize()
    reps = max(5, args.steps // 4)
    t_gemm = time_graph(g_graph, reps, stream) / (reps * len(gu))
    n_gu = gu[0].out_features
    gemm_b = gemm_bytes(M_TOKENS, n_gu, 4096)
    peak, peak_kind = measured_peaks()
    achieved = gemm_b / t_gemm / 1e9

    total_bytes = step_bytes(M_TOKENS, args.layers)
    weight_bytes = args.layers * sum(n * k // 2 + 2 * n * k // 128 for _, n, k in SHAPES)
    value = world * total_bytes * args.steps / dt / 1e9  # all replicas' bytes over the slowest rank's time
    e2e = world * total_bytes * args.steps / dt_e2e / 1e9
    launches = 2 * 4 * args.layers * args.steps
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4xint4->fp32 (bf16 in/out)",
            "data": "synthetic (random-init weights, N(0,1) activations)",
            "config": {"workload": "config1-decode-chain", "m_tokens": M_TOKENS, "layers": args.layers,
                       "shapes": {n: [nn, kk] for n, nn, kk in SHAPES}, "layout": "block128", "clamp_lo": -8,
                       "parallelism": "single GPU" if world == 1 else f"dp{world} (replicas, batch 32 each)",
                       "global_batch": M_TOKENS * world,
                       "l2": f"weights {weight_bytes / 1e9:.2f} GB per step vs 126 MB L2, no flush",
                       "bytes_per_step": total_bytes},
            "tok_s_linears": world * M_TOKENS * args.steps / dt,
            "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": x_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 2, "ms_per_step": dt_e2e / args.steps * 1e3,
                    "api": "W4A4*ParallelLinear.forward chain captured in a CUDA graph"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": f"w4a4 grouped GEMM gate_up M=32 N={n_gu} K=4096",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "bytes_per_launch": gemm_b, "us_per_launch": t_gemm * 1e6,
                         "traffic": profiled_traffic(),
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, "
                                           "profiles/w4a4_stream_gemm_m32.md"},
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    del graph, g_graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
