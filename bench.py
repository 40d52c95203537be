"""Benchmark of the B200 quantized-inference path (one JSON line on rank 0).

Default workload (metric "int4 dequant-MatMul HBM GB/s"):
one decode step of a Llama-7B-shaped layer's weight-only int4 projections,
q/k/v/o [4096,4096], gate/up [4096,11008], down [11008,4096], int4 blocked
along K (block 128), FLOAT16 scales, no zero points, FLOAT16 activations
[B,1,4096] (B = --batch, default 1).  Each projection is one fused
DequantizeLinear -> MatMul call (b2_dequantize_matmul).  Inputs are seeded
synthetic data (onnx-light's SplitMix64 generators, produced on the device).

Timing: four copies of the layer's weights (417 MB > 126 MB L2) are used in
rotation, so every step streams its weights from HBM; each step is a CUDA
graph replay bracketed by CUDA events on the launching stream; W warm-up
steps, K timed steps, barrier + synchronize around the timed region, max over
ranks.  `value` = algorithmic bytes (packed weights + scales + activations in
and out) per step / device time.  `e2e` repeats the step through the public
Python API with host-resident activations: pinned H2D copy of the step input,
seven API calls, D2H of the result, all inside the timed region (weights stay
resident, as onnx-light initializers do).

--gpus N (torchrun): the weights are column-sharded; each rank computes its
output slice and the slices are all-gathered over NCCL after every
projection; `value` counts the whole layer's bytes once per step (strong
scaling).

--impl reference: onnx-light's own CPU kernels (oracle/_ref, compiled from the
reference sources) run the same chain on the host cores: DequantizeLinear then
MatMul for every projection.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "onnx-light_b200")

# Llama-7B layer projections: (name, K, N, input)
PROJ = [("q", 4096, 4096, "x"), ("k", 4096, 4096, "x"), ("v", 4096, 4096, "x"),
        ("o", 4096, 4096, "q"), ("gate", 4096, 11008, "o"), ("up", 4096, 11008, "o"),
        ("down", 11008, 4096, "gate")]
BLOCK = 128
NCOPIES = 4
INT4, FLOAT16 = 22, 10


def load_package():
    if "onnx_light_b200" in sys.modules:
        return sys.modules["onnx_light_b200"]
    spec = importlib.util.spec_from_file_location(
        "onnx_light_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["onnx_light_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def step_bytes(batch: int, shards: int = 1) -> int:
    """Algorithmic HBM bytes of one step: packed int4 weights + fp16 scales +
    fp16 activations read + fp16 outputs written (whole layer)."""
    total = 0
    for _, K, N, _ in PROJ:
        total += K * N // 2 + (K // BLOCK) * N * 2 + batch * K * 2 * shards + batch * N * 2
    return total


def step_flops(batch: int) -> int:
    return sum(2 * batch * K * N for _, K, N, _ in PROJ)


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._proc = None

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
        except (OSError, ValueError):
            self._proc = None
        return self

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        mx = max((float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for name, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def make_layer(b2, synth, copy: int, rank: int, world: int, device):
    """One copy of the layer's weights, column slice `rank` of `world`."""
    import torch  # noqa: F401
    layer = {}
    for j, (name, K, N, _) in enumerate(PROJ):
        n_loc = N // world
        seed = 3000 + 100 * copy + j
        codes = synth.randint(seed, (K * N,), -8, 7, device=device).view(K, N)
        codes = codes[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
        w = synth.convert(codes.view(-1), INT4, (K, n_loc))
        s = synth.uniform(seed + 50, (K // BLOCK, N), 0.002, 0.02, device=device)
        s = s[:, rank * n_loc:(rank + 1) * n_loc].contiguous()
        s16 = synth.convert(s.view(-1), FLOAT16, (K // BLOCK, n_loc))
        layer[name] = (w, s16)
    return layer


def gpu_arm(args):
    import torch
    import torch.distributed as dist

    b2 = load_package()
    from onnx_light_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    B = args.batch
    layers = [make_layer(b2, synth, c, rank, world, device) for c in range(NCOPIES)]
    x0 = synth.convert(synth.randn(2000, (B * 4096,), 0.0, 1.0, device=device), FLOAT16, (B, 4096))
    mm = b2.DequantizeMatMul()
    stream = torch.cuda.Stream(device)

    # Buffers: full activations per projection output, local slice outputs, gather buffers.
    acts = {"x": x0}
    loc = {}
    gat = {}
    for name, K, N, _ in PROJ:
        acts[name] = torch.empty((B, N), dtype=torch.float16, device=device)
        loc[name] = torch.empty((B, N // world), dtype=torch.float16, device=device)
        gat[name] = torch.empty((world, B, N // world), dtype=torch.float16, device=device)

    def run_step(layer):
        for name, K, N, src in PROJ:
            w, s = layer[name]
            if world == 1:
                mm(acts[src], w, s, None, axis=0, out=acts[name])
            else:
                mm(acts[src], w, s, None, axis=0, out=loc[name])
                dist.all_gather_into_tensor(gat[name].view(-1), loc[name].view(-1))
                acts[name].copy_(gat[name].permute(1, 0, 2).reshape(B, N))

    # warm up the library (plans, function attributes, workspace) outside capture
    with torch.cuda.stream(stream):
        for layer in layers:
            run_step(layer)
    torch.cuda.synchronize()

    use_graph = world == 1
    graphs = []
    if use_graph:
        for layer in layers:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run_step(layer)
            graphs.append(g)

    def launch(i):
        if use_graph:
            graphs[i % NCOPIES].replay()
        else:
            with torch.cuda.stream(stream):
                run_step(layers[i % NCOPIES])

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for i in range(args.steps):
            starts[i].record(stream)
            with torch.cuda.stream(stream):
                launch(i)
            ends[i].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    nbytes = step_bytes(B)
    value = nbytes / (ms * 1e-3) / 1e9

    # Dominant kernel: time each projection's GEMV alone (events on its stream),
    # rotating weight copies so every launch reads from HBM.
    roof = None
    if rank == 0:
        per = []
        with torch.cuda.stream(stream):
            for name, K, N, src in PROJ:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 8
                out = acts[name] if world == 1 else loc[name]
                for c in range(NCOPIES):  # warm
                    w, s = layers[c][name]
                    mm(acts[src], w, s, None, axis=0, out=out)
                ev0.record(stream)
                for r in range(reps):
                    w, s = layers[r % NCOPIES][name]
                    mm(acts[src], w, s, None, axis=0, out=out)
                ev1.record(stream)
                torch.cuda.synchronize()
                t_launch = ev0.elapsed_time(ev1) / reps
                n_loc = N // world
                b = K * n_loc // 2 + (K // BLOCK) * n_loc * 2 + B * K * 2 + B * n_loc * 2
                per.append((name, b, t_launch))
        tot_b = sum(p[1] for p in per)
        tot_t = sum(p[2] for p in per)
        peak, peak_src = measured_peak()
        achieved = tot_b / (tot_t * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "dq_gemv", "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": peak_src, "traffic": traffic_from_profile(),
                "per_launch_us": {p[0]: round(p[2] * 1e3, 2) for p in per},
                "algorithmic_bytes_per_step": tot_b}

    # e2e: public API with host buffers, H2D of x and D2H of the step's result.
    e2e = None
    if rank == 0 and world == 1:
        x_host = x0.cpu().pin_memory()
        y_host = torch.empty((B, 4096), dtype=torch.float16).pin_memory()
        for i in range(args.warmup):
            with torch.cuda.stream(stream):
                acts["x"].copy_(x_host, non_blocking=True)
                run_step(layers[i % NCOPIES])
                y_host.copy_(acts["down"], non_blocking=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                acts["x"].copy_(x_host, non_blocking=True)
                run_step(layers[i % NCOPIES])
                y_host.copy_(acts["down"], non_blocking=True)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps
        dev_ms = ev0.elapsed_time(ev1) / args.steps
        e2e_ms = max(wall * 1e3, dev_ms)
        e2e = {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
               "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": B * 4096 * 2,
               "d2h_bytes_per_step": B * 4096 * 2,
               "path": "DequantizeMatMul python API -> b2_dequantize_matmul, no graph"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(B)

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": "int4 dequant-MatMul HBM GB/s (Llama-7B decode layer, config 3)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights, fp16 activations",
            "data": "synthetic (SplitMix64 seeded, generated on device)",
            "config": {"workload": "config3: Llama-7B int4 decode layer (q,k,v,o,gate,up,down)",
                       "batch": B, "block_size": BLOCK, "scales": "fp16", "zero_points": "none",
                       "parallelism": f"column-sharded tp{world}" if world > 1 else "single GPU",
                       "l2_policy": f"{NCOPIES} weight copies in rotation "
                                    f"({NCOPIES * step_bytes(B) / 1e6:.0f} MB > 126 MB L2)",
                       "launch": "CUDA graph per step" if use_graph else "eager + NCCL all_gather"},
            "tflops": round(step_flops(B) / (ms * 1e-3) / 1e12, 3),
            "gpu_launches": 7 * args.steps if world == 1 else 7 * args.steps,
            "clocks": clocks,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def traffic_from_profile():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get("dq_gemv")
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------
# CPU baseline / reference arm (onnx-light's own kernels on the host cores)
# ---------------------------------------------------------------------------

def _ref_inputs(B, proj_subset):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    data = {}
    for j, (name, K, N, _) in enumerate(PROJ):
        if name not in proj_subset:
            continue
        seed = 3000 + j
        w = O.pack_bits(O.randint(seed, (K * N,), -8, 7), 4)
        s = O.f32_to_f16_bits(O.rand_uniform(seed + 50, (K // BLOCK * N,), 0.002, 0.02))
        data[name] = (w, s)
    x = O.f32_to_f16_bits(O.randn(2000, (B, 4096)))
    return O, np, data, x


def _ref_step(O, np, data, x, B, proj_subset):
    acts = {"x": x}
    for name, K, N, src in PROJ:
        if name not in proj_subset:
            continue
        w, s = data[name]
        wq = O.ref_dequantize_linear(w, O.INT4, (K, N), s, O.FLOAT16, (K // BLOCK, N), None, None, 0)
        acts[name] = O.ref_matmul(acts[src], wq, O.FLOAT16)
    return acts


def cpu_baseline_sample(B):
    """Times the reference CPU path on a bounded sample: the q projection
    (DequantizeLinear + MatMul, 4096x4096) once, scaled to the metric's unit."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        kind = "reference" if O.ref_available() else None
        if kind is None:
            return {"value": None, "unit": "GB/s", "cores": 0, "kind": "unavailable",
                    "sample": "oracle/_ref not built on this host"}
        subset = ("q",)
        O, np, data, x = _ref_inputs(B, subset)
        _ref_step(O, np, data, x, B, subset)  # warm
        t0 = time.perf_counter()
        reps = 2
        for _ in range(reps):
            _ref_step(O, np, data, x, B, subset)
        t = (time.perf_counter() - t0) / reps
        K, N = 4096, 4096
        b = K * N // 2 + (K // BLOCK) * N * 2 + B * K * 2 + B * N * 2
        return {"value": round(b / t / 1e9, 4), "unit": "GB/s", "cores": O.ref_thread_count(),
                "kind": "reference",
                "sample": f"q projection (DequantizeLinear int4 4096x4096 + MatMul fp16, B={B}), "
                          f"{t * 1e3:.1f} ms per call, onnx-light kernels compiled from source"}
    except Exception as e:  # the baseline must never break the GPU line
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "error", "sample": repr(e)[:200]}


def reference_arm(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    B = args.batch
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libref.so not built"}))
        return
    subset = tuple(p[0] for p in PROJ)
    O, np, data, x = _ref_inputs(B, subset)
    for _ in range(args.warmup):
        _ref_step(O, np, data, x, B, subset)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _ref_step(O, np, data, x, B, subset)
    t = (time.perf_counter() - t0) / args.steps
    value = step_bytes(B) / t / 1e9
    cores = O.ref_thread_count()
    sample = (f"full config-3 layer (7 x DequantizeLinear + MatMul fp16, B={B}) per step, "
              f"onnx-light kernels compiled from source, {cores} threads")
    print(json.dumps({
        "impl": "reference",
        "metric": "int4 dequant-MatMul HBM GB/s (Llama-7B decode layer, config 3)",
        "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights, fp16 activations",
        "data": "synthetic (SplitMix64 seeded)",
        "config": {"workload": "config3: Llama-7B int4 decode layer (q,k,v,o,gate,up,down)",
                   "batch": B, "block_size": BLOCK},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
