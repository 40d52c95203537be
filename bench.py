"""Benchmark of the B200 quantized-inference path (one JSON line on rank 0).

Default workload (metric "int4 dequant-MatMul HBM GB/s"):
one decode step of a Llama-7B-shaped layer's weight-only int4 projections,
q/k/v/o [4096,4096], gate/up [4096,11008], down [11008,4096], int4 blocked
along K (block 128), FLOAT16 scales, no zero points, FLOAT16 activations
[B,1,4096] (B = --batch, default 1).  Each projection is one fused
DequantizeLinear -> MatMul; projections that read the same activations run as
one call (q/k/v, gate/up: b2_dequantize_matmul_group, one launch whose CTAs
split all their weight tiles), so a step is 4 launches; the line's `per_node`
entry times the same step with one call per ONNX node (7 launches of
b2_dequantize_matmul).  Inputs are seeded synthetic data (onnx-light's
SplitMix64 generators, produced on the device).

Timing: four copies of the layer's weights (417 MB > 126 MB L2) are used in
rotation, so every step streams its weights from HBM; each step is a CUDA
graph replay bracketed by CUDA events on the launching stream; W warm-up
steps, K timed steps, barrier + synchronize around the timed region, max over
ranks.  `value` = algorithmic bytes (packed weights + scales + activations in
and out) per step / device time.  `e2e` repeats the step through the public
Python API with host-resident activations: pinned H2D copy of the step input,
four API calls, D2H of the result, all inside the timed region (weights stay
resident, as onnx-light initializers do).

--gpus N (torchrun): the weights are column-sharded; each rank computes its
output slice and the decode kernel stores it into every rank's output over
NVLink (peer stores; b2_allgather_cols after each projection above 16 rows);
`value` counts the whole layer's bytes once per step (strong scaling).

--impl reference: onnx-light's own CPU kernels (oracle/_ref, compiled from the
reference sources) run the same chain on the host cores: DequantizeLinear then
MatMul for every projection.
"""
from __future__ import annotations

import argparse
import contextlib
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
# The step's projections that read the same activations run as one call
# (DequantizeMatMulGroup -> b2_dequantize_matmul_group: one launch whose CTAs
# split all the members' weight tiles): q / k / v, o, gate / up, down.
GROUPS = [(("q", "k", "v"), "x"), (("o",), "q"), (("gate", "up"), "o"), (("down",), "gate")]
BLOCK = 128
NCOPIES = 4
INT4, FLOAT16, BF16 = 22, 10, 16


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


def workload_config(batch: int) -> dict:
    """The workload both arms run (identical dicts: the reference arm's column
    slice is reported beside it, not in it)."""
    return {"workload": "config3: Llama-7B int4 decode layer (q,k,v,o,gate,up,down)",
            "batch": batch, "block_size": BLOCK, "weights": "int4 [-8, 7]",
            "scales": "fp16 [0.002, 0.02]", "zero_points": "none", "activations": "fp16 N(0,1)"}


def step_flops(batch: int) -> int:
    return sum(2 * batch * K * N for _, K, N, _ in PROJ)


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """SM clock and throttle reasons of one GPU, polled through NVML every
    ~2 ms on a background thread while the block runs (nvidia-smi's fastest
    loop, 100 ms, would miss a timed region of a few tens of milliseconds)."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = self.gpu
            if vis:
                try:
                    index = int(vis.split(",")[self.gpu])
                except ValueError:
                    index = self.gpu
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def _poll(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(0.002)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        sm = sorted(m for m, _ in self.samples)
        reasons = sorted({name for _, r in self.samples for name, bit in self.REASONS if r & bit})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "NVML, 2 ms polling over the timed region"}


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
    gm = b2.DequantizeMatMulGroup()
    stream = torch.cuda.Stream(device)

    # Buffers: the full activation of every projection output and, sharded,
    # this rank's column slice.  Sharded, the full outputs are peer buffers:
    # b2_allgather_cols stores each rank's slice into every rank's copy over
    # NVLink (sharding.PeerGroup), one kernel per projection.
    acts = {"x": x0}
    loc = {}
    peers = None
    if world > 1:
        from onnx_light_b200.sharding import PeerGroup
        peers = PeerGroup()
    for name, K, N, _ in PROJ:
        if world == 1:
            acts[name] = torch.empty((B, N), dtype=torch.float16, device=device)
        else:
            acts[name] = peers.buffer(name, (B, N), torch.float16)
            loc[name] = torch.empty((B, N // world), dtype=torch.float16, device=device)

    # Sharded decode (up to 16 rows): the fused kernel stores each rank's
    # column slice into every rank's output itself (b2_dequantize_matmul_peer,
    # b2_dequantize_matmul_group_peer) and a call whose input is such an
    # output first waits for every rank's previous call.  That chain also
    # orders every overwrite of a peer buffer after its readers on all ranks
    # (each buffer's next writer waits, directly or through its stream, for
    # a call that follows those readers on every rank), so a step needs no
    # wait of its own; a host read of an output waits first (peers.wait).
    # Larger batches: each rank's slice, then b2_allgather_cols.
    fused = world > 1 and B <= 16

    def run_step(layer, per_node=False):
        if per_node:
            # one call per ONNX node (b2_dequantize_matmul, _peer)
            for name, K, N, src in PROJ:
                w, s = layer[name]
                if world == 1:
                    mm(acts[src], w, s, None, axis=0, out=acts[name])
                elif fused:
                    peers.matmul(name, acts[src], w, s)
                else:
                    mm(acts[src], w, s, None, axis=0, out=loc[name])
                    peers.gather(name, loc[name])
            return
        for names, src in GROUPS:
            ws = [layer[n][0] for n in names]
            ss = [layer[n][1] for n in names]
            if fused:
                peers.matmul_group(names, acts[src], ws, ss)
            elif world == 1:
                if len(names) == 1:
                    mm(acts[src], ws[0], ss[0], None, axis=0, out=acts[names[0]])
                else:
                    gm(acts[src], ws, ss, axis=0, outs=[acts[n] for n in names])
            else:
                gm(acts[src], ws, ss, axis=0, outs=[loc[n] for n in names])
                for n in names:
                    peers.gather(n, loc[n])

    def run_steps(n, offset, per_node=False):
        for i in range(n):
            run_step(layers[(offset + i) % NCOPIES], per_node)

    # Warm the library (plans, function attributes, workspace, NCCL
    # communicators) outside capture.
    with torch.cuda.stream(stream):
        run_steps(NCOPIES, 0)
        run_steps(NCOPIES, 0, per_node=True)
    torch.cuda.synchronize()

    # The steps run as CUDA graphs of up to CHUNK steps each (the peer gathers
    # captured too when sharded), so the device time measured is the steps'
    # own and never the host's launch rate.  K steps = K // CHUNK replays of the
    # chunk graph + one graph of the remainder.
    chunk = max(NCOPIES, min(256, args.steps) // NCOPIES * NCOPIES)
    graphs = {}

    def graph_of(n, per_node=False):
        if (n, per_node) not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run_steps(n, 0, per_node)
            graphs[(n, per_node)] = g
        return graphs[(n, per_node)]

    def play(n, per_node=False):
        with torch.cuda.stream(stream):
            for _ in range(n // chunk):
                graph_of(chunk, per_node).replay()
            if n % chunk:
                graph_of(n % chunk, per_node).replay()

    def timed(per_node, clk=None):
        """Device ms per step of args.steps steps after args.warmup, max over ranks."""
        graph_of(chunk, per_node)
        if args.steps % chunk:
            graph_of(args.steps % chunk, per_node)
        if args.warmup % chunk:
            graph_of(args.warmup % chunk, per_node)
        # Replay every graph of the timed region once before it (untimed extra
        # warm-up): the first replay of a graph uploads it to the device, which
        # a short timed region would otherwise pay inside its first step.
        with torch.cuda.stream(stream):
            for n in sorted({chunk, args.steps % chunk} - {0}):
                graph_of(n, per_node).replay()
        play(args.warmup, per_node)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with (clk if clk is not None else contextlib.nullcontext()):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            # a short device-side delay ahead of the start event keeps the GPU
            # busy while the host submits the graphs, so the events time the
            # steps' execution and not the submission (a 20-step region is
            # about 1 ms)
            with torch.cuda.stream(stream):
                torch.cuda._sleep(1_000_000)
            ev0.record(stream)
            play(args.steps, per_node)
            ev1.record(stream)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
        t_ms = ev0.elapsed_time(ev1) / args.steps
        if world > 1:
            t = torch.tensor([t_ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return t_ms

    clk = ClockSampler(local)
    ms = timed(False, clk)
    nbytes = step_bytes(B)
    value = nbytes / (ms * 1e-3) / 1e9
    # the same step with one call per ONNX node (7 launches), for comparison
    ms_node = timed(True)
    graphs.clear()
    if fused:
        with torch.cuda.stream(stream):
            peers.wait()
    torch.cuda.synchronize()

    # Roofline.  The fused decode kernel is the only kernel of a single-GPU
    # step (4 launches): achieved = algorithmic bytes of the step / step time.
    # Each projection is also timed alone: a graph of REPS launches rotating
    # the weight copies.
    roof = None
    if rank == 0:
        per = []
        reps = 8 * NCOPIES
        for name, K, N, src in PROJ:
            out = acts[name] if world == 1 else loc[name]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for r in range(reps):
                    w, s = layers[r % NCOPIES][name]
                    mm(acts[src], w, s, None, axis=0, out=out)
            with torch.cuda.stream(stream):
                g.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            n_loc = N // world
            b = K * n_loc // 2 + (K // BLOCK) * n_loc * 2 + B * K * 2 + B * n_loc * 2
            per.append((name, b, e0.elapsed_time(e1) / reps))
            del g
        peak, peak_src = measured_peak()
        if world == 1:
            achieved = nbytes / (ms * 1e-3) / 1e9
        else:
            achieved = sum(p[1] for p in per) / (sum(p[2] for p in per) * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": decode_kernel(B), "achieved": round(achieved, 1),
                "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": peak_src, "traffic": traffic_from_profile(B) if world == 1 else None,
                "traffic_unit": "DRAM bytes per step (ncu capture of batch 1, profiles/traffic.json)",
                "algorithmic_bytes_per_step": nbytes,
                "per_projection_us": {p[0]: round(p[2] * 1e3, 2) for p in per},
                "per_projection_gbs": {p[0]: round(p[1] / (p[2] * 1e-3) / 1e9, 1) for p in per}}

    # e2e: the public API (DequantizeMatMul -> b2_dequantize_matmul) with the
    # step input copied from pinned host memory and the step result copied
    # back to pinned host memory inside every step; the calls are captured in
    # CUDA graphs the way a serving loop captures its decode step.
    e2e = None
    if world > 1:
        dist.barrier()  # rank 0 timed the projections alone; line the ranks up again
    if rank == 0 or world > 1:  # sharded: every rank takes part (the gathers wait for all)
        x_host = x0.cpu().pin_memory()
        y_host = torch.empty((B, 4096), dtype=torch.float16).pin_memory()

        def e2e_steps(n):
            for i in range(n):
                acts["x"].copy_(x_host, non_blocking=True)
                run_step(layers[i % NCOPIES])
                if fused:
                    peers.wait()  # every rank's slice of the result is in
                y_host.copy_(acts["down"], non_blocking=True)

        ge = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ge, stream=stream):
            e2e_steps(chunk)
        with torch.cuda.stream(stream):
            ge.replay()
        torch.cuda.synchronize()
        reps_e2e = max(1, args.steps // chunk)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps_e2e):
                ge.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / (reps_e2e * chunk)
        dev_ms = e0.elapsed_time(e1) / (reps_e2e * chunk)
        e2e_ms = max(wall * 1e3, dev_ms)
        if world > 1:
            t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
               "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": B * 4096 * 2,
               "d2h_bytes_per_step": B * 4096 * 2,
               "path": "DequantizeMatMulGroup / DequantizeMatMul python API -> "
                       "b2_dequantize_matmul_group / b2_dequantize_matmul, pinned H2D + "
                       "4 calls + D2H per step, captured in CUDA graphs"
                       + ((" (fused peer stores, b2_dequantize_matmul_group_peer / _peer, a "
                           "completion wait before the D2H, max over ranks)" if fused
                           else " (+ b2_allgather_cols per projection, max over ranks)")
                          if world > 1 else "")}
        del ge

    # Sharded: the gathered full output of a step against the unsharded
    # projection computed on this rank (rel-L2, contract 1e-3).
    gather_check = None
    if world > 1:
        with torch.cuda.stream(stream):
            run_step(layers[0])
            if fused:
                peers.wait()
        torch.cuda.synchronize()
        full = make_layer(b2, synth, 0, 0, 1, device)
        ref_q = mm(x0, full["q"][0], full["q"][1], None, axis=0)
        torch.cuda.synchronize()
        err = float(((acts["q"].float() - ref_q.float()).norm() / ref_q.float().norm()).item())
        t = torch.tensor([err], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gather_check = {"projection": "q", "rel_l2_max_over_ranks": float(t.item()),
                        "ok": float(t.item()) <= 1e-3}
        del full, ref_q

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(B)

    # Secondary BASELINE metrics (same GPU, after the headline timing).
    secondary = None
    if world > 1 and not args.no_secondary:
        # the sharded configurations, every rank taking part
        secondary = {"attention_config4_sharded":
                     attention_config4_sharded(b2, synth, device, stream, peers, world, rank)}
    if rank == 0 and world == 1 and not args.no_secondary:
        want_cpu = not args.no_cpu_baseline
        secondary = {}
        for bb in (8, 32, 64):
            secondary[f"decode_config3_b{bb}"] = decode_config3(b2, layers, device, stream, bb,
                                                                want_cpu)
        secondary["dq_matmul_config1"] = dq_matmul_config1(b2, synth, device, stream, want_cpu)
        secondary["dequantize_linear"] = dequantize_standalone(b2, synth, device, stream, want_cpu)
        secondary["decoder_ops"] = decoder_ops(b2, synth, device, stream, want_cpu)
        secondary["attention_config4"] = attention_config4(b2, synth, device, stream, want_cpu)
        secondary["matmul_integer_config2"] = matmul_integer_config2(b2, synth, device, stream,
                                                                     want_cpu)
        secondary["prefill_config5"] = prefill_config5(b2, synth, device, stream, want_cpu)

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": "int4 dequant-MatMul HBM GB/s (Llama-7B decode layer, config 3)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights, fp16 activations",
            "data": "synthetic (SplitMix64 seeded, generated on device)",
            "config": workload_config(B),
            "parallelism": f"column-sharded over {world} GPUs" if world > 1 else "single GPU",
            "timing": {"l2_policy": f"{NCOPIES} weight copies in rotation "
                                    f"({NCOPIES * step_bytes(B) / 1e6:.0f} MB > 126 MB L2)",
                       "launch": f"CUDA graphs of {chunk} steps; projections sharing an input "
                                 "in one call (q/k/v, gate/up): 4 launches per step"
                                 + ((" with the column slices stored into every rank's output "
                                     "by the decode kernel itself (b2_dequantize_matmul_group_peer"
                                     " / _peer)" if fused else
                                     " with a peer-store all-gather (b2_allgather_cols) per "
                                     "projection") if world > 1 else "")},
            "per_node": {"value": round(nbytes / (ms_node * 1e-3) / 1e9, 1), "unit": "GB/s",
                         "ms_per_step": round(ms_node, 5),
                         "launches_per_step": 7 if (world == 1 or fused) else 14,
                         "note": "the same step with one call per ONNX node "
                                 "(DequantizeMatMul -> b2_dequantize_matmul"
                                 + (", _peer" if fused else "") + ")"},
            "tflops": round(step_flops(B) / (ms * 1e-3) / 1e12, 3),
            "gpu_launches": (4 if (world == 1 or fused) else 11) * args.steps,
            "gather_check": gather_check,
            "clocks": clocks,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        graphs.clear()
        torch.cuda.synchronize()
        peers.close()
        dist.barrier()
        dist.destroy_process_group()


def _pinned_like(t):
    import torch
    return torch.empty(t.shape, dtype=t.dtype).pin_memory()


def _e2e(stream, step_fn, h2d, d2h, reps, chunk):
    """End-to-end ms per step: every step copies its inputs from pinned host
    memory (h2d: list of (device tensor, pinned host tensor)), runs step_fn
    (the public API calls) and copies its result back to pinned host memory
    (d2h: list of (pinned host tensor, device tensor)); the steps are captured
    in CUDA graphs of `chunk` steps, as a serving loop captures its step.
    Returns (ms, h2d bytes, d2h bytes); ms = max(wall clock, device time)."""
    import torch

    def one():
        for dst, src in h2d:
            dst.copy_(src, non_blocking=True)
        step_fn()
        for dst, src in d2h:
            dst.copy_(src, non_blocking=True)

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(chunk):
            one()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    n = max(1, reps // chunk)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(n):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / (n * chunk)
    dev = e0.elapsed_time(e1) / (n * chunk)
    del g
    hb = sum(src.numel() * src.element_size() for _, src in h2d)
    db = sum(dst.numel() * dst.element_size() for dst, _ in d2h)
    return max(wall, dev), hb, db


def decode_kernel(B: int) -> str:
    """The decode kernel(s) the planner picks for config 3 at batch B."""
    if B <= 8:
        return "dq_gemv_mma"
    if B <= 16:
        return "dq_gemv_n (4096 x 4096), dq_gemv_mma (11008-column and 11008-row shapes)"
    if B <= 64:
        return "dq_gemv_n"
    return "dq_gemm_tc"


def decode_config3(b2, layers, device, stream, B, cpu):
    """BASELINE config 3 at batch B (8, 32, 64): the same seven int4
    projections, grouping and weight copies as the headline, activations
    [B, 4096].  The planner picks the decode kernel by batch (decode_kernel);
    above 16 rows a group runs one call per member."""
    import torch
    from onnx_light_b200 import synth
    mm = b2.DequantizeMatMul()
    gm = b2.DequantizeMatMulGroup()
    x = synth.convert(synth.randn(2000 + B, (B * 4096,), 0.0, 1.0, device=device), FLOAT16, (B, 4096))
    acts = {"x": x}
    for name, K, N, _ in PROJ:
        acts[name] = torch.empty((B, N), dtype=torch.float16, device=device)
    state = {"i": 0}

    def step():
        layer = layers[state["i"] % NCOPIES]
        state["i"] += 1
        for names, src in GROUPS:
            if len(names) == 1:
                w, sc = layer[names[0]]
                mm(acts[src], w, sc, None, axis=0, out=acts[names[0]])
            else:
                gm(acts[src], [layer[n][0] for n in names], [layer[n][1] for n in names],
                   axis=0, outs=[acts[n] for n in names])

    with torch.cuda.stream(stream):
        for _ in range(NCOPIES):
            step()
    torch.cuda.synchronize()
    ms = _graph_time(stream, step, 256, chunk=NCOPIES * 8)
    nbytes = step_bytes(B)
    gbs = nbytes / (ms * 1e-3) / 1e9
    peak, src = measured_peak()
    x_host = _pinned_like(x)
    x_host.copy_(x)
    y_host = _pinned_like(acts["down"])
    e2e_ms, hb, db = _e2e(stream, step, [(acts["x"], x_host)], [(y_host, acts["down"])], 256,
                          NCOPIES * 8)
    out = {"metric": f"int4 dequant-MatMul HBM GB/s (config 3, batch {B})", "value": round(gbs, 1),
           "unit": "GB/s", "ms_per_step": round(ms, 5),
           "kernel": decode_kernel(B),
           "tflops": round(step_flops(B) / (ms * 1e-3) / 1e12, 2),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "peak_source": src,
                        "algorithmic_bytes_per_step": nbytes},
           "e2e": {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                   "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": hb,
                   "d2h_bytes_per_step": db,
                   "path": "DequantizeMatMulGroup / DequantizeMatMul python API, pinned H2D + "
                           "4 calls + D2H per step"}}
    if cpu:
        out["cpu_baseline"] = cpu_baseline_sample(B)
    return out


def dq_matmul_config1(b2, synth, device, stream, cpu):
    """fp32 activations [1, 32, 4096] times an int4 weight
    [4096, 4096] dequantized with int4 zero points and fp32 scales blocked by
    32 along K; fp32 output.  The fp32 accumulation contract (rel-L2 1e-5)
    keeps it on the FP32 pipe: 1.07 GFLOP against 11.8 MB, so the roofline is
    the slower of the HBM and FP32 times (FP32: 148 SMs x 128 lanes x 2 FLOP x
    the SM clock)."""
    import torch
    K, N, M, bs = 4096, 4096, 32, 32
    w = synth.packed_randint(1001, (K, N), -8, 7, INT4, device=device)
    zp = synth.packed_randint(1003, (K // bs, N), -2, 2, INT4, device=device)
    sc = synth.uniform(1002, (K // bs, N), 0.005, 0.02, device=device)
    a = synth.randn(1004, (1, M, K), 0.0, 1.0, device=device)
    y = torch.empty((1, M, N), dtype=torch.float32, device=device)
    mm = b2.DequantizeMatMul()

    def step():
        mm(a, w, sc, zp, axis=0, out=y)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    ms = _graph_time(stream, step, 512, chunk=32)
    nbytes = K * N // 2 + (K // bs) * N * 4 + (K // bs) * N // 2 + M * K * 4 + M * N * 4
    flops = 2 * M * K * N
    hbm, hsrc = measured_peak()
    fp32_tf = 148 * 128 * 2 * 1.965e9 / 1e12
    t_hbm = nbytes / (hbm * 1e9)
    t_fp32 = flops / (fp32_tf * 1e12)
    bound = "fp32" if t_fp32 > t_hbm else "hbm"
    t_roof = max(t_hbm, t_fp32)
    a_host, y_host = _pinned_like(a), _pinned_like(y)
    a_host.copy_(a)
    e2e_ms, hb, db = _e2e(stream, step, [(a, a_host)], [(y_host, y)], 512, 32)
    out = {"metric": "DequantizeLinear int4 -> MatMul fp32 (config 1)",
           "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
           "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms_per_call": round(ms, 5),
           "dtype": "int4 weights, fp32 activations and accumulation",
           "config": {"M": M, "K": K, "N": N, "block_size": bs, "zero_points": "int4",
                      "scales": "fp32"},
           "roofline": {"bound": bound, "achieved": round(flops / (ms * 1e-3) / 1e12, 3),
                        "peak": round(fp32_tf, 1), "unit": "TFLOP/s",
                        "frac": round(t_roof / (ms * 1e-3), 4),
                        "peak_source": "FP32 pipe at the max SM clock (148 x 128 x 2 x 1.965 GHz); "
                                       f"HBM {hbm} GB/s ({hsrc}) gives {t_hbm * 1e6:.2f} us",
                        "algorithmic_bytes": nbytes, "flops": flops,
                        "roofline_us": round(t_roof * 1e6, 2)},
           "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                   "ms_per_call": round(e2e_ms, 5), "h2d_bytes_per_step": hb,
                   "d2h_bytes_per_step": db}}
    if cpu:
        out["cpu_baseline"] = _cpu_config1_sample()
    return out


def dequantize_standalone(b2, synth, device, stream, cpu):
    """Standalone DequantizeLinear (bit-exact with the reference) on the
    config-1 weight (int4 [4096, 4096], int4 zero points, fp32 scales blocked
    by 32 -> fp32) and the config-5 weight (float8e4m3fn [4096, 11008], fp32
    scales blocked by 32 -> fp32).  HBM-bound: bytes = packed x + scales + zero
    points + y."""
    import torch
    dq = b2.DequantizeLinear()
    out = {"metric": "DequantizeLinear HBM GB/s", "unit": "GB/s", "cases": {}}
    peak, src = measured_peak()
    K, N = 4096, 4096
    w = synth.packed_randint(1001, (K, N), -8, 7, INT4, device=device)
    zp = synth.packed_randint(1003, (K // 32, N), -2, 2, INT4, device=device)
    sc = synth.uniform(1002, (K // 32, N), 0.005, 0.02, device=device)
    y1 = torch.empty((K, N), dtype=torch.float32, device=device)
    K5, N5 = 4096, 11008
    w5 = synth.convert(synth.randn(5010, (K5 * N5,), 0.0, 1.0, device=device), 17, (K5, N5))
    s5 = synth.uniform(5020, (K5 // 32, N5), 0.01, 0.05, device=device)
    y5 = torch.empty((K5, N5), dtype=torch.float32, device=device)
    cases = [("config1_int4_zp_block32", lambda: dq(w, sc, zp, axis=0, out=y1),
              K * N // 2 + (K // 32) * N * 4 + (K // 32) * N // 2 + K * N * 4, y1, w.data),
             ("config5_float8e4m3fn_block32", lambda: dq(w5, s5, None, axis=0, out=y5),
              K5 * N5 + (K5 // 32) * N5 * 4 + K5 * N5 * 4, y5, w5.data)]
    for name, fn, nbytes, y, xin in cases:
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        ms = _graph_time(stream, fn, 256, chunk=16)
        gbs = nbytes / (ms * 1e-3) / 1e9
        x_host, y_host = _pinned_like(xin), _pinned_like(y)
        x_host.copy_(xin)
        e2e_ms, hb, db = _e2e(stream, fn, [(xin, x_host)], [(y_host, y)], 32, 8)
        out["cases"][name] = {
            "value": round(gbs, 1), "ms_per_call": round(ms, 5),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": src,
                         "algorithmic_bytes": nbytes},
            "e2e": {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_call": round(e2e_ms, 4), "h2d_bytes_per_step": hb,
                    "d2h_bytes_per_step": db}}
    out["value"] = out["cases"]["config1_int4_zp_block32"]["value"]
    if cpu:
        out["cpu_baseline"] = _cpu_dq_sample()
    del w5, s5, y5
    torch.cuda.empty_cache()
    return out


def decoder_ops(b2, synth, device, stream, cpu):
    """The decoder-layer operators around the projections at the config-5
    prefill shapes (bf16, B = 4, S = 8192, hidden 4096, 32 heads of 128,
    intermediate 11008): RMSNormalization of the hidden state, RotaryEmbedding
    of the queries (rank 3, cos/sin rows by position_ids) and SwiGLU of the
    gate / up outputs.  All HBM-bound: bytes = inputs + outputs (every tensor
    far above L2)."""
    import torch
    B, S, H, Dh, F = 4, 8192, 4096, 128, 11008
    peak, src = measured_peak()
    x = synth.convert(synth.randn(6001, (B * S * H,), 0.0, 1.0, device=device), BF16, (B, S, H))
    sc = synth.convert(synth.uniform(6002, (H,), 0.5, 1.5, device=device), BF16, (H,))
    y = torch.empty_like(x)
    cos = synth.convert(synth.uniform(6003, (S * Dh // 2,), -1.0, 1.0, device=device), BF16,
                        (S, Dh // 2))
    sin = synth.convert(synth.uniform(6004, (S * Dh // 2,), -1.0, 1.0, device=device), BF16,
                        (S, Dh // 2))
    pos = torch.arange(S, dtype=torch.int64, device=device).repeat(B, 1)
    ga = synth.convert(synth.randn(6005, (B * S * F,), 0.0, 1.0, device=device), BF16, (B * S, F))
    ub = synth.convert(synth.randn(6006, (B * S * F,), 0.0, 1.0, device=device), BF16, (B * S, F))
    gy = torch.empty_like(ga)
    rms, rot, swi = b2.RMSNormalization(), b2.RotaryEmbedding(), b2.SwiGLU()
    xb = x.numel() * 2
    cases = [
        ("rms_normalization", lambda: rms(x, sc, axis=-1, epsilon=1e-5, out=y),
         2 * xb + H * 2, [x], y),
        ("rotary_embedding", lambda: rot(x, cos, sin, pos, num_heads=H // Dh, out=y),
         2 * xb + 2 * cos.numel() * 2 + pos.numel() * 8, [x], y),
        ("swiglu", lambda: swi(ga, ub, 1.0, out=gy), 3 * ga.numel() * 2, [ga, ub], gy),
    ]
    out = {"metric": "decoder-layer ops HBM GB/s (config-5 shapes, bf16)", "unit": "GB/s",
           "cases": {}}
    for name, fn, nbytes, ins, yy in cases:
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        ms = _graph_time(stream, fn, 32, chunk=8)
        gbs = nbytes / (ms * 1e-3) / 1e9
        hosts = [(t, _pinned_like(t)) for t in ins]
        for t, h in hosts:
            h.copy_(t)
        y_host = _pinned_like(yy)
        e2e_ms, hb, db = _e2e(stream, fn, hosts, [(y_host, yy)], 4, 2)
        out["cases"][name] = {
            "value": round(gbs, 1), "ms_per_call": round(ms, 4),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": src,
                         "algorithmic_bytes": nbytes},
            "e2e": {"value": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_call": round(e2e_ms, 3), "h2d_bytes_per_step": hb,
                    "d2h_bytes_per_step": db}}
        del hosts, y_host
    out["value"] = out["cases"]["rms_normalization"]["value"]
    if cpu:
        out["cpu_baseline"] = _cpu_decoder_sample()
    del x, y, ga, ub, gy
    torch.cuda.empty_cache()
    return out


def _graph_time(stream, fn, reps, chunk=64):
    """Device ms per call of fn(), replayed as CUDA graphs of `chunk` calls."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(chunk):
            fn()
    with torch.cuda.stream(stream):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        n = max(1, reps // chunk)
        for _ in range(n):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / (n * chunk)


def attention_config4(b2, synth, device, stream, cpu):
    """GQA decode, fp16, batch 32, 32 query / 8 KV heads,
    head 128, past 4096, causal, scale 1/sqrt(128); the new token is appended in
    place into a capacity-reserved cache.  Every step reads the whole cache
    (537 MB > L2).  Metric: tokens/s (batch rows per step / step time)."""
    import math
    import torch
    B, Hq, Hkv, D, past = 32, 32, 8, 128, 4096
    cache = b2.KVCache(B, Hkv, past + 1, D, device=device)
    n = B * Hkv * (past + 1) * D
    cache.k.view(-1).copy_(synth.convert(synth.randn(4001, (n,), 0.0, 0.5, device=device), FLOAT16, (n,)))
    cache.v.view(-1).copy_(synth.convert(synth.randn(4002, (n,), 0.0, 0.5, device=device), FLOAT16, (n,)))
    q = synth.convert(synth.randn(4003, (B * Hq * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hq, 1, D))
    k = synth.convert(synth.randn(4004, (B * Hkv * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, 1, D))
    v = synth.convert(synth.randn(4005, (B * Hkv * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, 1, D))
    y = torch.empty((B, Hq, 1, D), dtype=torch.float16, device=device)
    att = b2.Attention()
    attrs = b2.Attributes(has_scale=True, scale=1.0 / math.sqrt(D), is_causal=True)

    def step():
        cache.length = past
        att(q, k, v, attrs, cache=cache, out=y)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    ms = _graph_time(stream, step, 512, chunk=32)
    nbytes = 537657344  # KV read incl. the new token + Q/Y + the append
    peak, src = measured_peak()
    gbs = nbytes / (ms * 1e-3) / 1e9
    hq, hk, hv, hy = _pinned_like(q), _pinned_like(k), _pinned_like(v), _pinned_like(y)
    hq.copy_(q)
    hk.copy_(k)
    hv.copy_(v)
    e2e_ms, hb, db = _e2e(stream, step, [(q, hq), (k, hk), (v, hv)], [(hy, y)], 256, 32)
    out = {"metric": "GQA Attention decode tokens/s/GPU (config 4)",
           "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 5),
           "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                   "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": hb,
                   "d2h_bytes_per_step": db,
                   "path": "Attention python API with the KV cache resident; the new token's "
                           "Q/K/V in, Y out"},
           "dtype": "fp16", "config": {"batch": B, "q_heads": Hq, "kv_heads": Hkv, "head": D,
                                        "past": past, "causal": True},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 4), "peak_source": src,
                        "algorithmic_bytes_per_step": nbytes}}
    if cpu:
        out["cpu_baseline"] = _cpu_attention_sample()
    return out


def attention_config4_sharded(b2, synth, device, stream, peers, world, rank):
    """Config 4 sharded by KV head over `world` GPUs: rank r keeps the cache of
    KV heads [r Hkv/world, (r+1) Hkv/world) and the matching query heads (GQA
    groups never straddle ranks), runs the decode step on them and
    b2_allgather_cols gathers the [B, Hq/world * D] head slices into every
    rank's [B, Hq * D] output.  Fixed total work (strong scaling); tokens/s of
    the whole group, step time max over ranks; the gathered output is checked
    against an unsharded run on rank 0."""
    import math
    import torch
    import torch.distributed as dist
    B, Hq, Hkv, D, past = 32, 32, 8, 128, 4096
    hk, hq = Hkv // world, Hq // world
    n = B * Hkv * (past + 1) * D
    kf = synth.convert(synth.randn(4001, (n,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, past + 1, D))
    vf = synth.convert(synth.randn(4002, (n,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, past + 1, D))
    qf = synth.convert(synth.randn(4003, (B * Hq * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hq, 1, D))
    knf = synth.convert(synth.randn(4004, (B * Hkv * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, 1, D))
    vnf = synth.convert(synth.randn(4005, (B * Hkv * D,), 0.0, 0.5, device=device), FLOAT16, (B, Hkv, 1, D))
    cache = b2.KVCache(B, hk, past + 1, D, device=device)
    cache.k.copy_(kf[:, rank * hk:(rank + 1) * hk])
    cache.v.copy_(vf[:, rank * hk:(rank + 1) * hk])
    q = qf[:, rank * hq:(rank + 1) * hq].contiguous()
    k = knf[:, rank * hk:(rank + 1) * hk].contiguous()
    v = vnf[:, rank * hk:(rank + 1) * hk].contiguous()
    y = torch.empty((B, hq, 1, D), dtype=torch.float16, device=device)
    full = peers.buffer("attention4", (B, Hq * D), torch.float16)
    att = b2.Attention()
    attrs = b2.Attributes(has_scale=True, scale=1.0 / math.sqrt(D), is_causal=True)

    def step():
        cache.length = past
        att(q, k, v, attrs, cache=cache, out=y)
        peers.gather("attention4", y.view(B, hq * D))

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    ms = _graph_time(stream, step, 512, chunk=32)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # check: the gathered heads against one unsharded step (rank 0)
    check = None
    if rank == 0:
        cache_f = b2.KVCache(B, Hkv, past + 1, D, device=device)
        cache_f.k.copy_(kf)
        cache_f.v.copy_(vf)
        cache_f.length = past
        yf = att(qf, knf, vnf, attrs, cache=cache_f).Y
        torch.cuda.synchronize()
        ref = yf.view(B, Hq * D).float()
        check = float(((full.float() - ref).norm() / ref.norm()).item())
        del cache_f, yf
    dist.barrier()
    nbytes = 537657344
    peak, src = measured_peak()
    gbs = nbytes / (ms * 1e-3) / 1e9
    del kf, vf, cache
    torch.cuda.empty_cache()
    return {"metric": "GQA Attention decode tokens/s (config 4, sharded by KV head)",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
            "ms_per_step": round(ms, 5), "scaling": "strong",
            "config": {"batch": B, "q_heads": Hq, "kv_heads": Hkv, "head": D, "past": past,
                       "kv_heads_per_gpu": hk},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1),
                         "peak": round(peak * world, 1), "unit": "GB/s",
                         "frac": round(gbs / (peak * world), 4),
                         "peak_source": f"{world} x {src}"},
            "gather_check_rel_l2": check}


def matmul_integer_config2(b2, synth, device, stream, cpu):
    """MatMulInteger uint8 A [512, 4096] (zero point 128) x
    int8 B [4096, 11008] (per-column zero points in [-4, 4]) -> int32."""
    import torch
    M, K, N = 512, 4096, 11008
    a = synth.randint(2001, (M * K,), 0, 255, device=device).to(torch.uint8).view(M, K)
    bq = synth.randint(2002, (K * N,), -127, 127, device=device).to(torch.int8).view(K, N)
    azp = torch.tensor(128, dtype=torch.uint8, device=device)
    bzp = synth.randint(2003, (N,), -4, 4, device=device).to(torch.int8)
    y = torch.empty((M, N), dtype=torch.int32, device=device)
    mmi = b2.MatMulInteger()

    def step():
        mmi(a, bq, azp, bzp, out=y)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    ms = _graph_time(stream, step, 256, chunk=16)
    ops = 2 * M * K * N
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = 2.0 * float(json.load(f)["bf16_tflops"])
        src = "2 x measured bf16 (MEASURED_PEAKS.json; dense int8 is twice bf16)"
    except (OSError, KeyError, ValueError):
        peak, src = 4500.0, "nominal 4.5 POPS dense int8"
    tops = ops / (ms * 1e-3) / 1e12
    ha, hy = _pinned_like(a), _pinned_like(y)
    ha.copy_(a)
    e2e_ms, hb, db = _e2e(stream, step, [(a, ha)], [(hy, y)], 64, 8)
    out = {"metric": "MatMulInteger TOP/s (config 2)", "value": round(tops, 2), "unit": "TOP/s",
           "e2e": {"value": round(ops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TOP/s",
                   "ms_per_call": round(e2e_ms, 4), "h2d_bytes_per_step": hb,
                   "d2h_bytes_per_step": db,
                   "path": "MatMulInteger python API, B resident (an initializer), A in, Y out"},
           "ms_per_call": round(ms, 4), "dtype": "u8 x s8 -> s32",
           "config": {"M": M, "K": K, "N": N, "a_zero_point": "scalar 128",
                      "b_zero_point": "per column"},
           "roofline": {"bound": "tensor", "achieved": round(tops, 2), "peak": peak,
                        "unit": "TOP/s", "frac": round(tops / peak, 4), "peak_source": src}}
    if cpu:
        out["cpu_baseline"] = _cpu_mmi_sample()
    return out


def prefill_config5(b2, synth, device, stream, cpu):
    """BASELINE config 5 on one GPU: bf16 activations [4, 8192, 4096] through
    causal GQA Attention (32 query / 8 KV heads, head 128; K and V [4, 8192,
    1024]) and then the blocked-dequant MatMuls 4096x11008 and 11008x4096, once
    with float8e4m3fn weights and once with float4e2m1 weights (block 32 along
    K, fp32 scales).  Metric: TFLOP/s of the step (attention counted with the
    causal half, 2*M*K*N per MatMul)."""
    import torch
    B, S, Hq, Hkv, D = 4, 8192, 32, 8, 128
    M, K1, N1 = B * S, 4096, 11008
    x = synth.convert(synth.randn(5001, (B * S * Hq * D,), 0.0, 0.5, device=device), BF16,
                      (B, S, Hq * D))
    kk = synth.convert(synth.randn(5002, (B * S * Hkv * D,), 0.0, 0.5, device=device), BF16,
                       (B, S, Hkv * D))
    vv = synth.convert(synth.randn(5003, (B * S * Hkv * D,), 0.0, 0.5, device=device), BF16,
                       (B, S, Hkv * D))
    att = b2.Attention()
    attrs = b2.Attributes(is_causal=True, q_num_heads=Hq, kv_num_heads=Hkv)
    ao = torch.empty_like(x)
    h = torch.empty((M, N1), dtype=torch.bfloat16, device=device)
    y = torch.empty((M, K1), dtype=torch.bfloat16, device=device)
    mm = b2.DequantizeMatMul()
    att_flops = 4 * B * Hq * S * S * D // 2
    mm_flops = 2 * M * K1 * N1
    peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops_sustained"])
        src = "measured sustained bf16 (MEASURED_PEAKS.json; the block runs about 10 ms)"
    except (OSError, KeyError, ValueError):
        peak, src = 1408.4, "fallback sustained bf16"

    def ev_time(fn, reps=3):
        with torch.cuda.stream(stream):
            fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    a2 = ao.view(M, K1)
    t_att = ev_time(lambda: att(x, kk, vv, attrs, out=ao))
    out = {"metric": "Prefill block TFLOP/s (config 5: Attention + 2 dequant-MatMuls)",
           "unit": "TFLOP/s", "dtype": "bf16 activations",
           "config": {"batch": B, "seq": S, "q_heads": Hq, "kv_heads": Hkv, "head": D,
                      "causal": True, "matmuls": "4096x11008, 11008x4096", "block_size": 32,
                      "scales": "fp32"},
           "attention_ms": round(t_att, 3),
           "attention_tflops": round(att_flops / (t_att * 1e-3) / 1e12, 1), "formats": {}}
    for name, dt, lo, hi in (("float8e4m3fn", 17, 0.01, 0.05), ("float4e2m1", 23, 0.05, 0.2)):
        if dt == 17:
            w1 = synth.convert(synth.randn(5010, (K1 * N1,), 0.0, 1.0, device=device), dt, (K1, N1))
            w2 = synth.convert(synth.randn(5011, (N1 * K1,), 0.0, 1.0, device=device), dt, (N1, K1))
        else:
            w1 = synth.convert(synth.randint(5010, (K1 * N1,), 0, 15, device=device), dt, (K1, N1))
            w2 = synth.convert(synth.randint(5011, (N1 * K1,), 0, 15, device=device), dt, (N1, K1))
        s1 = synth.uniform(5020, (K1 // 32, N1), lo, hi, device=device)
        s2 = synth.uniform(5021, (N1 // 32, K1), lo, hi, device=device)
        t1 = ev_time(lambda: mm(a2, w1, s1, None, axis=0, cast_dtype=torch.bfloat16, out=h))
        t2 = ev_time(lambda: mm(h, w2, s2, None, axis=0, cast_dtype=torch.bfloat16, out=y))
        step = t_att + t1 + t2
        tf = (att_flops + 2 * mm_flops) / (step * 1e-3) / 1e12
        out["formats"][name] = {
            "value": round(tf, 1), "ms_per_step": round(step, 3),
            "matmul_ms": [round(t1, 3), round(t2, 3)],
            "matmul_tflops": [round(mm_flops / (t1 * 1e-3) / 1e12, 1),
                              round(mm_flops / (t2 * 1e-3) / 1e12, 1)],
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(tf / peak, 4), "peak_source": src}}
        del w1, w2, s1, s2
    out["value"] = out["formats"]["float8e4m3fn"]["value"]
    # e2e (float8e4m3fn weights resident as initializers): X, K, V in from
    # pinned host memory, the block, the block's output back to the host.
    w1 = synth.convert(synth.randn(5010, (K1 * N1,), 0.0, 1.0, device=device), 17, (K1, N1))
    w2 = synth.convert(synth.randn(5011, (N1 * K1,), 0.0, 1.0, device=device), 17, (N1, K1))
    s1 = synth.uniform(5020, (K1 // 32, N1), 0.01, 0.05, device=device)
    s2 = synth.uniform(5021, (N1 // 32, K1), 0.01, 0.05, device=device)

    def block():
        att(x, kk, vv, attrs, out=ao)
        mm(a2, w1, s1, None, axis=0, cast_dtype=torch.bfloat16, out=h)
        mm(h, w2, s2, None, axis=0, cast_dtype=torch.bfloat16, out=y)

    hx, hk, hv, hy = _pinned_like(x), _pinned_like(kk), _pinned_like(vv), _pinned_like(y)
    hx.copy_(x)
    hk.copy_(kk)
    hv.copy_(vv)
    with torch.cuda.stream(stream):
        block()
    torch.cuda.synchronize()
    e2e_ms, hb, db = _e2e(stream, block, [(x, hx), (kk, hk), (vv, hv)], [(hy, y)], 3, 1)
    out["e2e"] = {"value": round((att_flops + 2 * mm_flops) / (e2e_ms * 1e-3) / 1e12, 1),
                  "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": hb,
                  "d2h_bytes_per_step": db, "weights": "float8e4m3fn, resident"}
    del w1, w2, s1, s2, hx, hk, hv, hy
    if cpu:
        out["cpu_baseline"] = _cpu_prefill_sample()
    del x, kk, vv, ao, h, y
    torch.cuda.empty_cache()
    return out


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def traffic_from_profile(batch: int):
    """DRAM bytes of one decode step measured by ncu (profiles/traffic.json, batch 1);
    weights and scales are over 99.9 % of them, so other batches add their activation bytes."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)["dq_gemv_mma"]
        return int(t["bytes_per_step"]) + (batch - 1) * (step_bytes(batch) - step_bytes(batch - 1))
    except (OSError, ValueError, KeyError):
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


def _cpu_attention_sample():
    """Reference Attention (oracle/_ref) for config 4 at batch 1, scaled x32."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if not O.ref_available():
            return None
        Hq, Hkv, D, past = 32, 8, 128, 4096
        h = lambda seed, shape: O.f32_to_f16_bits(O.randn(seed, shape, 0.0, 0.5))
        q, k, v = h(1, (1, Hq, 1, D)), h(2, (1, Hkv, 1, D)), h(3, (1, Hkv, 1, D))
        pk, pv = h(4, (1, Hkv, past, D)), h(5, (1, Hkv, past, D))
        run = lambda: O.ref_attention(q, k, v, O.FLOAT16, scale=D ** -0.5, is_causal=True,
                                      past_k=pk, past_v=pv)
        run()
        t0 = time.perf_counter()
        run()
        t = (time.perf_counter() - t0) * 32
        return {"value": round(32 / t, 2), "unit": "tokens/s", "cores": O.ref_thread_count(),
                "kind": "reference",
                "sample": f"batch 1 of config 4 ({t / 32 * 1e3:.1f} ms), scaled x32 to batch 32"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


def _cpu_prefill_sample():
    """Reference Attention (oracle/_ref) on [1, 512, 4096] bf16 scaled by the
    FLOP ratio to [4, 8192, 4096], plus the reference DequantizeLinear
    (float8e4m3fn, block 32) and MatMul of 32 rows scaled to 32768 rows."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import numpy as np
        import oracle as O
        if not O.ref_available():
            return None
        S, Hq, Hkv, D = 512, 32, 8, 128
        b16 = lambda seed, shape: O.f32_to_bf16_bits(O.randn(seed, shape, 0.0, 0.5))
        q, k, v = b16(1, (1, S, Hq * D)), b16(2, (1, S, Hkv * D)), b16(3, (1, S, Hkv * D))
        t0 = time.perf_counter()
        O.ref_attention(q, k, v, O.BFLOAT16, is_causal=True, q_num_heads=Hq, kv_num_heads=Hkv)
        t_att = (time.perf_counter() - t0) * (4 * (8192 / S) ** 2)
        K, N, m = 4096, 11008, 32
        w = O.f32_to_f8e4m3fn(O.randn(4, (K, N), 0.0, 1.0))
        sc = O.rand_uniform(5, (K // 32, N), 0.01, 0.05).astype(np.float32)
        a = O.randn(6, (m, K), 0.0, 0.5).astype(np.float32)
        t0 = time.perf_counter()
        wd = O.ref_dequantize_linear(w, 17, (K, N), sc, O.FLOAT, (K // 32, N), axis=0)
        t_dq = time.perf_counter() - t0
        t0 = time.perf_counter()
        h = O.ref_matmul(a, wd, O.FLOAT)
        t_mm = (time.perf_counter() - t0) * (4 * 8192 / m)
        w2 = O.f32_to_f8e4m3fn(O.randn(7, (N, K), 0.0, 1.0))
        sc2 = O.rand_uniform(8, (N // 32, K), 0.01, 0.05).astype(np.float32)
        t0 = time.perf_counter()
        wd2 = O.ref_dequantize_linear(w2, 17, (N, K), sc2, O.FLOAT, (N // 32, K), axis=0)
        t_dq2 = time.perf_counter() - t0
        t0 = time.perf_counter()
        O.ref_matmul(h, wd2, O.FLOAT)
        t_mm2 = (time.perf_counter() - t0) * (4 * 8192 / m)
        step = t_att + t_dq + t_mm + t_dq2 + t_mm2
        flops = 4 * 4 * Hq * 8192 * 8192 * D // 2 + 2 * 2 * 4 * 8192 * K * N
        return {"value": round(flops / step / 1e12, 6), "unit": "TFLOP/s",
                "cores": O.ref_thread_count(), "kind": "reference",
                "sample": f"Attention [1,{S},4096] bf16 ({t_att / (4 * (8192 / S) ** 2):.2f} s, "
                          f"scaled by FLOPs) + DequantizeLinear fp8 4096x11008 "
                          f"({t_dq:.2f} s) + fp32 MatMul of {m} rows (scaled to 32768), then "
                          f"DequantizeLinear fp8 11008x4096 ({t_dq2:.2f} s) + MatMul of the "
                          f"same {m} rows (scaled)"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


def _cpu_config1_sample():
    """Reference DequantizeLinear (int4, zp, block 32) + fp32 MatMul of config 1."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import numpy as np
        import oracle as O
        if not O.ref_available():
            return None
        K, N, M, bs = 4096, 4096, 32, 32
        w = O.pack_bits(O.randint(1, (K * N,), -8, 7), 4)
        z = O.pack_bits(O.randint(2, (K // bs * N,), -2, 2), 4)
        sc = O.rand_uniform(3, (K // bs, N), 0.005, 0.02).astype(np.float32)
        a = O.randn(4, (M, K)).astype(np.float32)
        run = lambda: O.ref_matmul(a, O.ref_dequantize_linear(w, O.INT4, (K, N), sc, O.FLOAT,
                                                               (K // bs, N), z, (K // bs, N), 0),
                                   O.FLOAT)
        run()
        t0 = time.perf_counter()
        run()
        t = time.perf_counter() - t0
        return {"value": round(2 * M * K * N / t / 1e12, 6), "unit": "TFLOP/s",
                "cores": O.ref_thread_count(), "kind": "reference",
                "sample": f"the whole config-1 chain (DequantizeLinear + MatMul), {t * 1e3:.1f} ms"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


def _cpu_dq_sample():
    """Reference DequantizeLinear on the config-1 weight (int4, zp, block 32 -> fp32)."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import numpy as np
        import oracle as O
        if not O.ref_available():
            return None
        K, N, bs = 4096, 4096, 32
        w = O.pack_bits(O.randint(1, (K * N,), -8, 7), 4)
        z = O.pack_bits(O.randint(2, (K // bs * N,), -2, 2), 4)
        sc = O.rand_uniform(3, (K // bs, N), 0.005, 0.02).astype(np.float32)
        O.ref_dequantize_linear(w, O.INT4, (K, N), sc, O.FLOAT, (K // bs, N), z, (K // bs, N), 0)
        t0 = time.perf_counter()
        O.ref_dequantize_linear(w, O.INT4, (K, N), sc, O.FLOAT, (K // bs, N), z, (K // bs, N), 0)
        t = time.perf_counter() - t0
        nbytes = K * N // 2 + (K // bs) * N * 4 + (K // bs) * N // 2 + K * N * 4
        return {"value": round(nbytes / t / 1e9, 4), "unit": "GB/s", "cores": O.ref_thread_count(),
                "kind": "reference",
                "sample": f"config-1 weight, {t * 1e3:.1f} ms per call"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


def _cpu_decoder_sample():
    """Reference RMSNormalization, RotaryEmbedding and SwiGLU (bf16) on 1024 rows
    of the config-5 shapes: bytes moved / time of the three calls."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import numpy as np
        import oracle as O
        if not O.ref_available():
            return None
        R, H, Dh, F, S = 1024, 4096, 128, 11008, 8192
        x = O.f32_to_bf16_bits(O.randn(11, (1, R, H)))
        sc = O.f32_to_bf16_bits(O.rand_uniform(12, (H,), 0.5, 1.5))
        cs = O.f32_to_bf16_bits(O.rand_uniform(13, (S, Dh // 2), -1.0, 1.0))
        sn = O.f32_to_bf16_bits(O.rand_uniform(14, (S, Dh // 2), -1.0, 1.0))
        pos = np.arange(R, dtype=np.int64).reshape(1, R)
        a = O.f32_to_bf16_bits(O.randn(15, (R, F)))
        b = O.f32_to_bf16_bits(O.randn(16, (R, F)))
        t0 = time.perf_counter()
        O.ref_rms_normalization(x, sc, O.BFLOAT16, -1, 1e-5)
        O.ref_rotary_embedding(x, cs, sn, O.BFLOAT16, pos, False, 0, H // Dh)
        O.ref_swiglu(a, b, O.BFLOAT16, 1.0)
        t = time.perf_counter() - t0
        nbytes = 2 * x.nbytes + sc.nbytes + 2 * x.nbytes + 3 * a.nbytes
        return {"value": round(nbytes / t / 1e9, 4), "unit": "GB/s", "cores": O.ref_thread_count(),
                "kind": "reference",
                "sample": f"1024 rows of each op's config-5 shape (bf16), {t * 1e3:.1f} ms for the three"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


def _cpu_mmi_sample():
    """Reference MatMulInteger (single-threaded in onnx-light) on N = 128
    columns of config 2, scaled to N = 11008."""
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import numpy as np
        import oracle as O
        if not O.ref_available():
            return None
        M, K, n = 512, 4096, 128
        a = O.randint(1, (M * K,), 0, 255).astype(np.uint8).reshape(M, K)
        b = O.randint(2, (K * n,), -127, 127).astype(np.int8).reshape(K, n)
        bz = O.randint(3, (n,), -4, 4).astype(np.int8)
        t0 = time.perf_counter()
        O.ref_matmul_integer(a, O.UINT8, b, O.INT8, np.array([128], np.uint8), bz, (), (n,))
        t = (time.perf_counter() - t0) * (11008 / n)
        return {"value": round(2 * M * K * 11008 / t / 1e12, 6), "unit": "TOP/s", "cores": 1,
                "kind": "reference",
                "sample": f"N = 128 of config 2 ({t * n / 11008:.2f} s), scaled x86 to N = 11008; "
                          f"onnx-light's MatMulInteger is single-threaded"}
    except Exception as e:
        return {"value": None, "kind": "error", "sample": repr(e)[:200]}


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
    # Each step is a bounded sample of the layer: one projection (DequantizeLinear
    # + MatMul), q, k, v, o, gate, up, down in turn, restricted to its first
    # `cols` output columns, with `cols` sized from a calibration call so that
    # the W + K steps take about a minute; value = bytes processed / time.
    import numpy as np
    xs = {}
    for name, K, N, src in PROJ:
        xs[name] = O.f32_to_f16_bits(O.randn(2001, (B, K)))

    def col_slice(name, K, N, cols):
        seed = 3000 + [p[0] for p in PROJ].index(name)
        codes = O.randint(seed, (K * N,), -8, 7).reshape(K, N)[:, :cols]
        sc = O.f32_to_f16_bits(O.rand_uniform(seed + 50, (K // BLOCK * N,), 0.002, 0.02))
        sc = sc.reshape(K // BLOCK, N)[:, :cols]
        return O.pack_bits(np.ascontiguousarray(codes), 4), np.ascontiguousarray(sc)

    def run(name, K, w, sc, cols):
        wq = O.ref_dequantize_linear(w, O.INT4, (K, cols), sc, O.FLOAT16, (K // BLOCK, cols),
                                     None, None, 0)
        O.ref_matmul(xs[name], wq, O.FLOAT16)
        return K * cols // 2 + (K // BLOCK) * cols * 2 + B * K * 2 + B * cols * 2

    cal_w, cal_s = col_slice("q", 4096, 4096, 512)
    run("q", 4096, cal_w, cal_s, 512)
    t0 = time.perf_counter()
    run("q", 4096, cal_w, cal_s, 512)
    per_weight = (time.perf_counter() - t0) / (4096 * 512)
    budget = 60.0 / (args.steps + args.warmup)
    slices = []
    for name, K, N, _ in PROJ:
        cols = int(budget / per_weight / K) // 128 * 128
        cols = max(128, min(N, cols))
        slices.append((name, K, cols) + col_slice(name, K, N, cols))

    def proj_step(i):
        name, K, cols, w, sc = slices[i % len(slices)]
        return run(name, K, w, sc, cols)

    for i in range(args.warmup):
        proj_step(i)
    t0 = time.perf_counter()
    tot_b = 0
    for i in range(args.steps):
        tot_b += proj_step(i)
    el = time.perf_counter() - t0
    t = el / args.steps
    value = tot_b / el / 1e9
    col_note = ", ".join(f"{n}:{c}" for n, _, c, _, _ in slices)
    cores = O.ref_thread_count()
    sample = (f"one config-3 projection per step in turn (DequantizeLinear int4 + MatMul fp16, "
              f"B={B}) over its first columns ({col_note}), onnx-light kernels compiled "
              f"from source, {cores} threads")
    print(json.dumps({
        "impl": "reference",
        "metric": "int4 dequant-MatMul HBM GB/s (Llama-7B decode layer, config 3)",
        "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int4 weights, fp16 activations",
        "data": "synthetic (SplitMix64 seeded)",
        "config": workload_config(B),
        "parallelism": f"{cores} host threads",
        "sample_slice": {"per_step": "one projection, q k v o gate up down in turn",
                         "columns": {n: c for n, _, c, _, _ in slices}},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config-4 attention and config-2 MatMulInteger measurements")
    ap.add_argument("--only", choices=["attention4", "mmi2", "prefill5", "decoder",
                                       "config1", "dequantize"],
                    help="run one secondary measurement alone on cuda:0 (for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        import torch
        b2 = load_package()
        from onnx_light_b200 import synth
        device = torch.device("cuda", 0)
        stream = torch.cuda.Stream(device)
        fn = {"attention4": attention_config4, "mmi2": matmul_integer_config2,
              "prefill5": prefill_config5, "decoder": decoder_ops,
              "config1": dq_matmul_config1, "dequantize": dequantize_standalone}[args.only]
        print(json.dumps(fn(b2, synth, device, stream, False)), flush=True)
        return
    if args.impl == "reference":
        reference_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
