#!/usr/bin/env python
"""Benchmark of the packed-TCQ decode path on B200 (prints ONE JSON line).

Workload (BASELINE metric "TCQ GEMV achieved HBM GB/s; batch-1 decode tok/s,
3-bit Qwen3-4B shape"): one step = one batch-1 decode pass through every
packed linear of a Qwen3-4B-shaped decoder (36 layers x q/k/v/o/gate/up/down,
3-bit packed TCQ, S = 64, per-layer rotation seeds).  The step runs two
ways: as the persistent decode engine (every linear in one cooperative
launch, tp_engine_run) and as per-layer tp_tcq_gemv calls, each captured in
a CUDA graph; the faster is the headline, the other is reported beside it.  Weights are seeded random trellis streams (every bit string is a
valid TCQ codeword) with the reference's data-free trellis codebook; the
1.36 GB of packed weights exceed the 126 MB L2, so every step streams them
from HBM.

  value    = algorithmic bytes of all GEMVs of a step / device time of a step
  e2e      = the same metric through the public module API with the step's
             input copied from pinned host memory and the result read back
  roofline = the headline path's kernels alone, timed with CUDA events
             (the engine launch; or every fused GEMV in an instrumented
             graph replay)
  --impl reference : the reference path's CPU restatement (oracle port) on
             the host cores, on bounded samples of the same workload.

Under torchrun (N > 1) every rank first runs the tensor-parallel engine (each
linear row-sharded over the N GPUs, outputs exchanged over NVLink inside the
kernel) and reports it under "tp"; the line's value then comes from N
replicas, each GPU decoding its own batch-1 stream with the whole model
(scaling "weak"), which is how a 4B model is served on N GPUs.
--parallel tp makes the tensor-parallel step the line itself (the
Llama-3-70B-shaped configuration: --model llama3-70b --bits 2).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
import zlib
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

QWEN3_4B = dict(name="qwen3-4b", label="Qwen3-4B", layers=36, hidden=2560, inter=9728, q_heads=32, kv_heads=8,
                head_dim=128)
# the tensor-parallel configuration (2-bit, TP 1/2/4/8); not the contract line
LLAMA3_70B = dict(name="llama3-70b", label="Llama-3-70B", layers=80, hidden=8192, inter=28672, q_heads=64,
                  kv_heads=8, head_dim=128)
MODELS = {"qwen3-4b": QWEN3_4B, "llama3-70b": LLAMA3_70B}


def metric_name(cfg: dict, bits: int) -> str:
    return f"TCQ GEMV achieved HBM GB/s; batch-1 decode tok/s, {bits}-bit {cfg['label']} shape"
LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


# DRAM bytes (read + write) of one engine launch / algorithmic bytes of the
# step, from the ncu capture summarised under profiles/ (None: not captured)
TRAFFIC_RATIO = 1.025


def linear_shapes(cfg: dict) -> list[tuple[str, int, int]]:
    """(name, in_features d, out_features n) of one decoder layer."""
    h, i, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    return [("q_proj", h, cfg["q_heads"] * hd), ("k_proj", h, cfg["kv_heads"] * hd),
            ("v_proj", h, cfg["kv_heads"] * hd), ("o_proj", cfg["q_heads"] * hd, h),
            ("gate_proj", h, i), ("up_proj", h, i), ("down_proj", i, h)]


def gemv_bytes(n: int, d: int, bits: int, B: int, bias: bool = False) -> int:
    """Algorithmic bytes of one packed GEMV: true-rate path + member bits,
    fp16 scales, codebook, rot_scale, activations in and out (+ bias)."""
    b = n * math.ceil(d / 8) + n * math.ceil(d * (bits - 1) / 8) + 2 * n + 2 * 2 ** (bits + 1) + 2 * d
    b += 2 * B * d + 2 * B * n
    return b + (2 * n if bias else 0)


def layer_seed(seed: int, i: int, name: str) -> int:
    # per-layer rotation seed convention of turbopress/runtime.py:393
    return seed + 7919 * i + zlib.crc32(name.encode()) % 1000


def codebook(bits: int) -> np.ndarray:
    with np.load(ROOT / "tests" / "golden" / "codebooks.npz") as f:
        return f[f"opt_b{bits}_s64"]


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def build_model(cfg: dict, bits: int, device, seed: int = 0):
    import torch

    from turbopress_b200 import PackedTCQLinear

    cb = torch.from_numpy(codebook(bits)).to(device)
    mods = []
    for i in range(cfg["layers"]):
        for name, d, n in linear_shapes(cfg):
            s = layer_seed(seed, i, name)
            g = torch.Generator(device=device).manual_seed(s)
            payload = {
                "format": 2, "n": n, "d": d, "bits": bits, "n_states": 64, "block": d & -d, "seed": s,
                "path_packed": torch.randint(0, 256, (n, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
                "member_packed": torch.randint(0, 256, (n, -(-d * (bits - 1) // 8)), generator=g, dtype=torch.uint8,
                                               device=device) if bits > 1 else None,
                # unit-gain scales keep activations O(1) through the chained step
                "scales": ((torch.rand(n, generator=g, device=device) * 0.5 + 0.75) / math.sqrt(d)).half(),
                "signs_packed": torch.randint(0, 256, (1, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
                "inv_equil": (torch.rand(d, generator=g, device=device) * 0.4 + 0.8).half(),
                "codebook": cb.clone(),
                "bias": None,
            }
            mods.append(PackedTCQLinear(payload, mode="cuda"))
            del payload
    torch.cuda.synchronize()
    return mods


def decode_step(mods, h, layers: int):
    """Chained batch-B decode pass through every packed linear."""
    for i in range(layers):
        q, k, v, o, gate, up, down = mods[7 * i: 7 * i + 7]
        qo = q(h)
        k(h)
        v(h)
        oo = o(qo)
        go = gate(oo)
        up(oo)
        h = down(go)
    return h


def engine_inputs(layers: int) -> list[int | None]:
    """Data flow of decode_step as DecodeEngine inputs (op index of each
    linear's input; None = the step's external input)."""
    inputs: list[int | None] = []
    for i in range(layers):
        b = 7 * i
        prev = None if i == 0 else b - 1          # previous layer's down_proj
        inputs += [prev, prev, prev, b, b + 3, b + 3, b + 4]
    return inputs


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline_sample(cfg: dict, bits: int, which: list[int], seed: int = 0) -> tuple[float, int, float]:
    """Time the oracle port (CPU restatement of the reference tiled forward)
    on a sample of the workload's linears.  Returns (GB/s, bytes, seconds)."""
    from oracle import tcq_oracle as O

    shapes = linear_shapes(cfg)
    cb = codebook(bits)
    total_b, total_t = 0, 0.0
    rng = np.random.default_rng(seed)
    for idx in which:
        name, d, n = shapes[idx % len(shapes)]
        p = O.random_payload(n, d, bits, 64, seed=layer_seed(seed, 0, name), codebook=cb)
        x = rng.standard_normal((1, d)).astype(np.float16)
        t0 = time.perf_counter()
        O.forward_fp32(p, x)
        total_t += time.perf_counter() - t0
        total_b += gemv_bytes(n, d, bits, 1)
    return total_b / total_t / 1e9, total_b, total_t


def peaks_hbm() -> tuple[float, str]:
    pk = ROOT / "MEASURED_PEAKS.json"
    peaks = json.loads(pk.read_text()) if pk.exists() else {}
    if "hbm_gbs" in peaks:
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback 6650 GB/s"


def run_tp(args, cfg, rank, world, local, dev, dist) -> dict | None:
    """Tensor-parallel decode step: every linear split by output rows over the
    ranks, outputs exchanged inside the engine kernel over NVLink peer memory."""
    import torch

    from turbopress_b200.tp import TPDecodeEngine

    bits, B = args.bits, args.batch
    mods = build_model(cfg, bits, dev, seed=args.seed)  # identical on every rank
    step_bytes = sum(gemv_bytes(n, d, bits, B) for _ in range(cfg["layers"]) for _, d, n in linear_shapes(cfg))
    eng = TPDecodeEngine(mods, engine_inputs(cfg["layers"]), batch=B, input_dtype=torch.float16)
    del mods
    torch.cuda.empty_cache()
    stream = torch.cuda.Stream(device=dev)
    x_host = torch.randn(B, cfg["hidden"], dtype=torch.float16).pin_memory()
    y_host = torch.empty(B, cfg["hidden"], dtype=torch.float32).pin_memory()
    xin = eng.x_ext[cfg["hidden"]]

    def barrier():
        dist.barrier()
        torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        xin.copy_(x_host)
        for _ in range(max(args.warmup, 3)):
            eng.launch()
        stream.synchronize()
        eng.check()
        # graphs of two consecutive runs (the arena alternates per run)
        if eng.step % 2:
            eng.launch()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            eng.launch()
            eng.launch()
        graph_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_e2e, stream=stream):
            for k in range(2):
                xin.copy_(x_host, non_blocking=True)
                eng.launch()
                y_host.copy_(eng.outputs_buf[k][-1], non_blocking=True)
        # graph capture advanced the host step count without running: re-sync it
        eng.step = 0
        for _ in range(2):
            graph.replay()
        steps = args.steps + (args.steps % 2)
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            start.record(stream)
            for _ in range(steps // 2):
                graph.replay()
            end.record(stream)
            end.synchronize()
        barrier()
        ms = start.elapsed_time(end) / steps
        kd = []
        for _ in range(4):
            k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            k0.record(stream)
            eng.launch()
            k1.record(stream)
            k1.synchronize()
            kd.append(k0.elapsed_time(k1))
        if eng.step % 2:
            eng.launch()
        stream.synchronize()
        ms_kernel = float(np.median(kd))
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps // 2):
            graph_e2e.replay()
        e1.record(stream)
        e1.synchronize()
        ms_e2e = e0.elapsed_time(e1) / steps
        eng.check()
    t = torch.tensor([ms, ms_e2e, ms_kernel], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_kernel = (float(v) for v in t)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, peak_src = peaks_hbm()
    per_gpu_bytes = step_bytes / world
    ach = per_gpu_bytes / (ms_kernel * 1e-3) / 1e9
    out = {
        "metric": metric_name(cfg, bits),
        "value": round(step_bytes / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": f"u8 packed TCQ ({bits} bits/weight) -> fp16 activations, fp32 accumulate",
        "data": "synthetic: seeded random trellis streams + reference data-free codebook; x N(0,1) fp16",
        "config": {"workload": f"{cfg['name']} decoder linears, batch {B}, {bits}-bit packed TCQ, S=64",
                   "path": f"tensor-parallel persistent engine over {world} GPUs (row-sharded linears, "
                           "outputs added into every rank's arena over NVLink peer memory), CUDA graph",
                   "layers": cfg["layers"], "linears_per_step": cfg["layers"] * len(LINEARS), "batch": B,
                   "bits": bits, "weights_bytes_per_step": int(step_bytes),
                   "l2": "inputs larger than L2 (packed weights per GPU per step > 126 MB L2)",
                   "parallelism": f"tp{world}"},
        "tok_s": round(B * 1000.0 / ms, 1),
        "e2e": {"value": round(step_bytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": "GB/s",
                "tok_s": round(B * 1000.0 / ms_e2e, 1),
                "h2d_bytes_per_step": int(x_host.numel() * 2), "d2h_bytes_per_step": int(y_host.numel() * 4)},
        "gpu_launches": int(steps),
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach / peak, 4),
                     "traffic": round(per_gpu_bytes * TRAFFIC_RATIO) if TRAFFIC_RATIO else None,
                     "kernel": f"tcq_engine_kernel on each of {world} GPUs (its 1/{world} shard of every linear), "
                               "algorithmic bytes per GPU / median CUDA-event duration, max over ranks",
                     "kernel_ms": round(ms_kernel, 4), "peak_source": peak_src},
        "clocks": clk.summary(),
    }
    return out



def run_gpu(args) -> dict | None:
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    cfg, bits, B = dict(MODELS[args.model]), args.bits, args.batch
    if args.layers:
        cfg["layers"] = args.layers  # profiling of a small case only
    tp_line = None
    if world > 1:
        # tensor parallel: one model split over the ranks (latency of one stream)
        tp_line = run_tp(args, cfg, rank, world, local, dev, dist)
        if args.parallel == "tp":
            dist.destroy_process_group()
            return tp_line
        # replicas: every rank decodes its own batch-1 stream with the whole model
    mods = build_model(cfg, bits, dev, seed=args.seed)
    step_bytes = sum(gemv_bytes(n, d, bits, B) for _ in range(cfg["layers"]) for _, d, n in linear_shapes(cfg))
    n_gemv = cfg["layers"] * len(LINEARS)
    launches_per_gemv = 2 * math.ceil(B / 32)  # rotation + fused GEMV per batch chunk of 32

    x_static = torch.randn(B, cfg["hidden"], device=dev, dtype=torch.float16)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(3):
            decode_step(mods, x_static, cfg["layers"])
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            y_static = decode_step(mods, x_static, cfg["layers"])
        # instrumented graph: events around every packed linear
        ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
              for _ in range(n_gemv)]
        gbytes = [gemv_bytes(n, d, bits, B) for _ in range(cfg["layers"]) for _, d, n in linear_shapes(cfg)]
        graph_i = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_i, stream=stream):
            h = x_static
            it = iter(range(n_gemv))
            for i in range(cfg["layers"]):
                outs = []
                for j, m in enumerate(mods[7 * i: 7 * i + 7]):
                    inp = h if j in (0, 1, 2) else outs[3] if j in (4, 5) else outs[0] if j == 3 else outs[4]
                    k = next(it)
                    ev[k][0].record(stream)
                    outs.append(m(inp))
                    ev[k][1].record(stream)
                h = outs[6]
    torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
            end.synchronize()
        barrier()
        ms = start.elapsed_time(end) / args.steps

        # per-launch durations of the fused GEMV (instrumented replay)
        for _ in range(2):
            graph_i.replay()
        stream.synchronize()
        durs = np.array([a.elapsed_time(b) for a, b in ev])  # ms
        ach_gbs = float(np.sum(gbytes) / (np.sum(durs) * 1e-3) / 1e9)
        per_shape = {}
        for k, (name, d, n) in enumerate(linear_shapes(cfg)):
            sel = durs[k::7]
            per_shape[name] = {"us": round(float(np.mean(sel)) * 1e3, 2),
                               "gbs": round(gemv_bytes(n, d, bits, B) / (float(np.mean(sel)) * 1e-3) / 1e9, 1)}

        # end to end: pinned host input -> device, step, result -> pinned host
        x_host = torch.randn(B, cfg["hidden"], dtype=torch.float16).pin_memory()
        y_host = torch.empty(B, cfg["hidden"], dtype=torch.float16).pin_memory()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            x_static.copy_(x_host, non_blocking=True)
            graph.replay()
            y_host.copy_(y_static, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        ms_e2e = e0.elapsed_time(e1) / args.steps

    # persistent engine: the same step as ONE cooperative launch
    eng = None
    if B <= 4 and not args.no_engine:
        from turbopress_b200.engine import DecodeEngine
        eng = DecodeEngine(mods, engine_inputs(cfg["layers"]), batch=B, input_dtype=torch.float16)
        with torch.cuda.stream(stream):
            eng.set_input(x_static)
            eng.run()
            stream.synchronize()
            eng.check()
            graph_e = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph_e, stream=stream):
                eng.run()
            for _ in range(max(args.warmup, 3)):
                graph_e.replay()
            barrier()
            with ClockSampler(local) as clk_e:
                es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                es.record(stream)
                for _ in range(args.steps):
                    graph_e.replay()
                ee.record(stream)
                ee.synchronize()
            barrier()
            ms_eng = es.elapsed_time(ee) / args.steps
            # the engine kernel alone (outputs zeroed outside the events)
            kd = []
            for _ in range(3):
                eng.y_arena.zero_()
                eng.counters.zero_()
                k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                k0.record(stream)
                eng.launch()
                k1.record(stream)
                k1.synchronize()
                kd.append(k0.elapsed_time(k1))
            eng.check()
            ms_kernel = float(np.median(kd))
            # end to end through the engine: pinned host in, graph, fp32 result out
            y32_host = torch.empty(B, cfg["hidden"], dtype=torch.float32).pin_memory()
            xin = eng.x_ext[cfg["hidden"]]
            barrier()
            e0.record(stream)
            for _ in range(args.steps):
                xin.copy_(x_host, non_blocking=True)
                graph_e.replay()
                y32_host.copy_(eng.outputs[-1], non_blocking=True)
            e1.record(stream)
            e1.synchronize()
            ms_eng_e2e = e0.elapsed_time(e1) / args.steps
    else:
        ms_eng = ms_kernel = ms_eng_e2e = float("inf")

    t = torch.tensor([ms, ms_e2e, ms_eng, ms_eng_e2e, ms_kernel], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_eng, ms_eng_e2e, ms_kernel = (float(v) for v in t)
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return None

    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    use_engine = ms_eng < ms
    ms_head = ms_eng if use_engine else ms
    ms_head_e2e = ms_eng_e2e if use_engine else ms_e2e
    value = world * step_bytes / (ms_head * 1e-3) / 1e9
    graph_line = {"ms_per_step": round(ms, 4), "value": round(world * step_bytes / (ms * 1e-3) / 1e9, 1),
                  "tok_s": round(world * B * 1000.0 / ms, 1),
                  "e2e_tok_s": round(world * B * 1000.0 / ms_e2e, 1),
                  "gemv_achieved_gbs": round(ach_gbs, 1), "per_shape": per_shape,
                  "launches_per_step": n_gemv * launches_per_gemv}
    if use_engine:
        ach = step_bytes / (ms_kernel * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                "frac": round(ach / peak, 4),
                "traffic": round(step_bytes * TRAFFIC_RATIO) if TRAFFIC_RATIO else None,
                "kernel": "tcq_engine_kernel (one cooperative launch per step, all 252 GEMVs), "
                          "algorithmic bytes of the step / median CUDA-event duration of the launch",
                "kernel_ms": round(ms_kernel, 4),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                else "fallback 6650 GB/s"}
        launches = args.steps
        path = "persistent engine (tp_engine_run), CUDA graph"
    else:
        roof = {"bound": "hbm", "achieved": round(ach_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(ach_gbs / peak, 4), "traffic": None,
                "kernel": "tp_tcq_gemv (rotation + fused decode-GEMV launches), mean over the step's 252 GEMVs",
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)" if peak_src == "measured"
                else "fallback 6650 GB/s", "per_shape": per_shape}
        launches = args.steps * n_gemv * launches_per_gemv
        path = "per-layer tp_tcq_gemv calls, CUDA graph"
    out = {
        "metric": metric_name(cfg, bits),
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_head, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"u8 packed TCQ ({bits} bits/weight) -> fp16 activations, fp32 accumulate",
        "data": "synthetic: seeded random trellis streams + reference data-free codebook; x N(0,1) fp16",
        "config": {"workload": f"{cfg['name']} decoder linears, batch {B}, {bits}-bit packed TCQ, S=64",
                   "path": path,
                   "layers": cfg["layers"], "linears_per_step": n_gemv, "batch": B, "bits": bits,
                   "weights_bytes_per_step": int(step_bytes),
                   "l2": "inputs larger than L2 (packed weights per step > 126 MB L2)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "tok_s": round(world * B * 1000.0 / ms_head, 1),
        "e2e": {"value": round(world * step_bytes / (ms_head_e2e * 1e-3) / 1e9, 1), "unit": "GB/s",
                "tok_s": round(world * B * 1000.0 / ms_head_e2e, 1),
                "h2d_bytes_per_step": int(x_host.numel() * 2),
                "d2h_bytes_per_step": int(B * cfg["hidden"] * (4 if use_engine else 2))},
        "gpu_launches": int(launches),
        "roofline": roof,
        "clocks": (clk_e if use_engine else clk).summary(),
        "per_layer_graph": graph_line,
    }
    if ms_eng != float("inf"):
        out["engine"] = {"ms_per_step": round(ms_eng, 4), "kernel_ms": round(ms_kernel, 4),
                         "value": round(world * step_bytes / (ms_eng * 1e-3) / 1e9, 1),
                         "tok_s": round(world * B * 1000.0 / ms_eng, 1),
                         "e2e_tok_s": round(world * B * 1000.0 / ms_eng_e2e, 1)}
    if tp_line is not None:
        out["tp"] = {"parallelism": f"tp{world}", "ms_per_step": tp_line["ms_per_step"], "tok_s": tp_line["tok_s"],
                     "value": tp_line["value"], "unit": "GB/s", "e2e_tok_s": tp_line["e2e"]["tok_s"],
                     "kernel_ms": tp_line["roofline"]["kernel_ms"], "roofline_frac": tp_line["roofline"]["frac"],
                     "path": tp_line["config"]["path"]}
    if not args.no_cpu_baseline and world == 1:
        gbs, nbytes, secs = cpu_baseline_sample(cfg, bits, list(range(7)), seed=args.seed)
        out["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                               "sample": f"oracle forward of one decoder layer (7 linears, {nbytes / 1e6:.1f} MB "
                                         f"packed) in {secs:.1f} s",
                               "tok_s_extrapolated": round(1.0 / (secs * cfg["layers"]), 5)}
    if dist is not None:
        dist.destroy_process_group()
    return out


def random_linear(n: int, d: int, bits: int, device, seed: int, cb=None):
    """One PackedTCQLinear with seeded random trellis streams (GPU-generated)."""
    import torch

    from turbopress_b200 import PackedTCQLinear

    g = torch.Generator(device=device).manual_seed(seed)
    if cb is None:
        cb = torch.from_numpy(codebook(bits)).to(device)
    payload = {
        "format": 2, "n": n, "d": d, "bits": bits, "n_states": 64, "block": d & -d, "seed": seed,
        "path_packed": torch.randint(0, 256, (n, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
        "member_packed": torch.randint(0, 256, (n, -(-d * (bits - 1) // 8)), generator=g, dtype=torch.uint8,
                                       device=device) if bits > 1 else None,
        "scales": ((torch.rand(n, generator=g, device=device) * 0.5 + 0.75) / math.sqrt(d)).half(),
        "signs_packed": torch.randint(0, 256, (1, -(-d // 8)), generator=g, dtype=torch.uint8, device=device),
        "inv_equil": (torch.rand(d, generator=g, device=device) * 0.4 + 0.8).half(),
        "codebook": cb.clone(),
        "bias": None,
    }
    return PackedTCQLinear(payload, mode="cuda")


def run_gemv(args) -> dict:
    """Standalone packed GEMVs (BASELINE config 3 shapes by default): per shape,
    `copies` distinct weight sets in one CUDA graph (so each launch streams its
    weights from HBM), timed with CUDA events; --once runs one call per shape
    (for profiler captures)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = {}
    for shp in args.shapes.split(","):
        n, d = map(int, shp.lower().split("x"))
        copies = 1 if args.once else max(1, min(args.copies, int(2e9 // max(1, n * d * args.bits // 8))))
        mods = [random_linear(n, d, args.bits, dev, seed=c) for c in range(copies)]
        x = torch.randn(args.batch, d, device=dev, dtype=torch.float16)
        if args.once:
            mods[0](x)
            torch.cuda.synchronize()
            continue
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(s):
            for m in mods:
                m(x)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for m in mods:
                    m(x)
            for _ in range(max(args.warmup, 3)):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(args.steps):
                graph.replay()
            e1.record(s)
            e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.steps / copies
        nbytes = gemv_bytes(n, d, args.bits, args.batch)
        res[shp] = {"us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1), "MB": round(nbytes / 1e6, 2),
                    "TFLOPs": round(2 * args.batch * n * d / us / 1e6, 2), "copies": copies}
        del mods, graph
        torch.cuda.empty_cache()
    return {"workload": "gemv", "bits": args.bits, "batch": args.batch, "shapes": res}


def run_lmhead(args) -> dict:
    """Greedy LM head (fp16 vocabulary GEMV + argmax), Qwen3 vocabulary x the
    model's hidden size: GB/s of weight bytes over the kernel's event time."""
    import torch

    from turbopress_b200.lm_head import GreedyLMHead

    cfg = MODELS[args.model]
    V, h, B = 151936, cfg["hidden"], args.batch
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    w = (torch.randn(V, h, generator=g, device=dev) * 0.02).half()  # 0.78 GB at h = 2560: larger than L2
    x = torch.randn(B, h, generator=g, device=dev).half()
    head = GreedyLMHead(w)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            head(x)
        stream.synchronize()
        with ClockSampler(0) as clk:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                tok, _ = head(x)
            b.record(stream)
            b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    nbytes = V * h * 2 + B * h * 2 + B * 12
    peak, peak_src = peaks_hbm()
    ach = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "lmhead", "vocab": V, "hidden": h, "batch": B, "us": round(ms * 1e3, 2),
            "gbs": round(ach, 1), "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                                               "unit": "GB/s", "frac": round(ach / peak, 4),
                                               "peak_source": peak_src},
            "token": tok.cpu().tolist(), "clocks": clk.summary()}


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cfg, bits = dict(MODELS[args.model]), args.bits
    for i in range(args.warmup):
        cpu_baseline_sample(cfg, bits, [i], seed=args.seed)
    vals, tot_b, tot_t = [], 0, 0.0
    for i in range(args.steps):
        gbs, b, t = cpu_baseline_sample(cfg, bits, [i], seed=args.seed)
        vals.append(gbs)
        tot_b += b
        tot_t += t
    value = tot_b / tot_t / 1e9
    ms = tot_t / args.steps * 1e3
    return {
        "impl": "reference",
        "metric": metric_name(cfg, bits),
        "value": round(value, 3), "unit": "GB/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8 packed TCQ -> fp32 (reference CPU path)",
        "data": "synthetic: seeded random trellis streams + reference data-free codebook",
        "config": {"workload": f"{cfg['name']} decoder linears, batch 1, {bits}-bit packed TCQ, S=64",
                   "sample": "one linear per step, cycling q/k/v/o/gate/up/down"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": "oracle port of the reference tiled forward (unpack, window decode, fp16 "
                                   "dequant, fp32 matmul), one linear per step"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--bits", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", choices=sorted(MODELS), default="qwen3-4b",
                    help="decode workload: model shape (qwen3-4b is the contract line)")
    ap.add_argument("--parallel", choices=["replicas", "tp"], default="replicas",
                    help="N > 1: the JSON line's value from N independent batch-1 streams (replicas, with the "
                         "tensor-parallel step reported under 'tp') or from the tensor-parallel step itself")
    ap.add_argument("--layers", type=int, default=0, help="decoder layers (default: the model's 36; "
                    "smaller values are for ncu captures, not bench lines)")
    ap.add_argument("--no-engine", action="store_true", help="decode workload: per-layer graph only")
    ap.add_argument("--workload", choices=["decode", "gemv", "lmhead"], default="decode",
                    help="decode: the contract line (Qwen3-4B decode step); gemv: standalone GEMV table")
    ap.add_argument("--shapes", default="14336x4096,4096x14336,4096x4096,1024x4096",
                    help="gemv workload: comma-separated NxD (out x in) shapes")
    ap.add_argument("--copies", type=int, default=16, help="gemv workload: distinct weight sets per shape")
    ap.add_argument("--once", action="store_true", help="gemv workload: one call per shape (profiling)")
    args = ap.parse_args()
    if args.workload == "lmhead" and args.impl != "reference":
        print(json.dumps(run_lmhead(args)), flush=True)
        return
    if args.workload == "gemv" and args.impl != "reference":
        print(json.dumps(run_gemv(args)), flush=True)
        return
    out = run_reference(args) if args.impl == "reference" else run_gpu(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
