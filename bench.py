#!/usr/bin/env python
"""Benchmark of the packed-TCQ decode path on B200 (prints ONE JSON line).

Metric (BASELINE): "TCQ GEMV achieved HBM GB/s; batch-1 decode tok/s, 3-bit
Qwen3-4B shape".  One step = one greedy batch-1 decode step of a
Qwen3-4B-shaped decoder (36 layers, 3-bit packed TCQ, S = 64, random-init
weights: seeded random trellis streams with the reference's data-free
codebook) against a 1024-token synthetic KV cache: the whole-model step
kernel (tp_step_run: norms, q/k/v, head norms, RoPE, KV append, GQA
attention, o_proj, SiLU MLP, residuals, final norm) plus the greedy fp16 LM
head (151936 x 2560, tp_lm_head_argmax) and the embedding row of the chosen
token, replayed from a CUDA graph token after token.  The 1.37 GB of packed
weights and 0.78 GB LM head exceed the 126 MB L2, so every step streams them
from HBM.

  value    = algorithmic bytes of a step (packed weights + scales / codebooks
             / rotation scales, KV cache read + append, LM head, activations)
             / device time of a step
  tok_s    = batch * steps per second
  e2e      = the same step through the public API (DecodeStep + GreedyLMHead)
             with each step's token ids copied in from pinned host memory
             and the chosen tokens read back
  roofline = the step kernel alone (CUDA events around tp_step_run), its
             algorithmic bytes over its duration, against MEASURED_PEAKS.json
  gemv_c3  = the standalone packed GEMV (Llama-3-8B shapes x
             2/3/4 bits x batch 1/4/16) with an oracle spot check per shape
  c1       = BASELINE config 1 (1024 x 1024, 2-bit): the GPU GEMV and the
             reference's own CPU forward (tiled and cached) on this host
  decode_c4 = BASELINE config 4: mixed 2/3/4-bit Qwen3-4B at batch 1 and 8
  cpu_baseline / --impl reference : the reference's CPU tiled forward
             restated in torch (oracle/torch_cpu.py), all host threads.

Under torchrun (N > 1) every rank decodes its own batch-1 stream with the
whole model (replicas, scaling "weak"); the tensor-parallel engine of the
decoder linears is reported under "tp" (--parallel tp makes it the line).
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
# DRAM bytes (read 185.44 MB + write 4.13 MB) of one step_kernel launch over
# the first 4 layers of the Qwen3-4B 3-bit batch-1 line / its algorithmic
# bytes (169.12 MB); the traffic of every layer is the same, so the ratio
# scales to the full step (ncu --set full on step_kernel, 4-layer bench case)
STEP_TRAFFIC = {("qwen3-4b", 3, 1): (185_441_024 + 4_134_912) / 169_115_520}


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


def cpu_info() -> dict:
    import torch

    model = ""
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "cpu_model": model}


def cpu_layer_sample(cfg: dict, bits: int, which: list[int], seed: int = 0, cached: bool = False,
                     tile_rows: int = 1024) -> tuple[int, float]:
    """Time the reference's CPU forward (torch restatement, oracle/torch_cpu.py;
    tiled, or cached = decode once then F.linear) over linears of one decoder
    layer.  Returns (packed bytes, seconds)."""
    import torch

    from oracle import tcq_oracle as O
    from oracle import torch_cpu as T

    torch.set_num_threads(os.cpu_count() or 1)
    cb = codebook(bits)
    shapes = linear_shapes(cfg)
    tot_b, tot_t = 0, 0.0
    rng = np.random.default_rng(seed)
    for idx in which:
        name, d, n = shapes[idx % len(shapes)]
        p = O.random_payload(n, d, bits, 64, seed=layer_seed(seed, 0, name), codebook=cb)
        x = torch.from_numpy(rng.standard_normal((1, d)).astype(np.float16))
        with torch.no_grad():
            if cached:
                w16 = T.cached_weight(p)
                t0 = time.perf_counter()
                T.cached_forward(w16, x)
            else:
                rs = T.rot_scale(p)
                t0 = time.perf_counter()
                T.tiled_forward(p, x, rs, tile_rows)
        tot_t += time.perf_counter() - t0
        tot_b += gemv_bytes(n, d, bits, 1)
    return tot_b, tot_t

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
    x_host = torch.randn(B, cfg["hidden"], dtype=torch.float16, generator=torch.Generator().manual_seed(5)).pin_memory()
    # parity reference: the same model as a single-GPU engine on this rank
    from turbopress_b200.engine import DecodeEngine

    ref_eng = DecodeEngine(mods, engine_inputs(cfg["layers"]), batch=B, input_dtype=torch.float16)
    ref_out = [o.clone() for o in ref_eng.run(x_host.to(dev))]
    ref_eng.check()
    del ref_eng
    eng = TPDecodeEngine(mods, engine_inputs(cfg["layers"]), batch=B, input_dtype=torch.float16)
    del mods
    torch.cuda.empty_cache()
    stream = torch.cuda.Stream(device=dev)
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
        # every op's full output on this rank against the single-GPU engine
        parity = max(float((o - r).norm() / r.norm().clamp_min(1e-30)) for o, r in zip(eng.outputs, ref_out))
        del ref_out
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
    t = torch.tensor([ms, ms_e2e, ms_kernel, parity], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_kernel, parity = (float(v) for v in t)
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
        # worst relative L2 over every op's full output on every rank against a
        # single-GPU engine run of the same model (checked before timing); the
        # ops are chained (each output, rounded to fp16, is a later op's input),
        # so fp32 summation-order differences compound along the 252 ops
        "tp_parity_rel_l2": float(f"{parity:.3e}"),
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



def codebooks_t() -> dict:
    import torch

    return {b: torch.from_numpy(codebook(b)) for b in (2, 3, 4)}


def build_step(cfg: dict, layer_bits: list[int], B: int, dev, seed: int, ctx: int, max_tokens: int,
               layers=None, head=None):
    """DecodeStep over a synthetic decoder, its tied fp16 embedding / LM head
    matrix and an N(0,1) KV cache of `ctx` positions."""
    import torch

    from turbopress_b200.step import DecodeStep
    from turbopress_b200.synthetic import step_config, synthetic_decoder

    if layers is None:
        layers, fnorm = synthetic_decoder(cfg, layer_bits, codebooks_t(), dev, seed=seed)
    else:
        layers, fnorm = layers
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    if head is None:
        head = (torch.randn(cfg["vocab"], cfg["hidden"], generator=g, device=dev) * 0.02).half()
    step = DecodeStep(layers, step_config(cfg), fnorm, batch=B, max_tokens=max_tokens, lm_head=head)
    step.k_cache[:, :, :, :ctx].normal_(generator=g)
    step.v_cache[:, :, :, :ctx].normal_(generator=g)
    step.set_position(ctx)
    return step, (layers, fnorm), head


def step_bytes_total(step, cfg: dict, B: int, ctx: int) -> tuple[int, int]:
    """(step-kernel algorithmic bytes, whole-step bytes incl. LM head and the
    embedding rows)."""
    from turbopress_b200.step import step_algorithmic_bytes

    kb = step_algorithmic_bytes(step.layers, step.cfg, B, ctx)
    kb += 2 * B * cfg["hidden"] * 2 + 2 * cfg["hidden"]  # final norm in/out + weight
    head = 2 * cfg["vocab"] * cfg["hidden"] + 2 * B * cfg["hidden"] + 12 * B
    return kb, kb + head + 2 * B * cfg["hidden"]


def time_decode(step, head, B: int, ctx: int, steps: int, warmup: int, stream, local: int, with_clocks=True):
    """Greedy decode steps replayed from a CUDA graph: device ms per step,
    kernel-only ms of tp_step_run, e2e ms per step, clocks."""
    import torch

    dev = step.device
    tok = torch.zeros(B, dtype=torch.int64, device=dev)
    # everything built on the default stream (weights, caches, tok) is ready
    # before the side stream uses it
    stream.wait_stream(torch.cuda.current_stream(dev))

    V = head.shape[0]

    def one_token():
        # token ids are clamped into the vocabulary before the lookup
        step.hidden.copy_(head.index_select(0, tok.clamp(0, V - 1)))
        out = step.run()
        nxt, _ = step.lm_head(out)
        step.advance()
        tok.copy_(nxt)

    with torch.cuda.stream(stream):
        one_token()
        stream.synchronize()
        step.status()
        t0 = tok.cpu()
        if int(t0.min()) < 0 or int(t0.max()) >= V or not bool(torch.isfinite(step.final_out).all()):
            raise RuntimeError(f"decode step produced token ids {t0.tolist()} (vocabulary {V}) / non-finite output")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            one_token()
        step.set_position(ctx)
        for _ in range(max(warmup, 3)):
            graph.replay()
        step.set_position(ctx)
        stream.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk = ClockSampler(local) if with_clocks else None
        if clk:
            clk.__enter__()
        a.record(stream)
        for _ in range(steps):
            graph.replay()
        b.record(stream)
        b.synchronize()
        if clk:
            clk.__exit__(None, None, None)
        ms = a.elapsed_time(b) / steps
        # the step kernel alone
        step.set_position(ctx)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(steps):
            step.run()
        k1.record(stream)
        k1.synchronize()
        ms_kernel = k0.elapsed_time(k1) / steps
        step.status()
        # end to end: token ids in from pinned host memory, chosen tokens out
        step.set_position(ctx)
        t_in = torch.zeros(B, dtype=torch.int64).pin_memory()
        t_out = torch.zeros(B, dtype=torch.int64).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            tok.copy_(t_in, non_blocking=True)
            graph.replay()
            t_out.copy_(tok, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        ms_e2e = e0.elapsed_time(e1) / steps
    return ms, ms_kernel, ms_e2e, (clk.summary() if clk else None), int(t_in.numel() * 8), int(t_out.numel() * 8)


def run_decode(args) -> dict | None:
    import torch

    from turbopress_b200.synthetic import MODELS as SMODELS, mixed_bits

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

    cfg = dict(SMODELS[args.model])
    if args.layers > 0:  # profiling: the first layers of the model only
        cfg["layers"] = args.layers
    B, bits = args.batch, args.bits
    tp_line = None
    if world > 1:
        # tensor-parallel engine of the decoder linears (one stream over N GPUs)
        tp_line = run_tp(args, dict(MODELS[args.model]), rank, world, local, dev, dist)
        if args.parallel == "tp":
            dist.destroy_process_group()
            return tp_line
    ctx = 1024 if args.model == "qwen3-4b" else 512 if args.model == "qwen3-0.6b" else 2048
    layer_bits = [bits] * cfg["layers"]
    steps, warm = args.steps, max(args.warmup, 3)
    max_tok = ctx + 3 * steps + warm + 16
    stream = torch.cuda.Stream(device=dev)
    step, parts, head = build_step(cfg, layer_bits, B, dev, args.seed, ctx, max_tok)
    barrier()
    ms, ms_kernel, ms_e2e, clocks, h2d, d2h = time_decode(step, head, B, ctx, steps, warm, stream, local)
    kbytes, sbytes = step_bytes_total(step, cfg, B, ctx)
    extra = {}
    if world == 1 and not args.quick:
        # mixed 2/3/4-bit layers, batch 1 and 8
        mb = mixed_bits(cfg["layers"], seed=args.seed)
        del step
        torch.cuda.empty_cache()
        c4 = {"bits_per_layer": mb, "avg_bits": sum(mb) / len(mb)}
        shared = None
        for b in (1, 8):
            st, shared, _ = build_step(cfg, mb, b, dev, args.seed + 1, ctx, max_tok, layers=shared, head=head)
            m, mk, me, _, _, _ = time_decode(st, head, b, ctx, steps, warm, stream, local, with_clocks=False)
            kb, sb = step_bytes_total(st, cfg, b, ctx)
            c4[f"batch{b}"] = {"ms_per_step": round(m, 4), "tok_s": round(b * 1000.0 / m, 1),
                              "kernel_ms": round(mk, 4), "gbs": round(sb / (m * 1e-3) / 1e9, 1),
                              "e2e_tok_s": round(b * 1000.0 / me, 1)}
            del st
            torch.cuda.empty_cache()
        extra["decode_c4"] = c4
        del shared
        torch.cuda.empty_cache()
    t = torch.tensor([ms, ms_e2e, ms_kernel], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e, ms_kernel = (float(v) for v in t)
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return None
    peak, peak_src = peaks_hbm()
    ach = kbytes / (ms_kernel * 1e-3) / 1e9
    out = {
        "metric": metric_name(MODELS[args.model], bits),
        "value": round(world * sbytes / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"u8 packed TCQ ({bits} bits/weight) -> fp16 activations, fp32 accumulate",
        "data": "synthetic: random-init decoder (seeded random trellis streams + reference data-free codebook, "
                "norm weights 1+N(0,0.1^2), fp16 LM head N(0,0.02^2)), KV cache N(0,1)",
        "config": {"workload": f"{cfg['name']} greedy decode step, batch {B}, {bits}-bit packed TCQ (S=64), "
                               f"{ctx}-token KV cache, LM head {cfg['vocab']}x{cfg['hidden']} fp16",
                   "path": "tp_step_run (one cooperative launch per step) + tp_lm_head_argmax, CUDA graph",
                   "layers": cfg["layers"], "batch": B, "bits": bits, "kv_tokens": ctx,
                   "step_bytes": int(sbytes), "step_kernel_bytes": int(kbytes),
                   "l2": "inputs larger than L2 (packed weights + LM head per step > 126 MB L2)",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "tok_s": round(world * B * 1000.0 / ms, 1),
        "e2e": {"value": round(world * sbytes / (ms_e2e * 1e-3) / 1e9, 1), "unit": "GB/s",
                "tok_s": round(world * B * 1000.0 / ms_e2e, 1), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(2 * steps),
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach / peak, 4),
                     "traffic": (round(kbytes * STEP_TRAFFIC[(args.model, bits, B)])
                                 if (args.model, bits, B) in STEP_TRAFFIC else None),
                     "kernel": "step_kernel (tp_step_run): step-kernel algorithmic bytes / CUDA-event duration, "
                               "mean over the timed launches",
                     "kernel_ms": round(ms_kernel, 4), "peak_source": peak_src},
        "clocks": clocks,
    }
    out.update(extra)
    if tp_line is not None:
        out["tp"] = {"parallelism": f"tp{world}", "ms_per_step": tp_line["ms_per_step"], "tok_s": tp_line["tok_s"],
                     "value": tp_line["value"], "unit": "GB/s", "e2e_tok_s": tp_line["e2e"]["tok_s"],
                     "kernel_ms": tp_line["roofline"]["kernel_ms"], "roofline_frac": tp_line["roofline"]["frac"],
                     "path": tp_line["config"]["path"], "workload": "decoder linears only (no attention)",
                     "tp_parity_rel_l2": tp_line["tp_parity_rel_l2"]}
    if world == 1 and not args.quick:
        out["gemv_c3"] = gemv_table(args, dev)
        out["c1"] = c1_section(args, dev)
    if not args.no_cpu_baseline and world == 1:
        info = cpu_info()
        nb, secs = cpu_layer_sample(dict(MODELS[args.model]), bits, list(range(7)), seed=args.seed)
        nbc, secc = cpu_layer_sample(dict(MODELS[args.model]), bits, list(range(7)), seed=args.seed, cached=True)
        out["cpu_baseline"] = {
            "value": round(nb / secs / 1e9, 3), "unit": "GB/s", "cores": info["torch_threads"], "kind": "port",
            "sample": f"reference tiled forward (torch restatement, oracle/torch_cpu.py) of one {cfg['name']} "
                      f"decoder layer's 7 linears ({nb / 1e6:.1f} MB packed) in {secs:.2f} s",
            "ms_per_mweight": round(secs * 1e3 / (sum(n * d for _, d, n in linear_shapes(MODELS[args.model])) / 1e6),
                                    3),
            "tok_s_extrapolated": round(1.0 / (secs * cfg["layers"]), 4),
            "cached_tok_s_extrapolated": round(1.0 / (secc * cfg["layers"]), 4),
            **info}
    if dist is not None:
        dist.destroy_process_group()
    return out


def host_payload(n: int, d: int, bits: int, seed: int) -> dict:
    """A format-v2 payload of uniform random packed bits (every bit string is
    a valid trellis codeword) with the reference's data-free codebook."""
    rng = np.random.default_rng(seed)
    return {"format": 2, "n": n, "d": d, "bits": bits, "n_states": 64, "block": d & -d, "seed": seed,
            "path_packed": rng.integers(0, 256, (n, -(-d // 8)), dtype=np.uint8),
            "member_packed": rng.integers(0, 256, (n, -(-d * (bits - 1) // 8)), dtype=np.uint8) if bits > 1 else None,
            "scales": ((rng.random(n) * 0.5 + 0.75) / math.sqrt(d)).astype(np.float16),
            "signs_packed": rng.integers(0, 256, (1, -(-d // 8)), dtype=np.uint8),
            "inv_equil": (rng.random(d) * 0.4 + 0.8).astype(np.float16),
            "codebook": codebook(bits).astype(np.float16), "bias": None}


def gemv_table(args, dev) -> dict:
    """Llama-3-8B linear shapes x 2/3/4 bits x batch 1/4/16,
    each GEMV in a CUDA graph of distinct weight copies (> 2x L2 in total),
    GB/s and fraction of measured HBM peak, and an oracle spot check."""
    import torch

    from oracle import tcq_oracle as O

    peak, _ = peaks_hbm()
    res = {}
    for n, d in ((4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)):
        for bits in (2, 3, 4):
            nbytes1 = n * d * bits // 8
            copies = max(2, min(16, math.ceil(3 * 126e6 / nbytes1)))
            # copy 0 from a host payload (kept for the oracle spot check), the rest generated on the GPU
            from turbopress_b200 import PackedTCQLinear
            p0 = host_payload(n, d, bits, seed=1000 * bits)
            mods = [PackedTCQLinear({k: (torch.from_numpy(v).to(dev) if isinstance(v, np.ndarray) else v)
                                     for k, v in p0.items()}, mode="cuda")]
            mods += [random_linear(n, d, bits, dev, seed=1000 * bits + c) for c in range(1, copies)]
            for B in (1, 4, 16):
                x = torch.randn(B, d, device=dev, dtype=torch.float16)
                s = torch.cuda.Stream(device=dev)
                s.wait_stream(torch.cuda.current_stream())
                with torch.no_grad(), torch.cuda.stream(s):
                    ys = [m(x) for m in mods]
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=s):
                        for m in mods:
                            m(x)
                    for _ in range(3):
                        graph.replay()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    reps = 10
                    e0.record(s)
                    for _ in range(reps):
                        graph.replay()
                    e1.record(s)
                    e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps / copies
                gb = gemv_bytes(n, d, bits, B) / (us * 1e-6) / 1e9
                # oracle spot check: the first 32 rows of copy 0
                p = dict(p0, n=32, path_packed=p0["path_packed"][:32], scales=p0["scales"][:32],
                         member_packed=None if p0["member_packed"] is None else p0["member_packed"][:32])
                ref = O.forward_fp32(p, x.cpu().numpy())
                got = ys[0][:, :32].float().cpu().numpy()
                rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
                res[f"{n}x{d}_b{bits}_B{B}"] = {"us": round(us, 2), "GBps": round(gb, 1),
                                                 "frac": round(gb / peak, 4), "spot_rows": 32,
                                                 "spot_rel_l2": float(f"{rel:.3e}")}
                del graph, ys
            del mods
            torch.cuda.empty_cache()
    return res


def c1_section(args, dev) -> dict:
    """BASELINE config 1 (the reference's CPU-runnable case): 1024 x 1024
    2-bit, from the reference encoder (golden fixture).  GPU: the packed GEMV
    (one layer, L2-resident); CPU: the reference tiled and cached forwards."""
    import torch

    from oracle import torch_cpu as T
    from tests.conftest import load_golden, payload_from
    from turbopress_b200 import PackedTCQLinear

    g = load_golden("layers")
    p = payload_from(g, "c1_")
    x = g["c1_x"]
    pd = {k: (torch.from_numpy(v).to(dev) if isinstance(v, np.ndarray) else v) for k, v in p.items()}
    m = PackedTCQLinear(pd, mode="cuda")
    xd = torch.from_numpy(x).to(dev)
    with torch.no_grad():
        y = m(xd)
        for _ in range(10):
            m(xd)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(100):
            m(xd)
        b.record()
        b.synchronize()
    us_gpu = a.elapsed_time(b) * 10.0
    rel = float(np.linalg.norm(y.float().cpu().numpy() - g["c1_y_tiled"]) / np.linalg.norm(g["c1_y_tiled"]))
    torch.set_num_threads(os.cpu_count() or 1)
    xt = torch.from_numpy(x)
    rs = T.rot_scale(p)
    T.tiled_forward(p, xt, rs)
    t0 = time.perf_counter()
    for _ in range(5):
        T.tiled_forward(p, xt, rs)
    ms_tiled = (time.perf_counter() - t0) / 5 * 1e3
    w16 = T.cached_weight(p)
    T.cached_forward(w16, xt)
    t0 = time.perf_counter()
    for _ in range(50):
        T.cached_forward(w16, xt)
    ms_cached = (time.perf_counter() - t0) / 50 * 1e3
    return {"shape": "1024x1024", "bits": 2, "gpu_us_per_call": round(us_gpu, 2),
            "gpu_rel_l2_vs_reference_tiled": float(f"{rel:.3e}"),
            "cpu_tiled_ms": round(ms_tiled, 3), "cpu_cached_ms": round(ms_cached, 4),
            "cpu_threads": torch.get_num_threads(),
            "note": "GPU time is per-call latency (the 0.26 MB layer is L2-resident)"}

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
    """Standalone packed GEMVs: the BASELINE config 3 table, or with --once
    one call per --shapes entry at --bits / --batch (for profiler captures)."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if not args.once:
        return {"workload": "gemv", "gemv_c3": gemv_table(args, dev)}
    for shp in args.shapes.split(","):
        n, d = map(int, shp.lower().split("x"))
        m = random_linear(n, d, args.bits, dev, seed=1)
        x = torch.randn(args.batch, d, device=dev, dtype=torch.float16)
        with torch.no_grad():
            m(x)
        torch.cuda.synchronize()
    return {"workload": "gemv", "once": args.shapes, "bits": args.bits, "batch": args.batch}

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
    """The reference arm: the reference's own CPU forward (tiled; torch
    restatement in oracle/torch_cpu.py) on this host's cores, one linear of
    the workload's decoder layer per step (cycling q/k/v/o/gate/up/down)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    cfg, bits = dict(MODELS[args.model]), args.bits
    for i in range(args.warmup):
        cpu_layer_sample(cfg, bits, [i], seed=args.seed)
    tot_b, tot_t = 0, 0.0
    for i in range(args.steps):
        b, t = cpu_layer_sample(cfg, bits, [i], seed=args.seed)
        tot_b += b
        tot_t += t
    value = tot_b / tot_t / 1e9
    info = cpu_info()
    return {
        "impl": "reference",
        "metric": metric_name(cfg, bits),
        "value": round(value, 3), "unit": "GB/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(tot_t / args.steps * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8 packed TCQ -> fp32 (reference CPU tiled path)",
        "data": "synthetic: seeded random trellis streams + reference data-free codebook",
        "config": {"workload": f"{cfg['name']} decoder linears, batch 1, {bits}-bit packed TCQ, S=64",
                   "sample": "one linear per step, cycling q/k/v/o/gate/up/down"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": info["torch_threads"], "kind": "port",
                         "sample": "reference tiled forward (torch restatement of turbopress/runtime.py:291-331: "
                                   "unpack, window decode, fp16 dequant per 1024-row tile, fp32 matmul), one "
                                   "linear per step", **info},
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
    ap.add_argument("--quick", action="store_true", help="decode line only (no gemv_c3 / c1 / decode_c4 keys)")
    ap.add_argument("--model", choices=sorted(MODELS), default="qwen3-4b",
                    help="decode workload: model shape (qwen3-4b is the contract line)")
    ap.add_argument("--parallel", choices=["replicas", "tp"], default="replicas",
                    help="N > 1: the line from N independent decode streams (replicas, with the tensor-parallel "
                         "engine of the decoder linears under 'tp') or the tensor-parallel engine itself")
    ap.add_argument("--layers", type=int, default=0, help="profiling: decoder layers of the model (0: all)")
    ap.add_argument("--workload", choices=["decode", "gemv", "lmhead"], default="decode",
                    help="decode: the contract line; gemv: the config-3 GEMV table; lmhead: the greedy LM head")
    ap.add_argument("--shapes", default="14336x4096", help="gemv --once: comma-separated NxD (out x in) shapes")
    ap.add_argument("--once", action="store_true", help="gemv workload: one call per shape (profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        out = run_reference(args)
    elif args.workload == "lmhead":
        out = run_lmhead(args)
    elif args.workload == "gemv":
        out = run_gemv(args)
    else:
        out = run_decode(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

