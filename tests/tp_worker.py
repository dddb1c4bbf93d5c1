"""Worker of the 2+ GPU tensor-parallel engine test (run under torchrun).

Each rank builds the same decoder-like chain of packed linears, runs the
tensor-parallel engine twice (both arena buffers) and checks every op's full
output against the oracle's fp32 dequant-then-matmul on the input the engine
fed that op.  Exit code 0 = parity on this rank.
"""

import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from oracle import tcq_oracle as O  # noqa: E402
from turbopress_b200 import PackedTCQLinear  # noqa: E402
from turbopress_b200.tp import TPDecodeEngine  # noqa: E402

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    rank = dist.get_rank()
    bits, B = int(os.environ.get("TP_BITS", "3")), int(os.environ.get("TP_BATCH", "2"))
    h, inter, q = 640, 1536, 1024
    cb = np.sort(np.random.default_rng(bits).standard_normal(1 << (bits + 1)) * 1.2)
    payloads, inputs = [], []
    seed = 100 * bits
    for _ in range(2):
        base = len(payloads)
        for n, d, dep in [(q, h, None if base == 0 else base - 1), (256, h, None if base == 0 else base - 1),
                          (256, h, None if base == 0 else base - 1), (h, q, base), (inter, h, base + 3),
                          (inter, h, base + 3), (h, inter, base + 4)]:
            payloads.append(O.random_payload(n, d, bits, 64, seed=seed, codebook=cb, bias=(seed % 3 == 0)))
            inputs.append(dep)
            seed += 1
    mods = [PackedTCQLinear({k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) if isinstance(v, np.ndarray)
                             else v for k, v in p.items()}, mode="cuda") for p in payloads]
    eng = TPDecodeEngine(mods, inputs, batch=B)
    x = np.random.default_rng(7).standard_normal((B, h)).astype(np.float16)
    worst = 0.0
    for rep in range(3):
        outs = eng.run(torch.from_numpy(x).to(dev))
        torch.cuda.synchronize()
        eng.check()
        for i, (p, dep) in enumerate(zip(payloads, inputs)):
            xin = x if dep is None else outs[dep].cpu().numpy()
            err = rel_l2(outs[i].cpu().numpy(), O.forward_fp32(p, xin))
            worst = max(worst, err)
            if err >= REL_L2_TOL:
                print(f"rank {rank} rep {rep} op {i}: rel L2 {err:.3e}", flush=True)
                return 1
    # graph capture of the launch (kernel only)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            eng.launch()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    eng.check()
    out_last = eng.outputs_buf[(eng.step - 1) % 2][-1].cpu().numpy()
    xin = eng.outputs_buf[(eng.step - 1) % 2][inputs[-1]].cpu().numpy()
    err = rel_l2(out_last, O.forward_fp32(payloads[-1], xin))
    if err >= REL_L2_TOL:
        print(f"rank {rank} graph: rel L2 {err:.3e}", flush=True)
        return 1
    print(f"rank {rank} ok, worst rel L2 {worst:.2e}", flush=True)
    eng.close()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
