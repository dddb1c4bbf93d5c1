"""Device-side failure reporting, tested without a GPU fault.

The step kernel's grid barriers are bounded waits: a barrier that is made to
wait for an arrival that never comes (``set_wait(extra_arrivals=1)``: a
count nothing reaches) gives up after its limit, the step returns, the status
word says so and the same context runs the next step correctly.  The GEMV's
status word is checked the same way from a host-written failure record (the
status bit and a half-counted split-K counter that a call which gave up
leaves behind).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

DEV = "cuda"
STATUS_OFF = 16384 * 4          # tp_gemv_sk.cuh kStatusOff
COUNTER_BYTES = STATUS_OFF + 256  # tp_gemv_sk.cuh kCounterBytes


def _codebooks():
    with np.load(GOLDEN / "codebooks.npz") as f:
        return {b: torch.from_numpy(f[f"opt_b{b}_s64"]) for b in (2, 3, 4)}


def test_step_barrier_timeout_is_reported_and_context_recovers():
    from turbopress_b200.step import DecodeStep
    from turbopress_b200.synthetic import step_config, synthetic_decoder

    cfg = dict(name="test", layers=2, hidden=1024, inter=3072, q_heads=16, kv_heads=8, head_dim=128,
               rope_theta=1_000_000.0, qk_norm=True)
    layers, fnorm = synthetic_decoder(cfg, [3, 3], _codebooks(), DEV, seed=3)
    step = DecodeStep(layers, step_config(cfg), fnorm, batch=1, max_tokens=64)
    g = torch.Generator(device=DEV).manual_seed(0)
    step.k_cache.normal_(generator=g)
    step.v_cache.normal_(generator=g)
    step.set_position(20)
    x = torch.randn(1, cfg["hidden"], device=DEV, generator=g).half()
    step.hidden.copy_(x)
    ref = step.run().clone()
    step.status()

    # every barrier now waits for one arrival more than the grid makes
    step.set_wait(barrier_us=2000, extra_arrivals=1)
    step.hidden.copy_(x)
    step.run()
    with pytest.raises(RuntimeError, match="barrier"):
        step.status()
    # the status was cleared by reading it
    step.status()

    # back to normal: the same context gives the same result
    step.set_wait(0, 0)
    step.hidden.copy_(x)
    out = step.run()
    step.status()
    torch.cuda.synchronize()
    # the linears' partial sums meet in fp32 atomics (summation order varies
    # between runs), so the comparison allows a few fp16 ulps
    assert float((out.float() - ref.float()).norm() / ref.float().norm()) < 2e-3


def test_gemv_status_reports_and_clears_counter_block():
    from turbopress_b200 import runtime as R
    from turbopress_b200.synthetic import random_packed_linear

    lin = random_packed_linear(512, 2560, 3, _codebooks()[3], DEV, seed=5)
    x = torch.randn(1, 2560, device=DEV).half()
    ref = lin(x).clone()
    R.check_device_status()  # nothing to report

    idx = torch.cuda.current_device()
    ws = R.WORKSPACE._bufs[idx]
    # what a call that gave up leaves: a status bit and a counter part-way
    ws[STATUS_OFF] = 2
    ws[0:4] = torch.tensor([3, 0, 0, 0], dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="bounded device wait"):
        R.check_device_status()
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    R.check_device_status()

    y = lin(x)
    R.check_device_status()
    assert torch.equal(y, ref)


def test_gemv_noalloc_status_ok_after_calls():
    from turbopress_b200 import _abi
    from turbopress_b200.synthetic import random_packed_linear

    lin = random_packed_linear(256, 1024, 2, _codebooks()[2], DEV, seed=9)
    x = torch.randn(2, 1024, device=DEV).half()
    y = torch.empty(2, 256, device=DEV, dtype=torch.float16)
    lib = _abi.lib()
    st = torch.cuda.current_stream().cuda_stream
    _abi.check(lib.tp_tcq_gemv_noalloc(
        x.data_ptr(), _abi.dtype_code(x.dtype), lin.rot_scale.data_ptr(), lin.tcq_stream.data_ptr(),
        lin.scales.data_ptr(), lin.codebook.data_ptr(), None, y.data_ptr(), _abi.dtype_code(y.dtype), 2, 256, 1024,
        lin.block, lin.bits, lin.n_states, st), "noalloc")
    _abi.check(lib.tp_gemv_noalloc_status(st), "noalloc status")
    assert torch.isfinite(y.float()).all()
