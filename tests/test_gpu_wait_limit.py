"""Failure detection on the GPU without a fault: the pipelined expert kernel's bounded waits
run out on purpose (k3d_set_wait_limit set far below one weight stage's copy latency), the
kernel records K3D_ETIMEOUT in the device error flag, drains the copies it issued, frees
its tensor memory and returns; the host reads the status, and the next call with the
default limit succeeds and gives the same result as before."""
import ctypes

import numpy as np
import pytest

import k3cuda
import synth
from conftest import max_rel_err
from test_gpu_moe import run_layer, small_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [4, 0])
def test_expert_pass_wait_limit_times_out_and_context_recovers(k3, oracle, kind):
    """kind 4: the one-launch expert pass (cross-CTA counters and an abort word); kind 0: the
    three-launch pass."""
    hidden, inter, E, T = 1024, 512, 16, 1
    g, experts, W, bias, sh = small_layer(2077, E=E)
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    k3cuda.check(k3.k3d_set_expert_kernel(kind))
    try:
        _run_timeout_case(k3, oracle, mw, x, T, hidden, inter, E, W, bias, experts, sh)
    finally:
        k3cuda.check(k3.k3d_set_expert_kernel(0))


def _run_timeout_case(k3, oracle, mw, x, T, hidden, inter, E, W, bias, experts, sh):
    y0, idx0, _ = run_layer(k3, mw, x, T)

    k3cuda.check(k3.k3d_set_wait_limit(200))          # ~0.1 us: no stage lands that fast
    try:
        with pytest.raises(k3cuda.K3Error):
            run_layer(k3, mw, x, T)
        code, site = ctypes.c_int(), ctypes.c_int()
        k3.k3d_device_error(ctypes.byref(code), ctypes.byref(site))
        assert code.value == k3cuda.K3D_ETIMEOUT
        assert site.value == 1                        # the MXFP4 expert kernel
    finally:
        k3cuda.check(k3.k3d_set_wait_limit(0))
        k3.k3d_clear_status()

    y1, idx1, _ = run_layer(k3, mw, x, T)             # tensor memory was released
    assert np.array_equal(idx1, idx0)
    assert np.array_equal(y1, y0)
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert max_rel_err(y1, want) <= 1e-4
