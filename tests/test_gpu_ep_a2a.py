"""Mode A expert parallelism (k3d_moe_swiglu_a2a: all-to-all dispatch and combine of
data-parallel tokens) on the GPU. One rank: every expert is local, the rows still go
through the plan, the pack, the exchange and the top-k combine, and the result equals the
replicated-activation layer (k3d_moe_swiglu) and the oracle. Two GPUs: NCCL send/recv
between the ranks, each with its own batch, against the oracle."""
import multiprocessing as mp
import socket
import subprocess

import numpy as np
import pytest

import k3cuda
import synth
from conftest import max_rel_err
from test_gpu_moe import run_layer, small_layer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,tiled", [(1, True), (8, True), (64, True), (8, False), (64, False)])
def test_moe_a2a_one_rank_matches_replicated_layer(k3, oracle, T, tiled):
    g, experts, W, bias, sh = small_layer(900 + T, E=16)
    hidden, inter, E = 1024, 512, 16
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=tiled)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    y_r, idx_r, w_r = run_layer(k3, mw, x, T)
    X = k3cuda.DevBuf.from_array(x)
    prev = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    O = k3cuda.DevBuf.from_array(prev)
    I = k3cuda.DevBuf(T * 8 * 4)
    Wt = k3cuda.DevBuf(T * 8 * 4)
    n = mw.a2a_ws_bytes(T, 1)
    WS = k3cuda.DevBuf(n)
    k3cuda.check(mw.run_a2a(O.ptr, X.ptr, T, T, WS.ptr, n, 1, I.ptr, Wt.ptr))
    k3cuda.check(k3.k3d_sync())
    y = O.download(np.float32, (T, hidden))
    assert np.array_equal(I.download(np.int32, (T, 8)), idx_r)
    assert np.array_equal(Wt.download(np.float32, (T, 8)), w_r)
    assert np.array_equal(y, prev + y_r)         # accumulate: prev + the same layer output
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert max_rel_err(y - prev, want) <= 1e-4


@pytest.mark.parametrize("T,tiled", [(1, True), (8, True), (64, True), (8, False)])
def test_moe_a2a_dev_one_rank_matches_replicated_layer_and_captures(k3, oracle, T, tiled):
    """Mode A planned on the device: the plan kernel, fixed-region exchanges, the masked
    received rows and the top-k combine give the replicated layer's bits; then the call is
    captured into a CUDA graph and replayed on new inputs, with the same bits as an eager
    replicated call on those inputs."""
    g, experts, W, bias, sh = small_layer(700 + T, E=16)
    hidden, inter, E = 1024, 512, 16
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=tiled)
    n = mw.a2a_ws_bytes(T, 1)
    WS = k3cuda.DevBuf(n)
    X = k3cuda.DevBuf(T * hidden * 4)
    O = k3cuda.DevBuf(T * hidden * 4)
    I = k3cuda.DevBuf(T * 8 * 4)
    xs = [synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0)) for _ in range(3)]
    prev = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))

    def replicated(x):
        y, idx, _ = run_layer(k3, mw, x, T)
        return y, idx

    # eager, accumulating into prev
    X.upload(xs[0])
    O.upload(prev)
    k3cuda.check(mw.run_a2a_dev(O.ptr, X.ptr, T, WS.ptr, n, 1, I.ptr, None))
    k3cuda.check(k3.k3d_sync())
    y_r, idx_r = replicated(xs[0])
    assert np.array_equal(I.download(np.int32, (T, 8)), idx_r)
    assert np.array_equal(O.download(np.float32, (T, hidden)), prev + y_r)
    want, _, _ = oracle.moe_swiglu(xs[0], T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert max_rel_err(O.download(np.float32, (T, hidden)) - prev, want) <= 1e-4
    # captured once, replayed on new inputs
    k3cuda.check(k3.k3d_graph_begin())
    r = mw.run_a2a_dev(O.ptr, X.ptr, T, WS.ptr, n, 0, I.ptr, None)
    graph = k3.k3d_graph_end()
    k3cuda.check(r, "capture")
    assert graph, k3.k3d_last_message()
    try:
        for x in xs[1:]:
            X.upload(x)
            k3cuda.check(k3.k3d_graph_launch(graph))
            k3cuda.check(k3.k3d_sync())
            y_r, idx_r = replicated(x)
            assert np.array_equal(I.download(np.int32, (T, 8)), idx_r)
            assert np.array_equal(O.download(np.float32, (T, hidden)), y_r)
    finally:
        k3.k3d_graph_destroy(graph)


def test_moe_a2a_rejects_wrong_expert_range(k3):
    g, experts, W, bias, sh = small_layer(950, E=16)
    mw = k3cuda.MoeWeights(1024, 512, 16, 8, W, bias, shared=sh, experts=experts, lo=0, hi=8)
    X = k3cuda.DevBuf(1024 * 4)
    O = k3cuda.DevBuf(1024 * 4)
    n = mw.a2a_ws_bytes(1, 1)
    WS = k3cuda.DevBuf(n)
    assert mw.run_a2a(O.ptr, X.ptr, 1, 1, WS.ptr, n) == k3cuda.K3D_EINVAL
    k3.k3d_clear_status()


def _gpu_count():
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=60).stdout
    except (OSError, subprocess.SubprocessError):
        return 0
    return sum(1 for line in out.splitlines() if line.startswith("GPU "))


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("tiled,dev", [(True, False), (False, False), (True, True)])
def test_moe_a2a_two_gpus_matches_oracle(tiled, dev):
    import ep_a2a_gpu_worker
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=ep_a2a_gpu_worker.run, args=(r, 2, port, 31, tiled, dev)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_lm_head_vocab_split_two_gpus():
    """Each rank holds half of the LM head's rows; the packed (logit, index) maxima are
    combined by an NCCL max, so every rank gets the argmax over the whole vocabulary (the
    streamed GEMV path at batch 3, the tensor-core GEMM path at batch 6)."""
    import ep_lm_gpu_worker
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=ep_lm_gpu_worker.run, args=(r, 2, port, 41)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes
