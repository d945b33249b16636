"""The three MXFP4 expert kernels (tcgen05 block-scaled, mma.sync, CUDA cores), selected
with k3d_set_expert_kernel, each against the oracle (the CPU engine's scalar MXFP4 dot in
fp64, k3_ops.c:1380-1785) at the expert tolerance: normwise max relative error 1e-4
(north star: 1e-3 for fp32-accumulated outputs)."""
import ctypes

import numpy as np
import pytest

import k3cuda
import synth
from conftest import max_rel_err
from test_gpu_moe import run_layer, small_layer

pytestmark = pytest.mark.gpu

KINDS = [0, 1, 2]          # 0 tcgen05 (default), 1 mma.sync, 2 CUDA cores


@pytest.fixture
def kernel_kind(k3, request):
    k3cuda.check(k3.k3d_set_expert_kernel(request.param))
    yield request.param
    k3cuda.check(k3.k3d_set_expert_kernel(0))


def run_expert(k3, x, e, hidden, inter, calls=2):
    bufs = {k: k3cuda.DevBuf.from_array(v) for k, v in e.items()}
    q = k3cuda.K3ExpertQ(*(bufs[k].ptr for k in ("p1", "s1", "p3", "s3", "p2", "s2")))
    X = k3cuda.DevBuf.from_array(x)
    Y = k3cuda.DevBuf(hidden * 4)
    n = k3.k3d_expert_ws_bytes(hidden, inter)
    WS = k3cuda.DevBuf(n)
    outs = []
    for _ in range(calls):
        Y.zero()
        k3cuda.check(k3.k3d_expert_swiglu(Y.ptr, X.ptr, ctypes.byref(q), hidden, inter, WS.ptr, n))
        k3cuda.check(k3.k3d_sync())
        outs.append(Y.download(np.float32, hidden))
    return outs


@pytest.mark.parametrize("kernel_kind", KINDS, indirect=True)
@pytest.mark.parametrize("hidden,inter", [(512, 512), (1024, 512), (2048, 1024)])
def test_single_expert_each_kernel(k3, oracle, kernel_kind, hidden, inter):
    g = synth.rng(hidden + inter + 7)
    e = synth.mxfp4_expert(g, hidden, inter)
    x = synth.bf16_to_f32(synth.bf16_normal(g, hidden, 1.0))
    want = oracle.expert_swiglu(x, e, hidden, inter)
    y1, y2 = run_expert(k3, x, e, hidden, inter)
    assert max_rel_err(y1, want) <= 1e-4
    assert np.array_equal(y1, y2), "repeated calls must give identical results"


@pytest.mark.parametrize("kernel_kind", [0], indirect=True)
def test_tcgen05_scale_edge_bytes(k3, oracle, kernel_kind):
    """E8M0 255 (NaN to the tensor core) counts as zero like the CPU engine; 0 is 2^-127;
    the extremes 1 and 254 with small/large activations stay finite and match."""
    hidden, inter = 1024, 512
    g = synth.rng(31)
    e = synth.mxfp4_expert(g, hidden, inter)
    for k in ("s1", "s3", "s2"):
        s = e[k].reshape(-1)
        s[::7] = 255
        s[3::11] = 0
    x = synth.bf16_to_f32(synth.bf16_normal(g, hidden, 1.0))
    want = oracle.expert_swiglu(x, e, hidden, inter)
    y, _ = run_expert(k3, x, e, hidden, inter)
    assert np.all(np.isfinite(y))
    assert max_rel_err(y, want) <= 1e-4


@pytest.mark.parametrize("kernel_kind", [0], indirect=True)
def test_tcgen05_activation_dynamic_range(k3, oracle, kernel_kind):
    """Activations spanning ~2^-60..2^20 inside 32-element blocks and exact zeros: the
    E2M1 piece decomposition of the B operand keeps the result at fp32 accuracy."""
    hidden, inter = 1024, 512
    g = synth.rng(32)
    e = synth.mxfp4_expert(g, hidden, inter)
    x = (g.standard_normal(hidden) * np.exp2(g.integers(-60, 20, hidden))).astype(np.float32)
    x[::5] = 0.0
    want = oracle.expert_swiglu(x, e, hidden, inter)
    y, _ = run_expert(k3, x, e, hidden, inter)
    assert max_rel_err(y, want) <= 1e-4


@pytest.mark.parametrize("kernel_kind", KINDS, indirect=True)
@pytest.mark.parametrize("T", [1, 3, 8])
def test_moe_layer_each_kernel(k3, oracle, kernel_kind, T):
    g, experts, W, bias, sh = small_layer(300 + T, E=16)
    hidden, inter, E = 1024, 512, 16
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    y, idx, wts = run_layer(k3, mw, x, T)
    want, oi, ow = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256,
                                     *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(y, want) <= 1e-4


def test_pretile_round_trip(k3):
    """k3d_expert_pretile is a pure rearrangement (plus E8M0 255 -> 0): un-tiling its output
    on the host gives the checkpoint bytes back exactly."""
    from test_gpu_stack import untile_expert
    hidden, inter = 1024, 512
    g = synth.rng(41)
    e = synth.mxfp4_expert(g, hidden, inter)
    for k in ("s1", "s3", "s2"):
        e[k].reshape(-1)[5::13] = 255
    src = {k: k3cuda.DevBuf.from_array(v) for k, v in e.items()}
    q = k3cuda.K3ExpertQ(*(src[k].ptr for k in ("p1", "s1", "p3", "s3", "p2", "s2")))
    gu, gus = inter * hidden // 2, inter * hidden // 32
    sizes = [2 * gu, 2 * gus, gu, gus]
    offs, o = [], 0
    for s_ in sizes:
        offs.append(o)
        o += (s_ + 255) // 256 * 256
    slot = k3cuda.DevBuf(o)
    slot.zero()
    dst = k3cuda.K3ExpertQ(slot.ptr + offs[0], slot.ptr + offs[1], None, None,
                           slot.ptr + offs[2], slot.ptr + offs[3])
    k3cuda.check(k3.k3d_expert_pretile(ctypes.byref(dst), ctypes.byref(q), hidden, inter))
    k3cuda.check(k3.k3d_sync())
    back = untile_expert(slot.download(np.uint8, o), hidden, inter)
    for k, v in e.items():
        want = np.ascontiguousarray(v).reshape(-1).copy()
        if k.startswith("s"):
            want[want == 255] = 0
        assert np.array_equal(back[k], want), k


@pytest.mark.parametrize("T", [1, 3, 8, 64])
def test_moe_layer_tiled_experts(k3, oracle, T):
    """Experts in the tiled layout: the tcgen05 kernel streams whole stages with bulk
    copies. T = 64 (512 assignments) runs with one K slice."""
    g, experts, W, bias, sh = small_layer(500 + T, E=16)
    hidden, inter, E = 1024, 512, 16
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    y, idx, wts = run_layer(k3, mw, x, T)
    want, oi, ow = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256,
                                     *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(y, want) <= 1e-4


@pytest.mark.parametrize("T,E", [(9, 16), (16, 16), (64, 16), (33, 64)])
def test_grouped_pass_matches_one_token_items_and_oracle(k3, oracle, T, E):
    """Batches (more than 64 assignments, tiled experts): up to four tokens routed to one
    expert share each weight stage (B = their stacked pieces, N = 64, partials by position,
    the combine maps assignments to positions). Against one token per item (kind 3) and the
    oracle; E = 64 leaves single-token experts and groups of every size."""
    g, experts, W, bias, sh = small_layer(1100 + T, E=E)
    hidden, inter = 1024, 512
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    ys = {}
    try:
        for kind in (0, 3, 0):
            k3cuda.check(k3.k3d_set_expert_kernel(kind))
            y, idx, _ = run_layer(k3, mw, x, T)
            ys.setdefault(kind, []).append(y)
    finally:
        k3cuda.check(k3.k3d_set_expert_kernel(0))
    assert np.array_equal(ys[0][0], ys[0][1])
    assert max_rel_err(ys[0][0], ys[3][0]) <= 1e-5
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(ys[0][0], want) <= 1e-4


def test_grouped_pass_config1_shapes(k3, oracle):
    """The grouped pass at config 1's expert shapes (7168 -> 2048) for 16 tokens over 16
    tiled experts (many tokens per expert), against the oracle."""
    hidden, inter, E, T = 7168, 2048, 16, 16
    g, experts, W, bias, sh = small_layer(1211, hidden=hidden, inter=inter, E=E, shared_inter=256)
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    y, idx, _ = run_layer(k3, mw, x, T)
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(y, want) <= 1e-4


@pytest.mark.parametrize("T", [1, 3, 8])
def test_resident_b_matches_per_stage_b_and_oracle(k3, oracle, T):
    """Tiled experts up to 64 assignments: items ordered (token, K chunk, tile) so that B is
    loaded once per run into a slot beside a 6-stage weight ring; against the kernel that
    carries B in every stage (kind 3) and the oracle."""
    g, experts, W, bias, sh = small_layer(1300 + T, E=16)
    hidden, inter, E = 1024, 512, 16
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    ys = {}
    try:
        for kind in (0, 3, 0):
            k3cuda.check(k3.k3d_set_expert_kernel(kind))
            y, idx, _ = run_layer(k3, mw, x, T)
            ys.setdefault(kind, []).append(y)
    finally:
        k3cuda.check(k3.k3d_set_expert_kernel(0))
    assert np.array_equal(ys[0][0], ys[0][1])
    assert max_rel_err(ys[0][0], ys[3][0]) <= 1e-5
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(ys[0][0], want) <= 1e-4


@pytest.mark.parametrize("T,hidden,inter,E", [(1, 1024, 512, 16), (2, 1024, 512, 16), (1, 7168, 2048, 16)])
def test_fused_pass_matches_three_launches_and_oracle(k3, oracle, T, hidden, inter, E):
    """Kind 4: decode-sized work lists (up to 16 assignments) run gate/up, the act split and
    down as one launch (k_mxfp4_fused) with cross-CTA counters; the result is bit-identical
    to the three-launch form (kind 0) and matches the oracle; repeated calls agree (the
    router zeroes the counters every call, so a fresh workspace needs no set-up)."""
    g, experts, W, bias, sh = small_layer(1400 + T + hidden, hidden=hidden, inter=inter, E=E)
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, tiled=True)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    ys = {}
    try:
        for kind in (4, 0, 4):
            k3cuda.check(k3.k3d_set_expert_kernel(kind))
            y, idx, _ = run_layer(k3, mw, x, T)
            ys.setdefault(kind, []).append(y)
    finally:
        k3cuda.check(k3.k3d_set_expert_kernel(0))
    assert np.array_equal(ys[4][0], ys[0][0])
    assert np.array_equal(ys[4][0], ys[4][1])
    want, oi, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert np.array_equal(idx, oi)
    assert max_rel_err(ys[0][0], want) <= 1e-4
