"""Config 1 (MoE layer: bit-exact router, MXFP4 SwiGLU experts in top-k order, bf16 shared
expert) on the GPU through the C ABI, against the oracle."""
import numpy as np
import pytest

import k3cuda
from conftest import max_rel_err
import synth

pytestmark = pytest.mark.gpu


def small_layer(seed, hidden=1024, inter=512, E=64, topk=8, shared_inter=256):
    g = synth.rng(seed)
    experts = [synth.mxfp4_expert(g, hidden, inter) for _ in range(E)]
    W = synth.bf16_normal(g, (E, hidden), 0.02)
    bias = g.uniform(-0.1, 0.1, E).astype(np.float32)
    sh = (synth.bf16_normal(g, (shared_inter, hidden), 0.02),
          synth.bf16_normal(g, (shared_inter, hidden), 0.02),
          synth.bf16_normal(g, (hidden, shared_inter), 0.02))
    return g, experts, W, bias, sh


def run_layer(k3, mw, x, T, accumulate_into=None):
    hidden = x.shape[1]
    X = k3cuda.DevBuf.from_array(x)
    out0 = accumulate_into if accumulate_into is not None else np.zeros((T, hidden), np.float32)
    O = k3cuda.DevBuf.from_array(out0)
    I = k3cuda.DevBuf(T * mw.shape.topk * 4)
    Wt = k3cuda.DevBuf(T * mw.shape.topk * 4)
    n = mw.ws_bytes(T)
    WS = k3cuda.DevBuf(n)
    k3cuda.check(mw.run(O.ptr, X.ptr, T, WS.ptr, n, 1 if accumulate_into is not None else 0,
                        I.ptr, Wt.ptr))
    k3cuda.check(k3.k3d_sync())
    return (O.download(np.float32, (T, hidden)), I.download(np.int32, (T, mw.shape.topk)),
            Wt.download(np.float32, (T, mw.shape.topk)))


@pytest.mark.parametrize("T,inter", [(1, 512), (8, 512), (64, 512), (512, 512), (8, 256)])
def test_moe_layer_matches_oracle(k3, oracle, T, inter):
    """inter 512 runs the tensor-core expert kernels, inter 256 the CUDA-core ones."""
    g, experts, W, bias, sh = small_layer(100 + T, inter=inter)
    hidden, E = 1024, 64
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    y, idx, wts = run_layer(k3, mw, x, T)
    want, oi, ow = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256,
                                     *sh)
    assert np.array_equal(idx, oi)
    assert np.array_equal(wts.view(np.uint32), ow.view(np.uint32))
    assert max_rel_err(y, want) <= 1e-4


def test_moe_residual_accumulate_and_expert_parallel_partials(k3, oracle):
    """Two ranks' partials (experts split in halves, shared expert on rank 0) sum to the
    whole layer, and accumulate=1 adds onto the residual."""
    T = 8
    g, experts, W, bias, sh = small_layer(7)
    hidden, inter, E = 1024, 512, 64
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, hidden), 1.0))
    resid = g.standard_normal((T, hidden), dtype=np.float32)
    parts = []
    for lo, hi, add in ((0, 32, 1), (32, 64, 0)):
        mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts, lo=lo,
                               hi=hi, add_shared=add)
        y, _, _ = run_layer(k3, mw, x, T)
        want, _, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256,
                                       *sh, lo=lo, hi=hi, add_shared=add)
        assert max_rel_err(y, want) <= 1e-4
        parts.append(y)
    full, _, _ = oracle.moe_swiglu(x, T, hidden, inter, E, 8, 1, 2.5, W, bias, experts, 256, *sh)
    assert max_rel_err(parts[0] + parts[1], full) <= 1e-4
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, experts=experts)
    y, _, _ = run_layer(k3, mw, x, T, accumulate_into=resid.copy())
    assert max_rel_err(y, resid + full) <= 1e-4


def test_moe_config1_full_size_T1(k3, oracle):
    """384 device-filled experts at 7168 -> 2048 (9 GB in HBM); the oracle reads back only
    the eight the router selected."""
    hidden, inter, E = 7168, 2048, 384
    g = synth.rng(2024)
    W = synth.bf16_normal(g, (E, hidden), 0.02)
    bias = g.uniform(-0.1, 0.1, E).astype(np.float32)
    sh = (synth.bf16_normal(g, (inter, hidden), 0.02), synth.bf16_normal(g, (inter, hidden), 0.02),
          synth.bf16_normal(g, (hidden, inter), 0.02))
    mw = k3cuda.MoeWeights(hidden, inter, E, 8, W, bias, shared=sh, seed=99)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (1, hidden), 1.0))
    y, idx, wts = run_layer(k3, mw, x, 1)
    oi, ow = oracle.router_bf16(x[0], W, bias, 8, 1, 2.5)
    assert np.array_equal(idx[0], oi)
    assert np.array_equal(wts[0].view(np.uint32), ow.view(np.uint32))
    experts = [None] * E
    for e in oi:
        d = mw.download_expert(int(e))
        experts[e] = {"p1": d["p1"].reshape(inter, hidden // 2), "s1": d["s1"],
                      "p3": d["p3"].reshape(inter, hidden // 2), "s3": d["s3"],
                      "p2": d["p2"].reshape(hidden, inter // 2), "s2": d["s2"]}
    want, _, _ = oracle.moe_swiglu(x, 1, hidden, inter, E, 8, 1, 2.5, W, bias, experts, inter, *sh)
    assert max_rel_err(y, want) <= 1e-4
    assert k3.k3d_moe_last_unique() == 8
