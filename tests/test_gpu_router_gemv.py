"""Router (bit-exact), GEMVs and the KDA step on the GPU through the C ABI."""
import ctypes

import numpy as np
import pytest

import k3cuda
from conftest import assert_close_elementwise, load_npz, manifest_tol, max_rel_err
import synth

pytestmark = pytest.mark.gpu


def test_router_reference_fixture_exact(k3, oracle):
    d, meta = load_npz("ref_ops/router.npz")
    k = int(meta["top_k"])
    for t in range(d["in"].shape[0]):
        idx = np.empty(k, np.int32)
        w = np.empty(k, np.float32)
        k3.k3_router(idx.ctypes.data, w.ctypes.data, d["in"][t].ctypes.data,
                     d["gate_weight"].ctypes.data, d["bias"].ctypes.data, d["in"].shape[1],
                     d["gate_weight"].shape[0], k, 1, 1.0)
        oi, ow = oracle.router(d["in"][t], d["gate_weight"], d["bias"], k, 1, 1.0)
        assert np.array_equal(idx, oi) and np.array_equal(w.view(np.uint32), ow.view(np.uint32))
        assert list(idx) == list(d["topk_idx"][t].astype(int))


def test_router_config1_golden_bit_exact(k3):
    """Indices AND weights equal the compiled reference's, bit for bit (config-1 shape)."""
    d, _ = load_npz("ref_router.npz")
    x, W, bias = synth.router_inputs()
    T = x.shape[0]
    X, Wd, B = (k3cuda.DevBuf.from_array(a) for a in (x, W, bias))
    I = k3cuda.DevBuf(T * 8 * 4)
    Wt = k3cuda.DevBuf(T * 8 * 4)
    k3cuda.check(k3.k3d_router_bf16(I.ptr, Wt.ptr, X.ptr, Wd.ptr, B.ptr, T, 7168, 384, 8, 1, 2.5))
    k3cuda.check(k3.k3d_sync())
    assert np.array_equal(I.download(np.int32, (T, 8)), d["idx"])
    assert np.array_equal(Wt.download(np.float32, (T, 8)).view(np.uint32), d["w"].view(np.uint32))


def test_router_many_tokens_and_ties_bit_exact(k3, oracle):
    g = synth.rng(5)
    T, hidden, E = 64, 7168, 384
    x, W, bias = synth.router_inputs(seed=77, T=T, hidden=hidden, n_experts=E)
    bias[10:20] = bias[10]           # equal biases
    W[30] = W[31]                    # identical rows -> exactly tied scores
    bias[30] = bias[31]
    X, Wd, B = (k3cuda.DevBuf.from_array(a) for a in (x, W, bias))
    I = k3cuda.DevBuf(T * 8 * 4)
    Wt = k3cuda.DevBuf(T * 8 * 4)
    k3cuda.check(k3.k3d_router_bf16(I.ptr, Wt.ptr, X.ptr, Wd.ptr, B.ptr, T, hidden, E, 8, 1, 2.5))
    k3cuda.check(k3.k3d_sync())
    gi = I.download(np.int32, (T, 8))
    gw = Wt.download(np.float32, (T, 8))
    for t in range(T):
        oi, ow = oracle.router_bf16(x[t], W, bias, 8, 1, 2.5)
        assert np.array_equal(gi[t], oi), t
        assert np.array_equal(gw[t].view(np.uint32), ow.view(np.uint32)), t


def _midpoint_row(hidden, sign):
    """bf16 row whose dot with x = ones is exactly sign * (1 + 2^-24), a float rounding
    midpoint, reached through two cancelling 2^-60 terms: the fast pass cannot settle it,
    and the tight pass cannot either (the tiny terms may round), so only the sequential
    loop decides it."""
    r = np.zeros(hidden, np.float32)
    r[0], r[1], r[2], r[3] = 1.0, 2.0 ** -24, 2.0 ** -60, -(2.0 ** -60)
    return synth.f32_to_bf16(sign * r)


def _route(k3, x, W, bias, T, hidden, E):
    X, Wd, B = (k3cuda.DevBuf.from_array(a) for a in (x, W, bias))
    I = k3cuda.DevBuf(T * 8 * 4)
    Wt = k3cuda.DevBuf(T * 8 * 4)
    k3cuda.check(k3.k3d_router_bf16(I.ptr, Wt.ptr, X.ptr, Wd.ptr, B.ptr, T, hidden, E, 8, 1, 2.5))
    k3cuda.check(k3.k3d_sync())
    return I.download(np.int32, (T, 8)), Wt.download(np.float32, (T, 8))


def test_router_unsettled_experts_only_where_they_matter(k3, oracle):
    """Expert 7 (large bias) is selected and sits on a rounding midpoint: it must be settled
    by the exact path. Expert 9 is as ambiguous but far below the top 8: the selection is
    proven without it, so it costs no sequential loop. Bit-exact against the CPU either way."""
    T, hidden, E = 4, 7168, 384
    _, W, bias = synth.router_inputs(seed=91, T=T, hidden=hidden, n_experts=E)
    x = np.ones((T, hidden), np.float32)
    W[7] = _midpoint_row(hidden, 1.0)
    W[9] = _midpoint_row(hidden, -1.0)
    bias[7], bias[9] = 1.0, -1.0
    f0 = k3.k3d_router_fallbacks()
    gi, gw = _route(k3, x, W, bias, T, hidden, E)
    nfb = k3.k3d_router_fallbacks() - f0
    for t in range(T):
        oi, ow = oracle.router_bf16(x[t], W, bias, 8, 1, 2.5)
        assert np.array_equal(gi[t], oi), t
        assert np.array_equal(gw[t].view(np.uint32), ow.view(np.uint32)), t
        assert 7 in gi[t] and 9 not in gi[t]
    assert nfb == T, f"{nfb} sequential loops for {T} tokens: expert 9 should not need one"


def test_router_nine_tied_unsettled_experts(k3, oracle):
    """Nine identical ambiguous experts dominate the choice: the first selection round picks
    eight of them by their lower bounds, the ninth overlaps the eighth, so all nine are
    settled exactly, then the ties go to the lowest indices."""
    T, hidden, E = 2, 7168, 384
    _, W, bias = synth.router_inputs(seed=92, T=T, hidden=hidden, n_experts=E)
    x = np.ones((T, hidden), np.float32)
    for e in range(100, 109):
        W[e] = _midpoint_row(hidden, 1.0)
        bias[e] = 2.0
    f0 = k3.k3d_router_fallbacks()
    gi, gw = _route(k3, x, W, bias, T, hidden, E)
    assert k3.k3d_router_fallbacks() - f0 == 9 * T
    for t in range(T):
        oi, ow = oracle.router_bf16(x[t], W, bias, 8, 1, 2.5)
        assert np.array_equal(gi[t], oi), t
        assert np.array_equal(gw[t].view(np.uint32), ow.view(np.uint32)), t
        assert list(gi[t]) == list(range(100, 108))


@pytest.mark.parametrize("inp,out", [(7168, 4096), (2048, 7168), (100, 33), (7, 5)])
def test_gemv_bf16_and_f32(k3, oracle, inp, out):
    g = synth.rng(inp + out)
    W = g.standard_normal((out, inp), dtype=np.float32) * np.float32(0.02)
    Wb = synth.f32_to_bf16(W)
    x = g.standard_normal(inp, dtype=np.float32)
    y = np.empty(out, np.float32)
    k3.k3_matmul_bf16(y.ctypes.data, x.ctypes.data, Wb.ctypes.data, inp, out)
    assert max_rel_err(y, oracle.matmul_bf16(x, Wb)) <= 1e-5
    k3.k3_matmul(y.ctypes.data, x.ctypes.data, W.ctypes.data, inp, out)
    assert max_rel_err(y, oracle.matmul(x, W)) <= 1e-5


@pytest.mark.parametrize("inp,out", [(7168, 4096), (257, 129), (100, 33), (15, 7), (16, 1)])
def test_k3_matmul_bit_exact_with_cpu_engine(k3, oracle, reference, inp, out):
    """k3_matmul and k3_matmul_bf16 reproduce the CPU engine's sixteen double accumulators
    and reduction tree (k3_ops.c:265-291) bit for bit, tails included; the CPU side is the
    compiled reference and the oracle's restatement of it."""
    g = synth.rng(3 * inp + out)
    W = g.standard_normal((out, inp), dtype=np.float32) * np.float32(0.5)
    Wb = synth.f32_to_bf16(W)
    x = g.standard_normal(inp, dtype=np.float32)
    y = np.empty(out, np.float32)
    k3.k3_matmul(y.ctypes.data, x.ctypes.data, W.ctypes.data, inp, out)
    assert np.array_equal(y.view(np.uint32), reference.matmul(x, W).view(np.uint32))
    assert np.array_equal(y.view(np.uint32), oracle.matmul(x, W).view(np.uint32))
    yb = np.empty(out, np.float32)
    k3.k3_matmul_bf16(yb.ctypes.data, x.ctypes.data, Wb.ctypes.data, inp, out)
    assert np.array_equal(yb.view(np.uint32), reference.matmul_bf16(x, Wb).view(np.uint32))
    # the engine's own gate: the bf16 path equals the fp32 path on the widened weights
    Ww = np.ascontiguousarray(synth.bf16_to_f32(Wb))
    k3.k3_matmul(y.ctypes.data, x.ctypes.data, Ww.ctypes.data, inp, out)
    assert np.array_equal(y.view(np.uint32), yb.view(np.uint32))


def test_kda_step_fixture_and_bit_exact(k3, oracle):
    d, meta = load_npz("ref_ops/kda_recur8.npz")
    atol, rtol = manifest_tol()
    T, H, dk = d["q"].shape
    dv = d["v"].shape[2]
    S = np.zeros((H, dk, dv), np.float32)
    So = S.copy()
    outs = np.zeros((T, H, dv), np.float32)
    for t in range(T):
        for h in range(H):
            q = (d["q"][t, h] * np.float32(meta["q_scale"])).astype(np.float32)
            o = np.empty(dv, np.float32)
            Sh = np.ascontiguousarray(S[h])
            k3.k3_kda_step(Sh.ctypes.data, o.ctypes.data, q.ctypes.data,
                           np.ascontiguousarray(d["k"][t, h]).ctypes.data,
                           np.ascontiguousarray(d["v"][t, h]).ctypes.data,
                           np.ascontiguousarray(d["alpha"][t, h]).ctypes.data,
                           float(d["beta"][t, h]), dk, dv)
            S[h] = Sh
            outs[t, h] = o
            So[h], oo = oracle.kda_step(So[h], q, d["k"][t, h], d["v"][t, h], d["alpha"][t, h],
                                        d["beta"][t, h])
            assert np.array_equal(o, oo) and np.array_equal(S[h], So[h])
    assert_close_elementwise(outs, d["out"], atol, rtol, "kda out")


@pytest.mark.parametrize("B", [1, 2, 32])
def test_kda_decode_config3_bit_exact(k3, oracle, B):
    """Config 3 decode (batches 1 and 32 in BASELINE): every state and output bit-identical
    to the oracle's k3_kda_step."""
    g = synth.rng(21 + B)
    H, D = 64, 128
    S = (g.standard_normal((B, H, D, D), dtype=np.float32) * np.float32(0.01))
    q = g.standard_normal((B, H, D), dtype=np.float32)
    k = g.standard_normal((B, H, D), dtype=np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = g.standard_normal((B, H, D), dtype=np.float32)
    al = g.uniform(0.9, 1.0, (B, H, D)).astype(np.float32)
    be = g.uniform(0, 1, (B, H)).astype(np.float32)
    bufs = [k3cuda.DevBuf.from_array(a) for a in (S, q, k, v, al, be)]
    O = k3cuda.DevBuf(B * H * D * 4)
    k3cuda.check(k3.k3d_kda_decode(bufs[0].ptr, O.ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                   bufs[4].ptr, bufs[5].ptr, B, H, D, D))
    k3cuda.check(k3.k3d_sync())
    So, oo = oracle.kda_decode(S, q, k, v, al, be)
    assert np.array_equal(bufs[0].download(np.float32, S.shape), So)
    assert np.array_equal(O.download(np.float32, (B, H, D)), oo)


def test_kda_prefill_sequential_bit_exact(k3, oracle):
    g = synth.rng(22)
    T, H, D = 12, 8, 128
    S = g.standard_normal((H, D, D), dtype=np.float32) * np.float32(0.01)
    q, k, v = (g.standard_normal((T, H, D), dtype=np.float32) for _ in range(3))
    al = g.uniform(0.9, 1.0, (T, H, D)).astype(np.float32)
    be = g.uniform(0, 1, (T, H)).astype(np.float32)
    bufs = [k3cuda.DevBuf.from_array(a) for a in (S, q, k, v, al, be)]
    O = k3cuda.DevBuf(T * H * D * 4)
    k3cuda.check(k3.k3d_kda_prefill(bufs[0].ptr, O.ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                    bufs[4].ptr, bufs[5].ptr, T, H, D, D, 0))
    k3cuda.check(k3.k3d_sync())
    So = S.copy()
    oo = np.zeros((T, H, D), np.float32)
    for t in range(T):
        So2, o2 = oracle.kda_decode(So[None], q[t][None], k[t][None], v[t][None], al[t][None],
                                    be[t][None])
        So = So2[0]
        oo[t] = o2[0]
    assert np.array_equal(bufs[0].download(np.float32, S.shape), So)
    assert np.array_equal(O.download(np.float32, (T, H, D)), oo)


def test_small_ops_against_reference_fixtures(k3):
    atol, rtol = manifest_tol()
    d, meta = load_npz("ref_ops/rmsnorm.npz")
    n = d["weight"].size
    rows = d["in"].reshape(-1, n)
    got = np.empty_like(rows)
    for i, r in enumerate(rows):
        k3.k3_rmsnorm(got[i].ctypes.data, np.ascontiguousarray(r).ctypes.data,
                      d["weight"].ctypes.data, n, float(meta["eps"]))
    assert_close_elementwise(got, d["out"], atol, rtol, "rmsnorm")
    d, meta = load_npz("ref_ops/situ_glu.npz")
    x = d["in"]
    n = x.shape[1] // 2
    got = np.empty((x.shape[0], n), np.float32)
    for i in range(x.shape[0]):
        k3.k3_situ_glu(got[i].ctypes.data, np.ascontiguousarray(x[i]).ctypes.data, n,
                       meta["beta"], meta["linear_beta"])
    assert_close_elementwise(got, d["out"], atol, rtol, "situ_glu")
    d, meta = load_npz("ref_ops/kda_decay.npz")
    H, D = d["A_log"].size, d["dt_bias"].size // d["A_log"].size
    z = np.ascontiguousarray(d["z"].reshape(-1, H * D))
    for t in range(z.shape[0]):
        gg = np.empty(H * D, np.float32)
        al = np.empty(H * D, np.float32)
        k3.k3_kda_decay(gg.ctypes.data, al.ctypes.data, z[t].ctypes.data, d["A_log"].ctypes.data,
                        d["dt_bias"].ctypes.data, H, D, float(meta["lower_bound"]))
        assert_close_elementwise(gg, d["g"].reshape(-1, H * D)[t], atol, rtol, "decay g")
        assert_close_elementwise(al, d["alpha"].reshape(-1, H * D)[t], atol, rtol, "decay alpha")
    d, meta = load_npz("ref_ops/shortconv.npz")
    C_, K = int(meta["channels"]), int(meta["kernel"])
    x = np.ascontiguousarray(d["in"].reshape(-1, C_))
    T = x.shape[0]
    state = np.zeros(C_ * (K - 1), np.float32)
    y = np.empty((T, C_), np.float32)
    w = np.ascontiguousarray(d["weight"].reshape(C_, K))
    k3.k3_shortconv(y.ctypes.data, x.ctypes.data, w.ctypes.data, state.ctypes.data, C_, K, T)
    assert_close_elementwise(y, d["out"], atol, rtol, "shortconv")
    assert_close_elementwise(state, d["state_after"], atol, rtol, "shortconv state")
    xn = np.ascontiguousarray(d["in_next"].reshape(-1, C_))
    yn = np.empty_like(xn)
    k3.k3_shortconv(yn.ctypes.data, xn.ctypes.data, w.ctypes.data, state.ctypes.data, C_, K,
                    xn.shape[0])
    assert_close_elementwise(yn, d["out_next"], atol, rtol, "shortconv continuation")
    d, meta = load_npz("ref_ops/attnres.npz")
    n = d["proj_weight"].size
    fold = (d["norm_weight"] * d["proj_weight"]).astype(np.float32)
    nb = d["block_residual"].reshape(-1, n).shape[0] // d["prefix_sum"].reshape(-1, n).shape[0]
    br = d["block_residual"].reshape(d["prefix_sum"].reshape(-1, n).shape[0], -1, n)
    ps = d["prefix_sum"].reshape(-1, n)
    for t in range(ps.shape[0]):
        src = np.ascontiguousarray(np.concatenate([br[t], ps[t][None]], 0).astype(np.float32))
        out = np.empty(n, np.float32)
        k3.k3_attn_res(out.ctypes.data, src.ctypes.data, fold.ctypes.data, src.shape[0], n,
                       float(meta["eps"]))
        assert_close_elementwise(out, d["out"].reshape(-1, n)[t], atol, rtol, "attn_res")
