"""The oracle pinned against the reference's own golden vectors and against the compiled
reference (CPU only)."""
import numpy as np
import pytest

from conftest import assert_close_elementwise, load_npz, manifest_tol
import synth


def test_mxfp4_dequant_exact_on_checkpoint_bytes(oracle):
    d, meta = load_npz("mxfp4.npz")
    rows, pcols = d["packed"].shape
    out = oracle.mxfp4_dequant(d["packed"], d["scales"], rows, pcols, 32)
    assert np.array_equal(out.view(np.uint32), d["expected"].reshape(rows, -1).view(np.uint32))
    # decoding the high nibble first gives the fixture's recorded wrong answer instead
    sw = ((d["packed"] >> 4) | (d["packed"] << 4)).astype(np.uint8)
    bad = oracle.mxfp4_dequant(sw, d["scales"], rows, pcols, 32)
    assert np.array_equal(bad.ravel()[:64], d["expected_swapped_nibbles"])
    assert not np.array_equal(bad, out)


def test_rmsnorm(oracle):
    d, meta = load_npz("ref_ops/rmsnorm.npz")
    atol, rtol = manifest_tol()
    n = d["weight"].size
    x = d["in"].reshape(-1, n)
    got = np.stack([oracle.rmsnorm(r, d["weight"], meta["eps"]) for r in x])
    assert_close_elementwise(got, d["out"], atol, rtol, "rmsnorm")


def test_situ_glu(oracle):
    d, meta = load_npz("ref_ops/situ_glu.npz")
    atol, rtol = manifest_tol()
    x = d["in"]
    n = x.shape[1] // 2
    got = np.stack([oracle.situ_glu(r, n, meta["beta"], meta["linear_beta"]) for r in x])
    assert_close_elementwise(got, d["out"], atol, rtol, "situ_glu")
    assert np.abs(got).max() <= 100.0


def test_kda_recurrence_T8(oracle):
    d, meta = load_npz("ref_ops/kda_recur8.npz")
    atol, rtol = manifest_tol()
    T, H, dk = d["q"].shape
    dv = d["v"].shape[2]
    S = np.zeros((H, dk, dv), np.float32)
    outs = np.zeros((T, H, dv), np.float32)
    for t in range(T):
        for h in range(H):
            q = d["q"][t, h] * np.float32(meta["q_scale"])
            S[h], outs[t, h] = oracle.kda_step(S[h], q, d["k"][t, h], d["v"][t, h],
                                               d["alpha"][t, h], d["beta"][t, h])
    assert_close_elementwise(outs, d["out"], atol, rtol, "kda out")
    assert_close_elementwise(S, d["state_out"], atol, rtol, "kda state")


def test_router_fixture(oracle):
    d, meta = load_npz("ref_ops/router.npz")
    atol, rtol = manifest_tol()
    W = d["gate_weight"]
    x = d["in"]
    k = int(meta["top_k"])
    for t in range(x.shape[0]):
        idx, w = oracle.router(x[t], W, d["bias"], k, 1, 1.0)
        want_idx = d["topk_idx"][t].astype(np.int32)
        # the fixture stores the selected set in descending biased-score order
        assert list(idx) == list(want_idx), (t, idx, want_idx)
        assert_close_elementwise(w, d["topk_weight"][t], atol, rtol, "router weights")


def test_oracle_matches_compiled_reference(oracle, reference):
    g = synth.rng(7)
    # fp32 / bf16 GEMV: same accumulator partition and tree -> identical bits
    W = g.standard_normal((96, 7168), dtype=np.float32)
    x = g.standard_normal(7168, dtype=np.float32)
    assert np.array_equal(oracle.matmul(x, W), reference.matmul(x, W))
    Wb = synth.f32_to_bf16(W)
    assert np.array_equal(oracle.matmul_bf16(x, Wb), reference.matmul_bf16(x, Wb))
    assert np.array_equal(oracle.matmul_bf16(x, Wb), reference.matmul(x, synth.bf16_to_f32(Wb)))
    # MXFP4: the reference's AVX2 flat path reassociates exact products (k3_ops.c:1364-1378)
    p, s = synth.mxfp4_matrix(g, 64, 7168)
    a = oracle.matmul_mxfp4(x, p, s, 64)
    b = reference.matmul_mxfp4(x, p, s, 64)
    assert np.abs(a.astype(np.float64) - b).max() <= 1e-6 * np.abs(b).max()
    # router: sequential double dot, float sigmoid -> identical indices and weights
    x2, Wr, bias = synth.router_inputs(seed=99, T=2, hidden=1024, n_experts=64)
    Wf = synth.bf16_to_f32(Wr)
    for t in range(2):
        i1, w1 = oracle.router(x2[t], Wf, bias, 8, 1, 2.5)
        i2, w2 = reference.router(x2[t], Wf, bias, 8, 1, 2.5)
        assert np.array_equal(i1, i2) and np.array_equal(w1.view(np.uint32), w2.view(np.uint32))
    # KDA step: same order of float operations
    S = g.standard_normal((128, 128), dtype=np.float32) * np.float32(0.01)
    q, k, v = (g.standard_normal(128, dtype=np.float32) for _ in range(3))
    al = g.uniform(0.9, 1.0, 128).astype(np.float32)
    S1, o1 = oracle.kda_step(S, q, k, v, al, 0.5)
    S2, o2 = reference.kda_step(S, q, k, v, al, 0.5)
    assert np.array_equal(S1, S2) and np.array_equal(o1, o2)


def test_config0_golden(oracle):
    d, _ = load_npz("ref_config0.npz")
    x, e = synth.config0_inputs()
    assert synth.digest(x, *e.values()) == bytes(d["digest"]).decode(), "synthetic input drift"
    y = oracle.expert_swiglu(x, e, 7168, 2048)
    rel = np.abs(y.astype(np.float64) - d["y"]).max() / np.abs(d["y"]).max()
    assert rel <= 1e-5, rel


def test_router_golden(oracle):
    d, _ = load_npz("ref_router.npz")
    x, W, bias = synth.router_inputs()
    assert synth.digest(x, W, bias) == bytes(d["digest"]).decode()
    for t in range(x.shape[0]):
        idx, w = oracle.router_bf16(x[t], W, bias, 8, 1, 2.5)
        assert np.array_equal(idx, d["idx"][t])
        assert np.array_equal(w.view(np.uint32), d["w"][t].view(np.uint32))


def test_decay_shortconv_attnres(oracle):
    atol, rtol = manifest_tol()
    d, meta = load_npz("ref_ops/kda_decay.npz")
    H, D = d["A_log"].size, d["dt_bias"].size // d["A_log"].size
    z = d["z"].reshape(-1, H * D)
    for t in range(z.shape[0]):
        g, al = oracle.kda_decay(z[t], d["A_log"], d["dt_bias"], H, D, float(meta["lower_bound"]))
        assert_close_elementwise(g, d["g"].reshape(-1, H * D)[t], atol, rtol, "decay g")
        assert_close_elementwise(al, d["alpha"].reshape(-1, H * D)[t], atol, rtol, "decay alpha")
    d, meta = load_npz("ref_ops/shortconv.npz")
    C_, K = int(meta["channels"]), int(meta["kernel"])
    state = np.zeros(C_ * (K - 1), np.float32)
    w = d["weight"].reshape(C_, K)
    y = oracle.shortconv(d["in"].reshape(-1, C_), w, state, C_, K)
    assert_close_elementwise(y, d["out"], atol, rtol, "shortconv")
    assert_close_elementwise(state, d["state_after"], atol, rtol, "shortconv state")
    yn = oracle.shortconv(d["in_next"].reshape(-1, C_), w, state, C_, K)
    assert_close_elementwise(yn, d["out_next"], atol, rtol, "shortconv continuation")
    d, meta = load_npz("ref_ops/attnres.npz")
    n = d["proj_weight"].size
    ps = d["prefix_sum"].reshape(-1, n)
    br = d["block_residual"].reshape(ps.shape[0], -1, n)
    fold = (d["norm_weight"] * d["proj_weight"]).astype(np.float32)
    for t in range(ps.shape[0]):
        src = np.concatenate([br[t], ps[t][None]], 0)
        assert src.shape[0] == int(meta["n_sources"])
        out = oracle.attn_res(src, fold, float(meta["eps"]))
        assert_close_elementwise(out, d["out"].reshape(-1, n)[t], atol, rtol, "attn_res")
