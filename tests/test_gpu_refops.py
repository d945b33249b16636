"""The reference-semantics composites (k3_mla, k3_moe, k3_kda_layer, k3_decoder_layer)
against the reference's own fixtures, called the way tests/unit/test_ops.c:407-738 calls
the CPU engine: fp32 host weights, host activations, caller scratch.

Tolerance: the fixtures' own, |got - want| <= 1e-5 + 1e-4 |want| (MANIFEST.json, the
bound test_ops.c:52-66 applies), times FP32_SLACK. The CPU engine accumulates dot
products in fp64; the GPU path accumulates in fp32, which at these widths (<= 128)
adds at most a few 1e-7 relative error per dot.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import load_npz, manifest_tol

pytestmark = pytest.mark.gpu

FP32_SLACK = 2.0


def _check(got, want, what):
    atol, rtol = manifest_tol()
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape, what
    ratio = np.abs(got - want) / (atol + rtol * np.abs(want))
    i = int(np.argmax(ratio))
    assert ratio[i] <= FP32_SLACK, (f"{what}: worst {ratio[i]:.2f}x tol at {i}: "
                                    f"got {got[i]:.7g} want {want[i]:.7g}")


def _f(a):
    return np.ascontiguousarray(a, np.float32)


class _Keep:
    """Holds the numpy arrays a ctypes struct points into."""

    def __init__(self):
        self.arrs = []

    def __call__(self, a):
        a = _f(a)
        self.arrs.append(a)
        return a.ctypes.data


def _mla_w(k3cuda, d, keep, prefix=""):
    w = k3cuda.K3MlaW()
    w.q_a = keep(d[prefix + "q_a_proj_weight"])
    w.q_a_norm = keep(d[prefix + "q_a_layernorm_weight"])
    w.q_b = keep(d[prefix + "q_b_proj_weight"])
    w.kv_a = keep(d[prefix + "kv_a_proj_with_mqa_weight"])
    w.kv_a_norm = keep(d[prefix + "kv_a_layernorm_weight"])
    w.kv_b = keep(d[prefix + "kv_b_proj_weight"])
    w.o = keep(d[prefix + "o_proj_weight"])
    w.g = keep(d[prefix + "g_proj_weight"])
    w.wdt = 0
    return w


def _moe_w(k3cuda, d, keep, n_experts, prefix=""):
    w = k3cuda.K3MoeW()
    w.gate = keep(d[prefix + "gate_weight"])
    w.bias = keep(d[prefix + "e_score_correction_bias"])
    w.down = keep(d[prefix + "down_weight"])
    w.up = keep(d[prefix + "up_weight"])
    w.latent_norm = keep(d[prefix + "norm_weight"])
    w.sh1 = keep(d[prefix + "shared_w1_weight"])
    w.sh3 = keep(d[prefix + "shared_w3_weight"])
    w.sh2 = keep(d[prefix + "shared_w2_weight"])
    for k in ("w1", "w3", "w2"):
        packed = np.stack([d[f"{prefix}experts_{e}_{k}_weight"] for e in range(n_experts)])
        setattr(w, k, keep(packed))
    w.wdt = 0
    return w


def _kda_w(k3cuda, d, keep, names):
    w = k3cuda.K3KdaW()
    for field, key in names.items():
        setattr(w, field, keep(d[key]))
    w.wdt = 0
    return w


KDA_NAMES = {"q": "q_proj", "k": "k_proj", "v": "v_proj", "q_conv": "q_conv", "k_conv": "k_conv",
             "v_conv": "v_conv", "f_a": "f_a", "f_b": "f_b", "A_log": "A_log",
             "dt_bias": "dt_bias", "b": "b_proj", "g": "g_proj", "o_norm": "o_norm",
             "o": "o_proj"}
LAYER_KDA_NAMES = {"q": "self_attn_q_proj_weight", "k": "self_attn_k_proj_weight",
                   "v": "self_attn_v_proj_weight", "q_conv": "self_attn_q_conv1d_weight",
                   "k_conv": "self_attn_k_conv1d_weight", "v_conv": "self_attn_v_conv1d_weight",
                   "f_a": "self_attn_f_a_proj_weight", "f_b": "self_attn_f_b_proj_weight",
                   "A_log": "self_attn_A_log", "dt_bias": "self_attn_dt_bias",
                   "b": "self_attn_b_proj_weight", "g": "self_attn_g_proj_weight",
                   "o_norm": "self_attn_o_norm_weight", "o": "self_attn_o_proj_weight"}


def test_mla_fixture(k3):
    """test_ops.c:407-459: k3_mla over T = 6 tokens, causal, RoPE on the rope slice."""
    import k3cuda
    d, meta = load_npz("ref_ops/mla.npz")
    keep = _Keep()
    c = k3cuda.K3Cfg()
    for k in ("qk_nope", "qk_rope", "kv_lora", "q_lora", "v_head", "n_heads"):
        setattr(c, k, int(meta[k]))
    c.rms_eps = meta.get("rms_eps", 1e-5)
    T, c.hidden = d["in"].shape[1], d["in"].shape[2]
    w = _mla_w(k3cuda, d, keep)
    sc = np.zeros(k3.k3_mla_scratch(C.byref(c), T), np.float32)
    x = _f(d["in"][0])
    y = np.full((T, c.hidden), np.nan, np.float32)
    k3.k3_mla(y.ctypes.data, x.ctypes.data, C.byref(w), C.byref(c), T, sc.ctypes.data)
    _check(y, d["out"][0], "mla")


def test_moe_fixture(k3):
    """test_ops.c:465-546: LatentMoE, SiTU into its caps, a bias that reorders top-k."""
    import k3cuda
    d, meta = load_npz("ref_ops/moe.npz")
    keep = _Keep()
    c = k3cuda.K3Cfg()
    c.hidden, c.latent, c.moe_inter = meta["hidden"], meta["latent"], meta["moe_inter"]
    c.n_experts, c.topk, c.n_shared = meta["n_experts"], meta["top_k"], meta["n_shared"]
    c.routed_scale, c.moe_renorm = meta["routed_scale"], meta["renorm"]
    c.latent_norm, c.rms_eps = meta["latent_norm"], meta["rms_eps"]
    c.situ_b1, c.situ_b2 = meta["situ_b1"], meta["situ_b2"]
    w = _moe_w(k3cuda, d, keep, c.n_experts)
    T = d["in"].shape[1]
    idx = np.zeros(c.topk, np.int32)
    wt = np.zeros(c.topk, np.float32)
    sc = np.zeros(k3.k3_moe_scratch(C.byref(c)), np.float32)
    y = np.full((T, c.hidden), np.nan, np.float32)
    x = _f(d["in"][0])
    k3.k3_moe(y.ctypes.data, x.ctypes.data, C.byref(w), C.byref(c), T, idx.ctypes.data,
              wt.ctypes.data, sc.ctypes.data)
    _check(y, d["out"][0], "moe")
    # the same layer through the prefill entry point gives the same rows
    y2 = np.full_like(y, np.nan)
    k3.k3_moe_prefill(y2.ctypes.data, x.ctypes.data, C.byref(w), C.byref(c), T,
                      idx.ctypes.data, wt.ctypes.data, sc.ctypes.data)
    np.testing.assert_array_equal(y2, y)


@pytest.mark.parametrize("name", ["kda_layer1", "kda_layer8"])
def test_kda_layer_fixture(k3, name):
    """test_ops.c:552-613: the full KDA layer at T = 1 and T = 8, output and state."""
    import k3cuda
    d, meta = load_npz(f"ref_ops/{name}.npz")
    keep = _Keep()
    c = k3cuda.K3Cfg()
    c.kda_heads, c.kda_head_dim = meta["H"], meta["d_k"]
    c.conv_k, c.gate_lb, c.rms_eps = meta["conv_k"], meta["lower_bound"], meta["rms_eps"]
    T, c.hidden = d["in"].shape[1], d["in"].shape[2]
    w = _kda_w(k3cuda, d, keep, KDA_NAMES)
    P = c.kda_heads * c.kda_head_dim
    st = np.zeros(P * c.kda_head_dim + 3 * P * (c.conv_k - 1), np.float32)
    sc = np.zeros(k3.k3_kda_scratch(C.byref(c), T), np.float32)
    y = np.full((T, c.hidden), np.nan, np.float32)
    k3.k3_kda_layer(y.ctypes.data, _f(d["in"][0]).ctypes.data, C.byref(w), C.byref(c), T,
                    st.ctypes.data, sc.ctypes.data)
    _check(y, d["out"][0], f"{name} out")
    _check(st[:P * c.kda_head_dim], d["state_out"], f"{name} state")


@pytest.mark.parametrize("name", ["layer_kda", "layer_mla"])
def test_decoder_layer_fixture(k3, name):
    """test_ops.c:627-738: AttnRes wiring + attention + MoE for one layer. layer_kda is
    index 1 (no block boundary), layer_mla index 3 (a boundary: a snapshot is pushed)."""
    import k3cuda
    d, meta = load_npz(f"ref_ops/{name}.npz")
    keep = _Keep()
    li, is_mla = meta["layer_idx"], meta["is_mla"]
    c = k3cuda.K3Cfg()
    c.hidden, c.rms_eps, c.attn_res_block = meta["hidden"], meta["rms_eps"], meta["attn_res_block_size"]
    c.n_layers = 13
    c.kda_heads, c.kda_head_dim, c.conv_k, c.gate_lb = 4, 16, 4, -5.0
    c.n_heads, c.q_lora, c.kv_lora, c.qk_nope, c.qk_rope, c.v_head = 4, 64, 32, 24, 8, 16
    c.n_experts, c.topk, c.n_shared, c.latent, c.moe_inter = 8, 2, 2, 64, 48
    c.routed_scale, c.moe_renorm, c.latent_norm = 1.0, 1, 1
    c.situ_b1, c.situ_b2 = 4.0, 25.0
    c.first_dense, c.dense_inter = 1, 96
    # the layer kind comes from which attention weights are set (k3_ops.c:1016-1017)

    lw = k3cuda.K3LayerW()
    lw.in_norm = keep(d["input_layernorm_weight"])
    lw.post_norm = keep(d["post_attention_layernorm_weight"])
    lw.attn_res_norm = keep(d["self_attention_res_norm_weight"])
    lw.attn_res_proj = keep(d["self_attention_res_proj_weight"])
    lw.mlp_res_norm = keep(d["mlp_res_norm_weight"])
    lw.mlp_res_proj = keep(d["mlp_res_proj_weight"])
    if is_mla:
        mw = _mla_w(k3cuda, d, keep, "self_attn_")
        lw.mla = C.pointer(mw)
    else:
        kw = _kda_w(k3cuda, d, keep, LAYER_KDA_NAMES)
        lw.kda = C.pointer(kw)
    ow = _moe_w(k3cuda, d, keep, c.n_experts, "mlp_")
    lw.moe = C.pointer(ow)
    lw.wdt = 0

    T = d["in"].shape[1]
    bri = d["block_residual_in"]
    nb_in = bri.shape[1]
    maxb = c.n_layers // c.attn_res_block + 2
    h = _f(d["in"][0]).copy()
    br = np.zeros((T, maxb, c.hidden), np.float32)
    br[:, :nb_in] = bri
    P = c.kda_heads * c.kda_head_dim
    st = np.zeros(P * c.kda_head_dim + 3 * P * (c.conv_k - 1), np.float32)
    sc = np.zeros(k3.k3_layer_scratch(C.byref(c), T), np.float32)
    nb = C.c_int(nb_in)
    k3.k3_decoder_layer(h.ctypes.data, br.ctypes.data, C.byref(nb), C.byref(lw), C.byref(c), li,
                        T, st.ctypes.data, sc.ctypes.data)
    _check(h, d["out"][0], name)
    bro = d["block_residual_out"]
    assert nb.value == bro.shape[1]
    _check(br[:, :nb.value], bro, f"{name} block residual")
