"""The KDA decode layer (k3d_kda_layer_decode: projections, per-head step, output
projection) on random bf16 weights: the default choice, the shared-tile head kernel
(k3d_set_kda_head_kernel(1)), the register-column kernel (2) and the cluster kernel (3) bit
for bit, output and state, over two steps (the conv history shifts); and against the
oracle's k3_kda_layer."""
import ctypes

import numpy as np
import pytest

import k3cuda
import synth
from conftest import max_rel_err
import oracle as orc_mod

pytestmark = pytest.mark.gpu


def make_layer(seed, hidden, H, D, K=4):
    g = synth.rng(seed)
    P = H * D
    w = {}
    for k, shp in (("q", (P, hidden)), ("k", (P, hidden)), ("v", (P, hidden)), ("g", (P, hidden)),
                   ("b", (H, hidden)), ("f_a", (D, hidden)), ("f_b", (P, D)), ("o", (hidden, P))):
        w[k] = synth.bf16_normal(g, shp, 1.0 / np.sqrt(shp[1]))
    for k in ("q_conv", "k_conv", "v_conv"):
        w[k] = (g.standard_normal((P, K)) * 0.5).astype(np.float32)
    w["A_log"] = (g.standard_normal(H) * 0.5).astype(np.float32)
    w["dt_bias"] = (g.standard_normal(P) * 0.1).astype(np.float32)
    w["o_norm"] = (1.0 + 0.1 * g.standard_normal(D)).astype(np.float32)
    return w


class DevLayer:
    def __init__(self, k3, w, hidden, H, D, K, B):
        self.k3 = k3
        self.bufs = {k: k3cuda.DevBuf.from_array(v, k3) for k, v in w.items()}
        self.W = k3cuda.K3dKdaW(**{k: self.bufs[k].ptr for k in w})
        self.shape = k3cuda.K3dKdaShape(hidden, H, D, K, -5.0, 1e-6)
        self.B = B
        self.ws_bytes = k3.k3d_kda_layer_ws_bytes(ctypes.byref(self.shape), B)
        self.ws = k3cuda.DevBuf(self.ws_bytes, k3)
        self.state_floats = k3.k3d_kda_state_floats(ctypes.byref(self.shape))

    def run(self, h, x, state):
        H_ = k3cuda.DevBuf.from_array(h, self.k3)
        X = k3cuda.DevBuf.from_array(x, self.k3)
        S = k3cuda.DevBuf.from_array(state, self.k3)
        k3cuda.check(self.k3.k3d_kda_layer_decode(H_.ptr, X.ptr, ctypes.byref(self.W),
                                                  ctypes.byref(self.shape), self.B, S.ptr,
                                                  self.ws.ptr, self.ws_bytes))
        k3cuda.check(self.k3.k3d_sync())
        return H_.download(np.float32, h.shape), S.download(np.float32, state.shape)


@pytest.mark.parametrize("H,D,B,hidden", [(64, 128, 1, 7168), (8, 128, 3, 1024), (4, 64, 2, 512),
                                          (4, 32, 1, 256)])
def test_register_head_matches_shared_tile_head(k3, H, D, B, hidden):
    K = 4
    w = make_layer(91 + D + B, hidden, H, D, K)
    L = DevLayer(k3, w, hidden, H, D, K, B)
    g = synth.rng(7 + H)
    state0 = (g.standard_normal((B, L.state_floats)) * 0.3).astype(np.float32)
    xs = [(g.standard_normal((B, hidden))).astype(np.float32) for _ in range(2)]
    h0 = g.standard_normal((B, hidden)).astype(np.float32)
    res = {}
    try:
        for kind in (1, 2, 3, 0):
            k3cuda.check(k3.k3d_set_kda_head_kernel(kind))
            h, st = h0.copy(), state0.copy()
            for x in xs:
                h, st = L.run(h, x, st)
            res[kind] = (h, st)
    finally:
        k3cuda.check(k3.k3d_set_kda_head_kernel(0))
    for kind in (0, 2, 3):
        assert np.array_equal(res[kind][1], res[1][1]), kind
        assert np.array_equal(res[kind][0], res[1][0]), kind
    assert not np.array_equal(res[0][1], state0)


def test_layer_matches_oracle(k3, oracle):
    hidden, H, D, K = 1024, 8, 128, 4
    w = make_layer(5, hidden, H, D, K)
    L = DevLayer(k3, w, hidden, H, D, K, 1)
    g = synth.rng(11)
    state = (g.standard_normal(L.state_floats) * 0.3).astype(np.float32)
    st_o = state.copy()
    h = np.zeros(hidden, np.float32)
    for step in range(2):
        x = g.standard_normal(hidden).astype(np.float32)
        hg, state = L.run(h, x, state)
        want = orc_mod.kda_layer(oracle, x, w, hidden, H, D, K, -5.0, 1e-6, st_o)
        assert max_rel_err(hg, want) <= 1e-4, step
        assert max_rel_err(state, st_o) <= 1e-4, step


def test_zero_keys_and_non_finite_state_agree_across_head_kernels(k3):
    """Keys and queries that are exactly zero (their conv weights zero) and infinite state
    entries: the register kernel's branch-free dot products must still agree bit for bit
    with the kernels that skip zero keys and queries. Head 0 has an infinite state entry in
    a row whose key and query are zero (finite output: the skipped products are 0 * inf),
    head 1 one in a row whose key alone is zero (its output is not finite)."""
    hidden, H, D, K, B = 1024, 8, 128, 4, 1
    w = make_layer(404, hidden, H, D, K)
    for h in range(H):
        for i in (3, 77):
            w["k_conv"][h * D + i] = 0.0
        for i in (5, 77):
            w["q_conv"][h * D + i] = 0.0
    L = DevLayer(k3, w, hidden, H, D, K, B)
    g = synth.rng(405)
    state0 = (g.standard_normal((B, L.state_floats)) * 0.3).astype(np.float32)
    state0[0, 0 * D * D + 77 * D + 5] = np.inf
    state0[0, 1 * D * D + 3 * D + 9] = -np.inf
    xs = [(g.standard_normal((B, hidden))).astype(np.float32) for _ in range(2)]
    h0 = g.standard_normal((B, hidden)).astype(np.float32)
    res = {}
    try:
        for kind in (1, 2, 3, 0):
            k3cuda.check(k3.k3d_set_kda_head_kernel(kind))
            h, st = h0.copy(), state0.copy()
            for x in xs:
                h, st = L.run(h, x, st)
            res[kind] = (h, st)
    finally:
        k3cuda.check(k3.k3d_set_kda_head_kernel(0))
    for kind in (0, 2, 3):
        assert np.array_equal(res[kind][1].view(np.uint32), res[1][1].view(np.uint32)), kind
        assert np.array_equal(res[kind][0].view(np.uint32), res[1][0].view(np.uint32)), kind
    st = res[1][1][0]
    assert np.isinf(st[77 * D + 5])                    # skipped row: the entry stays infinite
