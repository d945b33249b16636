"""Config 4 at reduced width: the 8-layer decode stack (KDA x6, MLA x2 at one-based layers 4
and 8, dense layer 0, MoE layers 1-7), graph-captured, against the oracle composed from the
reference routines, step by step from the same synthetic weights and context."""
import ctypes

import numpy as np
import pytest

import k3cuda
from conftest import max_rel_err
import oracle as orc_mod

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, vocab=1024, n_layers=8, eps=1e-6, kda_heads=4, kda_head_dim=64, conv_k=4,
           gate_lb=-5.0, first_dense=1, dense_inter=1024, mla_layers=[3, 7],
           mla=dict(hidden=512, H=8, q_lora=128, kv_lora=128, qn=32, qr=16, vh=32, theta=50000.0,
                    eps=1e-6),
           moe=dict(inter=512, n_experts=16, topk=4, routed_scale=2.5, shared_inter=256))


def make_cfg(c, batch=1, cap=64, layout=0):
    m, mo = c["mla"], c["moe"]
    sc = k3cuda.K3dStackCfg()
    sc.hidden, sc.vocab, sc.n_layers, sc.eps = c["hidden"], c["vocab"], c["n_layers"], c["eps"]
    sc.kda_heads, sc.kda_head_dim, sc.conv_k, sc.gate_lb = (c["kda_heads"], c["kda_head_dim"],
                                                            c["conv_k"], c["gate_lb"])
    sc.mla = k3cuda.K3dMlaShape(m["hidden"], m["H"], m["q_lora"], m["kv_lora"], m["qn"], m["qr"],
                                m["vh"], m["theta"], m["eps"], 1)
    sc.moe = k3cuda.K3dMoeShape(c["hidden"], mo["inter"], mo["n_experts"], mo["topk"], 1,
                                mo["routed_scale"], mo["shared_inter"], 0, mo["n_experts"], 1,
                                layout)
    sc.first_dense, sc.dense_inter = c["first_dense"], c["dense_inter"]
    for i in range(16):
        sc.mla_layers[i] = c["mla_layers"][i] if i < len(c["mla_layers"]) else -1
    sc.batch, sc.ctx_cap = batch, cap
    return sc


def download(k3, model, name, dtype, shape=None):
    n = ctypes.c_size_t()
    p = k3.k3d_model_tensor(model, name.encode(), ctypes.byref(n))
    assert p, name
    a = np.empty(n.value // np.dtype(dtype).itemsize, dtype)
    k3cuda.check(k3.k3d_download(a.ctypes.data, p, a.nbytes))
    return a.reshape(shape) if shape else a


def _untile(codes, sf, K, rows, gu):
    """Inverse of k3d_expert_pretile for one matrix pair: tiles of 128 rows x 512 elements
    (codes in the SWIZZLE_128B K-major image, scales as four 32x16-byte atoms), the block of
    (tile t, chunk c) at position c * ntiles + t."""
    nch = K // 512
    ntiles = rows // 64 if gu else rows // 128
    r = np.arange(128)[:, None]
    j = np.arange(16)[None, :]
    chunk_off = (j >> 3) * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + (((j & 7) ^ (r & 7)) << 4)
    byte_idx = (chunk_off[:, :, None] + np.arange(16)[None, None, :]).reshape(128, 256)
    rr = np.arange(128)[:, None]
    w = np.arange(4)[None, :]
    sf_off = (512 * w + 16 * (rr & 31) + 4 * (rr >> 5))[:, :, None] + np.arange(4)[None, None, :]
    sf_idx = sf_off.reshape(128, 16)
    out_c = np.zeros((ntiles * 128, K // 2), np.uint8)
    out_s = np.zeros((ntiles * 128, K // 32), np.uint8)
    for t in range(ntiles):
        for c in range(nch):
            blk = c * ntiles + t          # chunk-major blocks
            tile = codes[blk * 32768:(blk + 1) * 32768]
            out_c[t * 128:(t + 1) * 128, c * 256:(c + 1) * 256] = tile[byte_idx]
            atoms = sf[blk * 2048:(blk + 1) * 2048]
            out_s[t * 128:(t + 1) * 128, c * 16:(c + 1) * 16] = atoms[sf_idx]
    if not gu:
        return out_c, out_s
    # gate/up tiles hold 64 gate rows then the same 64 up rows
    oc = out_c.reshape(ntiles, 2, 64, K // 2)
    os_ = out_s.reshape(ntiles, 2, 64, K // 32)
    return (oc[:, 0].reshape(rows, K // 2), os_[:, 0].reshape(rows, K // 32),
            oc[:, 1].reshape(rows, K // 2), os_[:, 1].reshape(rows, K // 32))


def untile_expert(slot, hidden, inter):
    gu, gus = inter * hidden // 2, inter * hidden // 32
    sizes = [2 * gu, 2 * gus, gu, gus]
    offs, o = [], 0
    for s_ in sizes:
        offs.append(o)
        o += (s_ + 255) // 256 * 256
    parts = [slot[off:off + s_] for off, s_ in zip(offs, sizes)]
    p1, s1, p3, s3 = _untile(parts[0], parts[1], hidden, inter, True)
    p2, s2 = _untile(parts[2], parts[3], inter, hidden, False)
    return {k: np.ascontiguousarray(v).reshape(-1) for k, v in
            (("p1", p1), ("s1", s1), ("p3", p3), ("s3", s3), ("p2", p2), ("s2", s2))}


class DeviceExperts:
    """A layer's routed experts left on the device and downloaded on demand (a full-width
    layer holds 8.98 GB of them): select(idx) returns the oracle's expert list with the
    experts idx names filled in (un-tiled for the tiled layout) and None elsewhere."""

    def __init__(self, k3, model, name, hidden, inter, n_experts, slot, layout):
        n = ctypes.c_size_t()
        self.base = k3.k3d_model_tensor(model, name.encode(), ctypes.byref(n))
        assert self.base, name
        self.k3, self.hidden, self.inter, self.n, self.slot, self.layout = (
            k3, hidden, inter, n_experts, slot, layout)
        gu, gus = inter * hidden // 2, inter * hidden // 32
        self.sizes = [gu, gus, gu, gus, gu, gus]
        self.offs, o = [], 0
        for s_ in self.sizes:
            self.offs.append(o)
            o += (s_ + 255) // 256 * 256
        assert o == slot
        self.cache = {}

    def get(self, e):
        if e not in self.cache:
            raw = np.empty(self.slot, np.uint8)
            k3cuda.check(self.k3.k3d_download(raw.ctypes.data, self.base + e * self.slot, self.slot))
            if self.layout == 1:
                self.cache[e] = untile_expert(raw, self.hidden, self.inter)
            else:
                self.cache[e] = {k: np.ascontiguousarray(raw[off:off + s_]) for k, off, s_ in
                                 zip(("p1", "s1", "p3", "s3", "p2", "s2"), self.offs, self.sizes)}
        return self.cache[e]

    def select(self, idx):
        out = [None] * self.n
        for e in np.asarray(idx).ravel():
            out[int(e)] = self.get(int(e))
        return out


def host_copy(k3, model, c, layout=0, batch=1, cap=64, lazy_experts=False):
    E, P, D, H = c["hidden"], c["kda_heads"] * c["kda_head_dim"], c["kda_head_dim"], c["kda_heads"]
    m, mo = c["mla"], c["moe"]
    W, S = {}, {}
    W["embed"] = download(k3, model, "embed", np.uint16)
    W["lm_head"] = download(k3, model, "lm_head", np.uint16, (c["vocab"], E))
    W["final_norm"] = download(k3, model, "final_norm", np.float32)
    for l in range(c["n_layers"]):
        p = f"layer{l}."
        W[p + "in_norm"] = download(k3, model, p + "in_norm", np.float32)
        W[p + "post_norm"] = download(k3, model, p + "post_norm", np.float32)
        if l in c["mla_layers"]:
            qh, kvw, kvd = m["qn"] + m["qr"], m["kv_lora"] + m["qr"], m["qn"] + m["vh"]
            shapes = {"q_a": (m["q_lora"], E), "q_b": (m["H"] * qh, m["q_lora"]), "kv_a": (kvw, E),
                      "kv_b": (m["H"] * kvd, m["kv_lora"]), "o": (E, m["H"] * m["vh"]),
                      "g": (m["H"] * m["vh"], E)}
            for k, shp in shapes.items():
                W[p + "mla." + k] = download(k3, model, p + "mla." + k, np.uint16, shp)
            for k in ("q_a_norm", "kv_a_norm"):
                W[p + "mla." + k] = download(k3, model, p + "mla." + k, np.float32)
            S[p + "mla.cache"] = download(k3, model, p + "mla.cache", np.uint16, (batch, cap, kvw))
        else:
            shapes = {"q": (P, E), "k": (P, E), "v": (P, E), "g": (P, E), "b": (H, E), "f_a": (D, E),
                      "f_b": (P, D), "o": (E, P)}
            for k, shp in shapes.items():
                W[p + "kda." + k] = download(k3, model, p + "kda." + k, np.uint16, shp)
            for k in ("q_conv", "k_conv", "v_conv", "A_log", "dt_bias", "o_norm"):
                W[p + "kda." + k] = download(k3, model, p + "kda." + k, np.float32)
            S[p + "kda.state"] = download(k3, model, p + "kda.state", np.float32)
        if l < c["first_dense"]:
            W[p + "dense.gate"] = download(k3, model, p + "dense.gate", np.uint16, (c["dense_inter"], E))
            W[p + "dense.up"] = download(k3, model, p + "dense.up", np.uint16, (c["dense_inter"], E))
            W[p + "dense.down"] = download(k3, model, p + "dense.down", np.uint16, (E, c["dense_inter"]))
        else:
            W[p + "moe.router_w"] = download(k3, model, p + "moe.router_w", np.uint16,
                                             (mo["n_experts"], E))
            W[p + "moe.router_bias"] = download(k3, model, p + "moe.router_bias", np.float32)
            for k, shp in (("sh_gate", (mo["shared_inter"], E)), ("sh_up", (mo["shared_inter"], E)),
                           ("sh_down", (E, mo["shared_inter"]))):
                W[p + "moe." + k] = download(k3, model, p + "moe." + k, np.uint16, shp)
            gu, gus = mo["inter"] * E // 2, mo["inter"] * E // 32
            sizes = [gu, gus, gu, gus, gu, gus]
            offs, o = [], 0
            for s_ in sizes:
                offs.append(o)
                o += (s_ + 255) // 256 * 256
            if lazy_experts:
                W[p + "moe.experts"] = DeviceExperts(k3, model, p + "moe.pool", E, mo["inter"],
                                                     mo["n_experts"], o, layout)
                continue
            pool = download(k3, model, p + "moe.pool", np.uint8)
            experts = []
            for e in range(mo["n_experts"]):
                base = e * o
                if layout == 1:
                    experts.append(untile_expert(pool[base:base + o], E, mo["inter"]))
                    continue
                d = {}
                for key, off, s_ in zip(("p1", "s1", "p3", "s3", "p2", "s2"), offs, sizes):
                    d[key] = np.ascontiguousarray(pool[base + off: base + off + s_])
                experts.append(d)
            W[p + "moe.experts"] = experts
    S["pos"] = int(download(k3, model, "pos", np.int32)[0])
    return W, S


@pytest.mark.parametrize("layout", [0, 1])
def test_stack_decode_matches_oracle_eager_and_graph(k3, oracle, layout):
    """layout 0: checkpoint-layout experts (mma.sync / tcgen05 cp.async path); layout 1:
    tiled experts on the tcgen05 bulk-copy path (the oracle gets the un-tiled bytes)."""
    c = CFG
    model = k3.k3d_model_create(ctypes.byref(make_cfg(c, layout=layout)), 1234)
    assert model, k3.k3d_last_message()
    try:
        k3cuda.check(k3.k3d_model_fill_context(model, 5, 99))
        k3cuda.check(k3.k3d_sync())
        W, S = host_copy(k3, model, c, layout)
        assert S["pos"] == 5
        tok = 17
        for step in range(4):          # step 0 eager, step 1 captures the graph, 2-3 replay
            ids = np.array([tok], np.int32)
            nxt = np.zeros(1, np.int32)
            k3cuda.check(k3.k3d_model_step_host(model, ids.ctypes.data, nxt.ctypes.data), f"step {step}")
            got = download(k3, model, "logits", np.float32)
            want = orc_mod.stack_step(oracle, c, W, S, tok)
            err = max_rel_err(got, want)
            assert err <= 1e-3, (step, err)
            top2 = np.sort(want)[-2:]
            if top2[1] - top2[0] > 1e-3 * np.abs(want).max():
                assert nxt[0] == int(np.argmax(want)), step
            tok = int(nxt[0])
        assert int(download(k3, model, "pos", np.int32)[0]) == 9
    finally:
        k3.k3d_model_destroy(model)


def sequence_state(c, S, b, batch):
    """Sequence b's own caches and states (copies the oracle updates in place)."""
    out = {"pos": S["pos"]}
    for l in range(c["n_layers"]):
        p = f"layer{l}."
        if p + "mla.cache" in S:
            out[p + "mla.cache"] = S[p + "mla.cache"][b:b + 1].copy()
        else:
            st = S[p + "kda.state"]
            n = st.size // batch
            out[p + "kda.state"] = st[b * n:(b + 1) * n].copy()
    return out


@pytest.mark.parametrize("B", [6, 64])
def test_stack_batch_decode_matches_oracle_per_sequence(k3, oracle, B):
    """A batch of 6 sequences (above 4: every projection runs the tensor-core GEMM; 24
    expert assignments per MoE layer, the resident expert pass) and of 64 (256 assignments:
    the grouped expert pass), eager then graph-captured; each sequence's logits against the
    oracle stepping that sequence alone from its own cache and state."""
    c = CFG
    model = k3.k3d_model_create(ctypes.byref(make_cfg(c, batch=B, layout=1)), 4321)
    assert model, k3.k3d_last_message()
    try:
        k3cuda.check(k3.k3d_model_fill_context(model, 7, 55))
        k3cuda.check(k3.k3d_sync())
        W, S = host_copy(k3, model, c, 1, batch=B)
        seqs = [sequence_state(c, S, b, B) for b in range(B)]
        toks = (np.array([3, 17, 17, 500, 1023, 42], np.int32) if B == 6 else
                ((np.arange(B) * 37 + 5) % c["vocab"]).astype(np.int32))
        for step in range(3):          # eager, capture, replay
            nxt = np.zeros(B, np.int32)
            k3cuda.check(k3.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data), f"step {step}")
            got = download(k3, model, "logits", np.float32).reshape(B, c["vocab"])
            for b in range(B):
                want = orc_mod.stack_step(oracle, c, W, seqs[b], int(toks[b]))
                err = max_rel_err(got[b], want)
                assert err <= 1e-3, (step, b, err)
                top2 = np.sort(want)[-2:]
                if top2[1] - top2[0] > 1e-3 * np.abs(want).max():
                    assert nxt[b] == int(np.argmax(want)), (step, b)
            toks = nxt.copy()
    finally:
        k3.k3d_model_destroy(model)


@pytest.mark.parametrize("B", [6, 64])
def test_stack_mode_a_one_rank_matches_mode_r(k3, B):
    """Mode A (ep_tokens = 1: every MoE layer through k3d_moe_swiglu_a2a_dev, the dispatch
    planned on the device) on one rank steps like the replicated path: the same logits and
    tokens, eager, captured and replayed."""
    c = CFG
    models = []
    try:
        for ep_tokens in (0, 1):
            sc = make_cfg(c, batch=B, layout=1)
            sc.ep_tokens = ep_tokens
            m = k3.k3d_model_create(ctypes.byref(sc), 4321)
            assert m, k3.k3d_last_message()
            models.append(m)
            k3cuda.check(k3.k3d_model_fill_context(m, 7, 55))
        toks = ((np.arange(B) * 37 + 5) % c["vocab"]).astype(np.int32)
        for step in range(3):              # eager, capture, replay
            outs = []
            for m in models:
                nxt = np.zeros(B, np.int32)
                k3cuda.check(k3.k3d_model_step_host(m, toks.ctypes.data, nxt.ctypes.data), f"step {step}")
                outs.append((nxt, download(k3, m, "logits", np.float32).copy()))
            assert np.array_equal(outs[0][1], outs[1][1]), step
            assert np.array_equal(outs[0][0], outs[1][0]), step
            toks = outs[0][0].copy()
    finally:
        for m in models:
            k3.k3d_model_destroy(m)


def test_step_past_the_cache_is_refused(k3):
    """A step needs a free cache position: with the cache full the host step is refused with
    K3D_EBOUND before anything launches (eager and graph-captured steps alike), no device
    error is left behind, and refilling the context makes the model step again."""
    c = CFG
    model = k3.k3d_model_create(ctypes.byref(make_cfg(c, batch=1, cap=8, layout=1)), 99)
    assert model, k3.k3d_last_message()
    try:
        k3cuda.check(k3.k3d_model_fill_context(model, 5, 3))
        toks = np.array([11], np.int32)
        for step in range(3):          # eager, capture, replay: positions 5, 6, 7
            nxt = np.zeros(1, np.int32)
            k3cuda.check(k3.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data), f"step {step}")
            toks = nxt.copy()
        assert int(download(k3, model, "pos", np.int32)[0]) == 8
        nxt = np.zeros(1, np.int32)
        assert k3.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data) == k3cuda.K3D_EBOUND
        k3cuda.check(k3.k3d_sync())
        code, site = ctypes.c_int(), ctypes.c_int()
        k3cuda.check(k3.k3d_device_error(ctypes.byref(code), ctypes.byref(site)))
        assert code.value == 0
        assert int(download(k3, model, "pos", np.int32)[0]) == 8
        k3cuda.check(k3.k3d_model_fill_context(model, 5, 3))
        k3cuda.check(k3.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data))
    finally:
        k3.k3d_model_destroy(model)
