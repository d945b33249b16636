"""TEST INFRASTRUCTURE, NOT PRODUCT CODE.

ctypes access to the two CPU checkers built by oracle/Makefile:
  Oracle     liboracle.so, the C restatement in oracle/k3_oracle.c (always buildable);
  Reference  _ref/libk3ref.so, the reference engine's own k3_ops.c compiled from its
             sources (present only where the reference tree was available at build time).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this module.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libk3ref.so")

vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float


def build():
    """Compile the checkers (liboracle.so always; _ref only when the reference exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def ptr(a):
    return a.ctypes.data_as(vp) if a is not None else None


class K3ExpertQ(C.Structure):
    _fields_ = [("p1", vp), ("s1", vp), ("p3", vp), ("s3", vp), ("p2", vp), ("s2", vp)]


def _declare(lib, prefix):
    p = prefix
    protos = {
        p + "rmsnorm": [vp, vp, vp, i32, f32],
        p + "situ_glu": [vp, vp, i32, f32, f32],
        p + "shortconv": [vp, vp, vp, vp, i32, i32, i32],
        p + "kda_decay": [vp, vp, vp, vp, vp, i32, i32, f32],
        p + "kda_step": [vp, vp, vp, vp, vp, vp, f32, i32, i32],
        p + "matmul": [vp, vp, vp, i32, i32],
        p + "matmul_bf16": [vp, vp, vp, i32, i32],
        p + "router": [vp, vp, vp, vp, vp, i32, i32, i32, i32, f32],
        p + "attn_res": [vp, vp, vp, i32, i32, f32],
        p + "mxfp4_dequant": [vp, vp, vp, i32, i32, i32],
        p + "matmul_mxfp4": [vp, vp, vp, vp, i32, i32, i32],
    }
    for name, args in protos.items():
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = args


class _Common:
    prefix = ""

    def f(self, name):
        return getattr(self.lib, self.prefix + name)

    def matmul_mxfp4(self, x, packed, scales, rows, group=32):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        self.f("matmul_mxfp4")(ptr(y), ptr(x), ptr(packed), ptr(scales), x.size, rows, group)
        return y

    def mxfp4_dequant(self, packed, scales, rows, pcols, group=32):
        out = np.empty(rows * pcols * 2, np.float32)
        self.f("mxfp4_dequant")(ptr(out), ptr(packed), ptr(scales), rows, pcols, group)
        return out.reshape(rows, pcols * 2)

    def matmul(self, x, W):
        W = np.ascontiguousarray(W, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(W.shape[0], np.float32)
        self.f("matmul")(ptr(y), ptr(x), ptr(W), W.shape[1], W.shape[0])
        return y

    def matmul_bf16(self, x, Wb):
        Wb = np.ascontiguousarray(Wb, np.uint16)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(Wb.shape[0], np.float32)
        self.f("matmul_bf16")(ptr(y), ptr(x), ptr(Wb), Wb.shape[1], Wb.shape[0])
        return y

    def router(self, x, W, bias, topk, renorm, scale):
        W = np.ascontiguousarray(W, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        idx = np.empty(topk, np.int32)
        w = np.empty(topk, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.f("router")(ptr(idx), ptr(w), ptr(x), ptr(W), ptr(b), W.shape[1], W.shape[0],
                         topk, renorm, scale)
        return idx, w

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.f("rmsnorm")(ptr(y), ptr(x), ptr(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return y

    def situ_glu(self, x, n, b1, b2):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(n, np.float32)
        self.f("situ_glu")(ptr(y), ptr(x), n, b1, b2)
        return y

    def shortconv(self, x, w, state, channels, k):
        x = np.ascontiguousarray(x, np.float32)
        T = x.size // channels
        y = np.empty_like(x)
        self.f("shortconv")(ptr(y), ptr(x), ptr(np.ascontiguousarray(w, np.float32)), ptr(state),
                            channels, k, T)
        return y

    def kda_decay(self, z, A_log, dt_bias, H, D, lb):
        g = np.empty(H * D, np.float32)
        al = np.empty(H * D, np.float32)
        self.f("kda_decay")(ptr(g), ptr(al), ptr(np.ascontiguousarray(z, np.float32)),
                            ptr(np.ascontiguousarray(A_log, np.float32)),
                            ptr(np.ascontiguousarray(dt_bias, np.float32)), H, D, lb)
        return g, al

    def attn_res(self, src, fold, eps):
        src = np.ascontiguousarray(src, np.float32)
        out = np.empty(src.shape[1], np.float32)
        self.f("attn_res")(ptr(out), ptr(src), ptr(np.ascontiguousarray(fold, np.float32)),
                           src.shape[0], src.shape[1], eps)
        return out

    def kda_step(self, S, q, k, v, alpha, beta):
        S = np.ascontiguousarray(S, np.float32).copy()
        dk, dv = S.shape
        o = np.empty(dv, np.float32)
        self.f("kda_step")(ptr(S), ptr(o), ptr(np.ascontiguousarray(q, np.float32)),
                           ptr(np.ascontiguousarray(k, np.float32)),
                           ptr(np.ascontiguousarray(v, np.float32)),
                           ptr(np.ascontiguousarray(alpha, np.float32)), float(beta), dk, dv)
        return S, o


class Oracle(_Common):
    """The C restatement (liboracle.so)."""
    prefix = "orc_"

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build()
        self.lib = C.CDLL(ORACLE_SO)
        _declare(self.lib, "orc_")
        L = self.lib
        L.orc_expert_swiglu.argtypes = [vp, vp, C.POINTER(K3ExpertQ), i32, i32]
        L.orc_expert_swiglu.restype = None
        L.orc_router_bf16.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, f32]
        L.orc_router_bf16.restype = None
        L.orc_moe_swiglu.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, f32, vp, vp,
                                     C.POINTER(K3ExpertQ), i32, vp, vp, vp, i32, i32, i32, vp, vp]
        L.orc_moe_swiglu.restype = None
        L.orc_kda_decode.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]
        L.orc_kda_decode.restype = None
        for fn in (L.orc_mla_decode, L.orc_mla_decode_absorbed):
            fn.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, f32, f32,
                           vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32]
            fn.restype = None

    def expert_swiglu(self, x, e, hidden, inter):
        """e: dict with numpy arrays p1,s1,p3,s3,p2,s2."""
        q = K3ExpertQ(*(e[k].ctypes.data for k in ("p1", "s1", "p3", "s3", "p2", "s2")))
        y = np.empty(hidden, np.float32)
        self.lib.orc_expert_swiglu(ptr(y), ptr(np.ascontiguousarray(x, np.float32)), C.byref(q),
                                   hidden, inter)
        return y

    def router_bf16(self, x, Wb, bias, topk, renorm, scale):
        x = np.ascontiguousarray(x, np.float32)
        idx = np.empty(topk, np.int32)
        w = np.empty(topk, np.float32)
        self.lib.orc_router_bf16(ptr(idx), ptr(w), ptr(x), ptr(Wb), ptr(bias), Wb.shape[1],
                                 Wb.shape[0], topk, renorm, scale)
        return idx, w

    def moe_swiglu(self, x, T, hidden, inter, n_experts, topk, renorm, scale, router_w, bias,
                   experts, shared_inter, sh_gate, sh_up, sh_down, lo=0, hi=None, add_shared=1):
        """experts: list of dicts (numpy arrays) for every expert id."""
        hi = n_experts if hi is None else hi
        arr = (K3ExpertQ * n_experts)()
        for e, d in enumerate(experts):
            if d is None:
                continue
            arr[e] = K3ExpertQ(*(d[k].ctypes.data for k in ("p1", "s1", "p3", "s3", "p2", "s2")))
        out = np.empty((T, hidden), np.float32)
        idx = np.empty((T, topk), np.int32)
        w = np.empty((T, topk), np.float32)
        self.lib.orc_moe_swiglu(ptr(out), ptr(np.ascontiguousarray(x, np.float32)), T, hidden,
                                inter, n_experts, topk, renorm, scale, ptr(router_w), ptr(bias),
                                arr, shared_inter, ptr(sh_gate), ptr(sh_up), ptr(sh_down), lo,
                                hi, add_shared, ptr(idx), ptr(w))
        return out, idx, w

    def kda_decode(self, S, q, k, v, alpha, beta):
        S = np.ascontiguousarray(S, np.float32).copy()
        B, H, dk, dv = S.shape
        o = np.empty((B, H, dv), np.float32)
        self.lib.orc_kda_decode(ptr(S), ptr(o), ptr(q), ptr(k), ptr(v), ptr(alpha), ptr(beta),
                                B, H, dk, dv)
        return S, o


class Reference(_Common):
    """The reference engine's k3_ops.c, compiled from its sources (oracle/_ref)."""
    prefix = "k3_"

    @staticmethod
    def available():
        return os.path.exists(REF_SO)

    def __init__(self):
        if not self.available():
            raise FileNotFoundError(REF_SO)
        self.lib = C.CDLL(REF_SO)
        _declare(self.lib, "k3_")


def mla_decode(orc, x, dims, w, cache, pos, absorbed=False):
    """config-2 oracle: x [B][hidden]; dims dict; w dict of numpy weights (bf16 as uint16,
    norms fp32); cache [B][cap][kvw] uint16, updated in place at `pos`. absorbed=True takes
    the absorbed form (orc_mla_decode_absorbed: same attention, O(L) per head), which the
    CPU tests check against the expanded form; the expanded form is checked against the
    compiled reference's k3_mla_cached."""
    B = x.shape[0]
    out = np.empty((B, dims["hidden"]), np.float32)
    fn = orc.lib.orc_mla_decode_absorbed if absorbed else orc.lib.orc_mla_decode
    fn(ptr(out), ptr(np.ascontiguousarray(x, np.float32)), B, dims["hidden"],
                           dims["H"], dims["q_lora"], dims["kv_lora"], dims["qn"], dims["qr"],
                           dims["vh"], dims["theta"], dims["eps"], ptr(w["q_a"]), ptr(w["q_b"]),
                           ptr(w["kv_a"]), ptr(w["kv_b"]), ptr(w["o"]), ptr(w.get("g")),
                           ptr(w["q_a_norm"]), ptr(w["kv_a_norm"]), ptr(cache), cache.shape[1], pos)
    return out


# ------------------------------------------------------------- decode stack (config 4)
class K3Cfg(C.Structure):
    _fields_ = [
        ("hidden", i32), ("n_layers", i32), ("vocab", i32), ("rms_eps", f32),
        ("kda_heads", i32), ("kda_head_dim", i32), ("conv_k", i32), ("gate_lb", f32),
        ("n_heads", i32), ("q_lora", i32), ("kv_lora", i32), ("qk_nope", i32),
        ("qk_rope", i32), ("v_head", i32), ("mla_out_gate", i32),
        ("n_experts", i32), ("topk", i32), ("n_shared", i32), ("latent", i32),
        ("moe_inter", i32), ("routed_scale", f32), ("moe_renorm", i32), ("latent_norm", i32),
        ("first_dense", i32), ("dense_inter", i32), ("attn_res_block", i32),
        ("situ_b1", f32), ("situ_b2", f32), ("n_full_attn", i32), ("full_attn", C.POINTER(i32)),
    ]


class K3KdaW(C.Structure):
    _fields_ = [("q", vp), ("k", vp), ("v", vp), ("q_conv", vp), ("k_conv", vp),
                ("v_conv", vp), ("f_a", vp), ("f_b", vp), ("A_log", vp), ("dt_bias", vp),
                ("b", vp), ("g", vp), ("o_norm", vp), ("o", vp), ("wdt", i32)]


def kda_layer(orc, x, w, hidden, H, D, conv_k, gate_lb, eps, state):
    """k3_kda_layer (T = 1) with bf16 weights on host copies; state updated in place."""
    L = orc.lib
    L.orc_kda_layer.argtypes = [vp, vp, C.POINTER(K3KdaW), C.POINTER(K3Cfg), i32, vp, vp]
    L.orc_kda_layer.restype = None
    L.orc_kda_scratch.argtypes = [C.POINTER(K3Cfg), i32]
    L.orc_kda_scratch.restype = C.c_size_t
    cfg = K3Cfg(hidden=hidden, kda_heads=H, kda_head_dim=D, conv_k=conv_k, gate_lb=gate_lb,
                rms_eps=eps)
    kw = K3KdaW(*(w[k].ctypes.data for k in ("q", "k", "v", "q_conv", "k_conv", "v_conv", "f_a",
                                               "f_b", "A_log", "dt_bias", "b", "g", "o_norm", "o")),
                1)
    scratch = np.empty(L.orc_kda_scratch(C.byref(cfg), 1), np.float32)
    out = np.empty(hidden, np.float32)
    L.orc_kda_layer(ptr(out), ptr(np.ascontiguousarray(x, np.float32)), C.byref(kw), C.byref(cfg), 1,
                    ptr(state), ptr(scratch))
    return out


def silu_mul(g, u):
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u.astype(np.float32)


def stack_step(orc, cfg, W, S, token):
    """One decode step of the synthetic stack on host copies. cfg: dict (cfg["mla_absorbed"]
    selects the absorbed MLA form); W: weights by name (numpy; a layer's "moe.experts" is a
    list of expert dicts, or an object whose select(idx) returns such a list holding at least
    the experts idx names); S: mutable state {"pos", "layer<l>.kda.state",
    "layer<l>.mla.cache"}. Returns logits (float32 [vocab])."""
    E = cfg["hidden"]
    h = (W["embed"].reshape(cfg["vocab"], E)[token].astype(np.uint32) << 16).view(np.float32).copy()
    for l in range(cfg["n_layers"]):
        p = f"layer{l}."
        xn = orc.rmsnorm(h, W[p + "in_norm"], cfg["eps"])
        if l in cfg["mla_layers"]:
            m = cfg["mla"]
            w = {k: W[p + "mla." + k] for k in ("q_a", "q_b", "kv_a", "kv_b", "o", "g",
                                                 "q_a_norm", "kv_a_norm")}
            cache = S[p + "mla.cache"]
            out = mla_decode(orc, xn[None], m, w, cache, S["pos"],
                             absorbed=cfg.get("mla_absorbed", False))[0]
        else:
            w = {k: W[p + "kda." + k] for k in ("q", "k", "v", "q_conv", "k_conv", "v_conv", "f_a",
                                                 "f_b", "A_log", "dt_bias", "b", "g", "o_norm", "o")}
            out = kda_layer(orc, xn, w, E, cfg["kda_heads"], cfg["kda_head_dim"], cfg["conv_k"],
                            cfg["gate_lb"], cfg["eps"], S[p + "kda.state"])
        h = (h + out).astype(np.float32)
        xn = orc.rmsnorm(h, W[p + "post_norm"], cfg["eps"])
        if l < cfg["first_dense"]:
            a = silu_mul(orc.matmul_bf16(xn, W[p + "dense.gate"]), orc.matmul_bf16(xn, W[p + "dense.up"]))
            out = orc.matmul_bf16(a, W[p + "dense.down"])
        else:
            mo = cfg["moe"]
            experts = W[p + "moe.experts"]
            if hasattr(experts, "select"):
                # experts held on the device and fetched on demand: route first (the same
                # deterministic router the layer runs again), then fetch the selected ones
                idx, _ = orc.router_bf16(xn, W[p + "moe.router_w"], W[p + "moe.router_bias"],
                                         mo["topk"], 1, mo["routed_scale"])
                experts = experts.select(idx)
            out, _, _ = orc.moe_swiglu(xn[None], 1, E, mo["inter"], mo["n_experts"], mo["topk"], 1,
                                       mo["routed_scale"], W[p + "moe.router_w"],
                                       W[p + "moe.router_bias"], experts,
                                       mo["shared_inter"], W[p + "moe.sh_gate"], W[p + "moe.sh_up"],
                                       W[p + "moe.sh_down"])
            out = out[0]
        h = (h + out).astype(np.float32)
    xn = orc.rmsnorm(h, W["final_norm"], cfg["eps"])
    logits = orc.matmul_bf16(xn, W["lm_head"])
    S["pos"] += 1
    return logits


class K3MlaW(C.Structure):
    _fields_ = [("q_a", vp), ("q_b", vp), ("kv_a", vp), ("kv_b", vp), ("o", vp), ("g", vp),
                ("q_a_norm", vp), ("kv_a_norm", vp), ("wdt", i32)]


def ref_kda_layer_fn(lib):
    lib.k3_kda_layer.argtypes = [vp, vp, C.POINTER(K3KdaW), C.POINTER(K3Cfg), i32, vp, vp]
    lib.k3_kda_layer.restype = None
    lib.k3_kda_scratch.argtypes = [C.POINTER(K3Cfg), i32]
    lib.k3_kda_scratch.restype = C.c_size_t
    lib.k3_mla_cached.argtypes = [vp, vp, C.POINTER(K3MlaW), C.POINTER(K3Cfg), i32, vp, vp, vp, i32, i32]
    lib.k3_mla_cached.restype = None
    lib.k3_mla_scratch_cached.argtypes = [C.POINTER(K3Cfg), i32, i32, i32]
    lib.k3_mla_scratch_cached.restype = C.c_size_t
