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
