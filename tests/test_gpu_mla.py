"""Config 2: MLA decode with absorbed weights over a bf16 latent cache, RoPE theta 50000,
against the oracle's expanded form (k3_mla_cached's arithmetic)."""
import ctypes

import numpy as np
import pytest

import k3cuda
from conftest import max_rel_err
import oracle as orc_mod
import synth

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=7168, H=64, q_lora=1536, kv_lora=512, qn=128, qr=64, vh=128,
            theta=50000.0, eps=1e-6)


def make(seed, d, B, cap, L):
    g = synth.rng(seed)
    qh, kvw, kvd = d["qn"] + d["qr"], d["kv_lora"] + d["qr"], d["qn"] + d["vh"]
    w = {
        "q_a": synth.bf16_normal(g, (d["q_lora"], d["hidden"]), 0.02),
        "q_b": synth.bf16_normal(g, (d["H"] * qh, d["q_lora"]), 0.02),
        "kv_a": synth.bf16_normal(g, (kvw, d["hidden"]), 0.02),
        "kv_b": synth.bf16_normal(g, (d["H"] * kvd, d["kv_lora"]), 0.02),
        "o": synth.bf16_normal(g, (d["hidden"], d["H"] * d["vh"]), 0.02),
        "g": synth.bf16_normal(g, (d["H"] * d["vh"], d["hidden"]), 0.02),
        "q_a_norm": (1.0 + 0.1 * g.standard_normal(d["q_lora"])).astype(np.float32),
        "kv_a_norm": (1.0 + 0.1 * g.standard_normal(d["kv_lora"])).astype(np.float32),
    }
    cache = np.zeros((B, cap, kvw), np.uint16)
    cache[:, :L] = synth.bf16_normal(g, (B, L, kvw), 1.0)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (B, d["hidden"]), 1.0))
    return w, cache, x


def run_gpu(k3, d, w, cache, x, pos, cap, accumulate=None):
    B = x.shape[0]
    shape = k3cuda.K3dMlaShape(d["hidden"], d["H"], d["q_lora"], d["kv_lora"], d["qn"], d["qr"],
                               d["vh"], d["theta"], d["eps"], 1)
    bufs = {k: k3cuda.DevBuf.from_array(v) for k, v in w.items()}
    mw = k3cuda.K3dMlaW(*(bufs[k].ptr for k in ("q_a", "q_b", "kv_a", "kv_b", "o", "g",
                                                 "q_a_norm", "kv_a_norm")))
    C = k3cuda.DevBuf.from_array(cache)
    X = k3cuda.DevBuf.from_array(x)
    O = k3cuda.DevBuf.from_array(accumulate if accumulate is not None else
                                 np.zeros((B, d["hidden"]), np.float32))
    P = k3cuda.DevBuf.from_array(np.array([pos], np.int32))
    n = k3.k3d_mla_ws_bytes(ctypes.byref(shape), B, cap)
    WS = k3cuda.DevBuf(n)
    k3cuda.check(k3.k3d_mla_decode(O.ptr, X.ptr, ctypes.byref(mw), ctypes.byref(shape), B, C.ptr,
                                   cap, P.ptr, 1 if accumulate is not None else 0, WS.ptr, n))
    k3cuda.check(k3.k3d_sync())
    return O.download(np.float32, (B, d["hidden"])), C.download(np.uint16, cache.shape)


@pytest.mark.parametrize("B,L", [(1, 200), (2, 37)])
def test_mla_decode_matches_oracle(k3, oracle, B, L):
    cap = 256
    w, cache, x = make(10 + B, DIMS, B, cap, L)
    y, cache_gpu = run_gpu(k3, DIMS, w, cache, x, L, cap)
    cache_cpu = cache.copy()
    want = orc_mod.mla_decode(oracle, x, DIMS, w, cache_cpu, L)
    # the new cache entry (normalised latent + rotated rope key, bf16) matches to rounding
    new_g = synth.bf16_to_f32(cache_gpu[:, L])
    new_c = synth.bf16_to_f32(cache_cpu[:, L])
    assert max_rel_err(new_g, new_c) <= 1e-2
    assert np.array_equal(cache_gpu[:, :L], cache[:, :L]), "earlier positions must be untouched"
    assert max_rel_err(y, want) <= 1e-3


def test_mla_decode_nope_small_dims_and_accumulate(k3, oracle):
    d = dict(hidden=256, H=8, q_lora=64, kv_lora=128, qn=32, qr=16, vh=32, theta=0.0, eps=1e-5)
    cap, L = 96, 70
    w, cache, x = make(3, d, 1, cap, L)
    resid = synth.rng(4).standard_normal((1, d["hidden"]), dtype=np.float32)
    y, _ = run_gpu(k3, d, w, cache, x, L, cap, accumulate=resid.copy())
    want = orc_mod.mla_decode(oracle, x, d, w, cache.copy(), L)
    assert max_rel_err(y - resid, want) <= 1e-3


def test_mla_decode_rejects_position_beyond_capacity(k3):
    d = dict(hidden=256, H=8, q_lora=64, kv_lora=128, qn=32, qr=16, vh=32, theta=0.0, eps=1e-5)
    cap = 16
    w, cache, x = make(5, d, 1, cap, 8)
    try:
        run_gpu(k3, d, w, cache, x, cap, cap)
    except k3cuda.K3Error:
        pass
    code, site = ctypes.c_int(), ctypes.c_int()
    k3.k3d_device_error(ctypes.byref(code), ctypes.byref(site))
    assert code.value == k3cuda.K3D_EBOUND
    k3.k3d_clear_status()
