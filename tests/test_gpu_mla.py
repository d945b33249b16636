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


# B = 32 is config 2's batched decode (128 attention CTAs of one or two position splits)
@pytest.mark.parametrize("B,L", [(1, 200), (2, 37), (32, 64)])
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


# config 2 at its own sizes: L = 4096 at B = 1 (the stack's context; 37 position splits
# and the merge) and at B = 32, and L = 32768 at B = 1; against the absorbed-form oracle
# (pinned to the expanded form and, through it, to the reference's k3_mla_cached)
@pytest.mark.parametrize("B,L", [(1, 4096), (32, 4096), (1, 32768)])
def test_mla_decode_config2_sizes_match_oracle(k3, oracle, B, L):
    cap = L + 8
    w, cache, x = make(20 + B + L, DIMS, B, cap, L)
    y, cache_gpu = run_gpu(k3, DIMS, w, cache, x, L, cap)
    cache_cpu = cache.copy()
    want = orc_mod.mla_decode(oracle, x, DIMS, w, cache_cpu, L, absorbed=True)
    new_g = synth.bf16_to_f32(cache_gpu[:, L])
    new_c = synth.bf16_to_f32(cache_cpu[:, L])
    assert max_rel_err(new_g, new_c) <= 1e-2
    assert np.array_equal(cache_gpu[:, :L], cache[:, :L]), "earlier positions must be untouched"
    for b in range(B):
        assert max_rel_err(y[b], want[b]) <= 1e-3, b


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


def test_mla_decode_normed_matches_separate_norm(k3):
    """k3d_mla_decode_normed on the raw residual (the input RMSNorm applied inside the
    projection GEMV's load) equals k3d_rmsnorm followed by k3d_mla_decode, to within the
    rounding of the sum of squares (a different reduction order)."""
    d, B, cap, L = DIMS, 1, 256, 100
    w, cache, _ = make(7, d, B, cap, L)
    g = synth.rng(8)
    h = (g.standard_normal((B, d["hidden"])) * 3.0).astype(np.float32)
    nw = (1.0 + 0.1 * g.standard_normal(d["hidden"])).astype(np.float32)
    eps = 1e-6
    H, NW = k3cuda.DevBuf.from_array(h), k3cuda.DevBuf.from_array(nw)
    XN = k3cuda.DevBuf(h.nbytes)
    k3cuda.check(k3.k3d_rmsnorm(XN.ptr, H.ptr, NW.ptr, d["hidden"], B, eps))
    k3cuda.check(k3.k3d_sync())
    xn = XN.download(np.float32, (B, d["hidden"]))
    want, want_cache = run_gpu(k3, d, w, cache, xn, L, cap)

    shape = k3cuda.K3dMlaShape(d["hidden"], d["H"], d["q_lora"], d["kv_lora"], d["qn"], d["qr"],
                               d["vh"], d["theta"], d["eps"], 1)
    bufs = {k: k3cuda.DevBuf.from_array(v) for k, v in w.items()}
    mw = k3cuda.K3dMlaW(*(bufs[k].ptr for k in ("q_a", "q_b", "kv_a", "kv_b", "o", "g",
                                                 "q_a_norm", "kv_a_norm")))
    C = k3cuda.DevBuf.from_array(cache)
    O = k3cuda.DevBuf.from_array(np.zeros((B, d["hidden"]), np.float32))
    P = k3cuda.DevBuf.from_array(np.array([L], np.int32))
    n = k3.k3d_mla_ws_bytes(ctypes.byref(shape), B, cap)
    WS = k3cuda.DevBuf(n)
    k3cuda.check(k3.k3d_mla_decode_normed(O.ptr, H.ptr, NW.ptr, eps, ctypes.byref(mw),
                                          ctypes.byref(shape), B, C.ptr, cap, P.ptr, 0, WS.ptr, n))
    k3cuda.check(k3.k3d_sync())
    got = O.download(np.float32, (B, d["hidden"]))
    assert max_rel_err(got, want) <= 1e-5
    got_cache = C.download(np.uint16, cache.shape)
    assert np.array_equal(got_cache[:, :L], want_cache[:, :L])


def test_lm_head_normed_matches_separate_norm(k3):
    g = synth.rng(9)
    hidden, vocab = 7168, 16384
    W = synth.bf16_normal(g, (vocab, hidden), 0.02)
    h = (g.standard_normal((1, hidden)) * 2.0).astype(np.float32)
    nw = (1.0 + 0.1 * g.standard_normal(hidden)).astype(np.float32)
    Wd, H, NW = (k3cuda.DevBuf.from_array(a) for a in (W, h, nw))
    XN = k3cuda.DevBuf(h.nbytes)
    key = k3cuda.DevBuf(64)
    L1, L2 = k3cuda.DevBuf(vocab * 4), k3cuda.DevBuf(vocab * 4)
    n1, n2 = k3cuda.DevBuf(16), k3cuda.DevBuf(16)
    k3cuda.check(k3.k3d_rmsnorm(XN.ptr, H.ptr, NW.ptr, hidden, 1, 1e-6))
    k3cuda.check(k3.k3d_lm_head_argmax(n1.ptr, L1.ptr, XN.ptr, Wd.ptr, vocab, hidden, 1, key.ptr))
    k3cuda.check(k3.k3d_lm_head_argmax_normed(n2.ptr, L2.ptr, H.ptr, NW.ptr, 1e-6, Wd.ptr, vocab,
                                              hidden, 1, key.ptr))
    k3cuda.check(k3.k3d_sync())
    a, b = L1.download(np.float32, vocab), L2.download(np.float32, vocab)
    assert max_rel_err(b, a) <= 1e-5
    assert int(n2.download(np.int32, 1)[0]) == int(np.argmax(b))
