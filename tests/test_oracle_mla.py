"""The config-2 MLA oracle pinned (CPU only).

1. The expanded form (orc_mla_decode, theta = 0) against the reference's own
   k3_mla_cached (src/core/k3_ops.c:321-410, compiled in oracle/_ref) in its cached mode:
   the bf16 latent cache is expanded through kv_b with the reference's k3_matmul_bf16 into
   the reference's fp32 per-head key/value cache and its shared rope cache.
2. The absorbed form (orc_mla_decode_absorbed), which the full-size GPU tests use because
   it is O(L) per head, against the expanded form, with RoPE (theta 50000) and without.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import max_rel_err
import oracle as orc_mod
import synth

SMALL = dict(hidden=256, H=8, q_lora=64, kv_lora=128, qn=32, qr=16, vh=32, eps=1e-6)


def make(seed, d, B, cap, L):
    g = synth.rng(seed)
    qh, kvw, kvd = d["qn"] + d["qr"], d["kv_lora"] + d["qr"], d["qn"] + d["vh"]
    w = {
        "q_a": synth.bf16_normal(g, (d["q_lora"], d["hidden"]), 0.05),
        "q_b": synth.bf16_normal(g, (d["H"] * qh, d["q_lora"]), 0.05),
        "kv_a": synth.bf16_normal(g, (kvw, d["hidden"]), 0.05),
        "kv_b": synth.bf16_normal(g, (d["H"] * kvd, d["kv_lora"]), 0.05),
        "o": synth.bf16_normal(g, (d["hidden"], d["H"] * d["vh"]), 0.05),
        "g": synth.bf16_normal(g, (d["H"] * d["vh"], d["hidden"]), 0.05),
        "q_a_norm": (1.0 + 0.1 * g.standard_normal(d["q_lora"])).astype(np.float32),
        "kv_a_norm": (1.0 + 0.1 * g.standard_normal(d["kv_lora"])).astype(np.float32),
    }
    cache = np.zeros((B, cap, kvw), np.uint16)
    cache[:, :L] = synth.bf16_normal(g, (B, L, kvw), 1.0)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (B, d["hidden"]), 1.0))
    return w, cache, x


@pytest.mark.parametrize("L", [0, 1, 17, 100])
def test_expanded_oracle_matches_reference_mla_cached(oracle, reference, L):
    d = dict(SMALL, theta=0.0)
    cap = 128
    w, cache, x = make(100 + L, d, 1, cap, L)
    want_in = cache.copy()
    oracle.lib.orc_set_mla_new_entry_fp32(1)
    try:
        got = orc_mod.mla_decode(oracle, x, d, w, cache, L)
    finally:
        oracle.lib.orc_set_mla_new_entry_fp32(0)

    lib = reference.lib
    orc_mod.ref_kda_layer_fn(lib)           # declares k3_mla_cached and its scratch sizer
    H, kvd, qr, kvl = d["H"], d["qn"] + d["vh"], d["qr"], d["kv_lora"]
    kvc = np.zeros((cap, H * kvd), np.float32)
    ropec = np.zeros((cap, qr), np.float32)
    for s in range(L):
        lat = synth.bf16_to_f32(want_in[0, s, :kvl])
        kvc[s] = reference.matmul_bf16(lat, w["kv_b"])
        ropec[s] = synth.bf16_to_f32(want_in[0, s, kvl:])
    cfg = orc_mod.K3Cfg(hidden=d["hidden"], n_heads=H, q_lora=d["q_lora"], kv_lora=kvl,
                        qk_nope=d["qn"], qk_rope=qr, v_head=d["vh"], mla_out_gate=1,
                        rms_eps=d["eps"])
    mw = orc_mod.K3MlaW(*(w[k].ctypes.data for k in ("q_a", "q_b", "kv_a", "kv_b", "o", "g",
                                                      "q_a_norm", "kv_a_norm")), 1)
    scratch = np.empty(lib.k3_mla_scratch_cached(C.byref(cfg), 1, cap, 1) + 64, np.float32)
    out = np.empty(d["hidden"], np.float32)
    lib.k3_mla_cached(out.ctypes.data, x.ctypes.data, C.byref(mw), C.byref(cfg), 1,
                      scratch.ctypes.data, kvc.ctypes.data, ropec.ctypes.data, L, cap)
    # with the new entry read in fp32 the oracle runs the reference's arithmetic: same
    # projections, the same kv_b expansion (dot16), the same float scores, float exp and
    # double sums, in the same order
    assert np.array_equal(got[0].view(np.uint32), out.view(np.uint32)), max_rel_err(got[0], out)
    # the new cache entry is the reference's latent and rope slot, rounded to bf16
    assert np.array_equal(cache[0, L, kvl:], synth.f32_to_bf16(ropec[L]))
    assert max_rel_err(synth.bf16_to_f32(cache[0, L, :kvl]),
                       reference_latent(reference, w, x[0], d)) <= 4e-3


def reference_latent(reference, w, x, d):
    c = reference.matmul_bf16(x, w["kv_a"])[:d["kv_lora"]]
    return reference.rmsnorm(c, w["kv_a_norm"], d["eps"])


@pytest.mark.parametrize("theta,B,L", [(50000.0, 1, 0), (50000.0, 2, 63), (50000.0, 1, 300),
                                       (0.0, 3, 41)])
def test_absorbed_oracle_matches_expanded(oracle, theta, B, L):
    d = dict(SMALL, theta=theta)
    cap = 320
    w, cache, x = make(7 + L, d, B, cap, L)
    c1, c2 = cache.copy(), cache.copy()
    a = orc_mod.mla_decode(oracle, x, d, w, c1, L)
    b = orc_mod.mla_decode(oracle, x, d, w, c2, L, absorbed=True)
    assert np.array_equal(c1, c2)
    assert max_rel_err(b, a) <= 1e-5
