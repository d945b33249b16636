"""Seeded synthetic inputs at the benchmark shapes (test infrastructure).

numpy's PCG64 bit stream is stable across platforms, so these regenerate bit-identically on
the GPU hosts; make_golden.py stores a digest of each generated input next to its golden
output so that any drift is caught rather than read as a kernel mismatch.
"""
import hashlib

import numpy as np


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def f32_to_bf16(a):
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_normal(g, shape, std):
    return f32_to_bf16(g.standard_normal(shape, dtype=np.float32) * np.float32(std))


def mxfp4_matrix(g, rows, cols, s_lo=117, s_hi=121):
    """Packed E2M1 codes uniform over all 16 values and E8M0 bytes uniform in [s_lo, s_hi]."""
    packed = g.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = g.integers(s_lo, s_hi + 1, size=(rows, cols // 32), dtype=np.uint8)
    return packed, scales


def mxfp4_expert(g, hidden, inter, s_lo=117, s_hi=121):
    p1, s1 = mxfp4_matrix(g, inter, hidden, s_lo, s_hi)
    p3, s3 = mxfp4_matrix(g, inter, hidden, s_lo, s_hi)
    p2, s2 = mxfp4_matrix(g, hidden, inter, s_lo, s_hi)
    return {"p1": p1, "s1": s1, "p3": p3, "s3": s3, "p2": p2, "s2": s2}


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:32]


def config0_inputs(seed=1234, hidden=7168, inter=2048):
    g = rng(seed)
    x = bf16_to_f32(bf16_normal(g, hidden, 1.0))
    e = mxfp4_expert(g, hidden, inter)
    return x, e


def router_inputs(seed=4321, T=4, hidden=7168, n_experts=384):
    g = rng(seed)
    W = bf16_normal(g, (n_experts, hidden), 0.02)
    bias = g.uniform(-0.1, 0.1, size=n_experts).astype(np.float32)
    x = bf16_to_f32(bf16_normal(g, (T, hidden), 1.0))
    return x, W, bias
