"""MXFP4 dequant and GEMV on the GPU through the C ABI, against the oracle and the
reference's golden vectors (real checkpoint bytes)."""
import ctypes

import numpy as np
import pytest

import k3cuda
from conftest import load_npz, max_rel_err
import synth

pytestmark = pytest.mark.gpu


def test_dequant_bit_exact_on_checkpoint_bytes_host_pointers(k3):
    d, _ = load_npz("mxfp4.npz")
    rows, pcols = d["packed"].shape
    out = np.empty((rows, 2 * pcols), np.float32)
    k3.k3_mxfp4_dequant(out.ctypes.data, d["packed"].ctypes.data, d["scales"].ctypes.data,
                        rows, pcols, 32)
    assert k3.k3d_status() == 0
    assert np.array_equal(out.view(np.uint32), d["expected"].reshape(rows, -1).view(np.uint32))


def test_dequant_bit_exact_device_pointers_all_scale_bytes(k3, oracle):
    g = synth.rng(11)
    rows, cols = 256, 512
    packed = g.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    # every E8M0 byte including 0 (denormal 2^-127), 254 and the NaN byte 255
    scales = (np.arange(rows * cols // 32) % 256).astype(np.uint8).reshape(rows, -1)
    P = k3cuda.DevBuf.from_array(packed)
    S = k3cuda.DevBuf.from_array(scales)
    O = k3cuda.DevBuf(rows * cols * 4)
    k3.k3_mxfp4_dequant(O.ptr, P.ptr, S.ptr, rows, cols // 2, 32)
    k3cuda.check(k3.k3d_sync())
    got = O.download(np.float32, (rows, cols))
    want = oracle.mxfp4_dequant(packed, scales, rows, cols // 2, 32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols,group", [(64, 3584, 32), (2048, 7168, 32), (7168, 2048, 32),
                                             (40, 1024, 32), (33, 96, 32), (17, 50, 25),
                                             (9, 64, 64), (5, 30, 7)])
def test_matmul_mxfp4_matches_oracle(k3, oracle, rows, cols, group):
    g = synth.rng(rows * 7 + cols)
    packed = g.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    ngrp = (cols + group - 1) // group
    scales = g.integers(110, 125, (rows, ngrp), dtype=np.uint8)
    scales[0, 0] = 255   # a NaN scale zeroes its group
    x = g.standard_normal(cols, dtype=np.float32)
    y = np.empty(rows, np.float32)
    k3.k3_matmul_mxfp4(y.ctypes.data, x.ctypes.data, packed.ctypes.data, scales.ctypes.data,
                       cols, rows, group)
    assert k3.k3d_status() == 0
    want = oracle.matmul_mxfp4(x, packed, scales, rows, group)
    assert max_rel_err(y, want) <= 1e-5


def test_matmul_mxfp4_checkpoint_bytes(k3, oracle):
    d, _ = load_npz("mxfp4.npz")
    rows, pcols = d["packed"].shape
    x = synth.rng(3).standard_normal(2 * pcols, dtype=np.float32)
    y = np.empty(rows, np.float32)
    k3.k3_matmul_mxfp4(y.ctypes.data, x.ctypes.data, d["packed"].ctypes.data,
                       d["scales"].ctypes.data, 2 * pcols, rows, 32)
    assert max_rel_err(y, oracle.matmul_mxfp4(x, d["packed"], d["scales"], rows)) <= 1e-5
    # dequantise-then-matmul (test_expert.c's check) agrees too
    W = d["expected"].reshape(rows, -1).astype(np.float64)
    assert max_rel_err(y, W @ x.astype(np.float64)) <= 1e-5


def test_matmul_mxfp4_rejects_what_the_reference_aborts_on(k3):
    y = np.zeros(4, np.float32)
    x = np.zeros(34, np.float32)
    p = np.zeros(4 * 17, np.uint8)
    s = np.zeros(8, np.uint8)
    k3.k3_matmul_mxfp4(y.ctypes.data, x.ctypes.data, p.ctypes.data, s.ctypes.data, 33, 4, 32)
    assert k3.k3d_status() == k3cuda.K3D_EINVAL
    k3.k3d_clear_status()
    k3.k3_matmul_mxfp4(y.ctypes.data, x.ctypes.data, p.ctypes.data, s.ctypes.data, 34, 4, 65)
    assert k3.k3d_status() == k3cuda.K3D_EINVAL
    k3.k3d_clear_status()


def test_config0_expert_full_size(k3, oracle):
    """BASELINE config 0 through k3d_expert_swiglu against the reference golden output."""
    d, _ = load_npz("ref_config0.npz")
    x, e = synth.config0_inputs()
    bufs = {k: k3cuda.DevBuf.from_array(v) for k, v in e.items()}
    q = k3cuda.K3ExpertQ(*(bufs[k].ptr for k in ("p1", "s1", "p3", "s3", "p2", "s2")))
    X = k3cuda.DevBuf.from_array(x)
    Y = k3cuda.DevBuf(7168 * 4)
    ws_n = k3.k3d_expert_ws_bytes(7168, 2048)
    WS = k3cuda.DevBuf(ws_n)
    for _ in range(2):  # the second call reuses the workspace
        k3cuda.check(k3.k3d_expert_swiglu(Y.ptr, X.ptr, ctypes.byref(q), 7168, 2048, WS.ptr, ws_n))
    k3cuda.check(k3.k3d_sync())
    y = Y.download(np.float32, 7168)
    assert max_rel_err(y, d["y"]) <= 1e-4
    assert max_rel_err(y, oracle.expert_swiglu(x, e, 7168, 2048)) <= 1e-4
