"""The tensor-core bf16 GEMM (k3_gemm_tc.cu: tcgen05 kind::f16, TMA weight tiles, tokens as
bf16 hi + lo) behind k3d_gemv_bf16 for batches of more than four tokens, against a float64
product of the same bf16 weights and fp32 inputs (the reference accumulates in double,
k3_ops.c:1108-1213). Normwise max relative error 1e-5 (fp32 accumulation, 16-bit split of
the inputs)."""
import numpy as np
import pytest

import k3cuda
import synth
from conftest import max_rel_err

pytestmark = pytest.mark.gpu


def gemv(k3, x, Wb, accumulate_into=None):
    T, n_in = x.shape
    out = Wb.shape[0]
    X = k3cuda.DevBuf.from_array(x)
    W = k3cuda.DevBuf.from_array(Wb)
    y0 = accumulate_into if accumulate_into is not None else np.zeros((T, out), np.float32)
    Y = k3cuda.DevBuf.from_array(y0)
    k3cuda.check(k3.k3d_gemv_bf16(Y.ptr, X.ptr, W.ptr, n_in, out, T, 1 if accumulate_into is not None else 0))
    k3cuda.check(k3.k3d_sync())
    return Y.download(np.float32, (T, out))


def want(x, Wb, prev=None):
    W = synth.bf16_to_f32(Wb).astype(np.float64)
    y = x.astype(np.float64) @ W.T
    return y if prev is None else y + prev


@pytest.mark.parametrize("T", [5, 8, 16, 33, 64, 130])
@pytest.mark.parametrize("n_in,out", [(7168, 2048), (1536, 576), (128, 1024), (2048, 7168)])
def test_gemm_tc_matches_float64(k3, T, n_in, out):
    g = synth.rng(T * 1000 + n_in + out)
    Wb = synth.bf16_normal(g, (out, n_in), 0.02)
    x = (g.standard_normal((T, n_in)) * np.exp2(g.integers(-4, 4, (T, n_in)))).astype(np.float32)
    y = gemv(k3, x, Wb)
    assert max_rel_err(y, want(x, Wb)) <= 1e-5


def test_gemm_tc_accumulates_and_repeats(k3):
    g = synth.rng(77)
    T, n_in, out = 24, 1024, 640
    Wb = synth.bf16_normal(g, (out, n_in), 0.02)
    x = synth.bf16_to_f32(synth.bf16_normal(g, (T, n_in), 1.0))
    prev = g.standard_normal((T, out)).astype(np.float32)
    y1 = gemv(k3, x, Wb, prev)
    y2 = gemv(k3, x, Wb, prev)
    assert np.array_equal(y1, y2)
    assert max_rel_err(y1, want(x, Wb, prev.astype(np.float64))) <= 1e-5
