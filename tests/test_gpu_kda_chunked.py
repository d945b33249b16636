"""KDA chunked prefill (chunk = 64, the WY form) against the sequential recurrence.

The reference has only the sequential step (k3_kda_step, k3_ops.c:186-243); the chunked
form regroups the same arithmetic, so its parity bar is the fp32 tolerance (1e-3
normwise relative to the sequential result), not bit equality. The sequential GPU path
itself is pinned bit-exact to the oracle in test_gpu_router_gemv.py, which lets the
full config-3 size (8192 tokens, 64 heads) be checked against it here."""
import numpy as np
import pytest

import k3cuda
from conftest import max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _inputs(seed, T, H, dk, dv, decay):
    g = np.random.default_rng(seed)

    def unit(x):
        return (x / np.linalg.norm(x, axis=-1, keepdims=True)).astype(np.float32)

    S = (g.standard_normal((H, dk, dv)) * 0.01).astype(np.float32)
    q = unit(g.standard_normal((T, H, dk)))
    k = unit(g.standard_normal((T, H, dk)))
    v = g.standard_normal((T, H, dv)).astype(np.float32)
    al = g.uniform(decay[0], decay[1], (T, H, dk)).astype(np.float32)
    be = g.uniform(0, 1, (T, H)).astype(np.float32)
    return S, q, k, v, al, be


def _prefill(k3, S, q, k, v, al, be, chunk):
    T, H, dk = q.shape
    dv = v.shape[2]
    bufs = [k3cuda.DevBuf.from_array(np.ascontiguousarray(a)) for a in (S, q, k, v, al, be)]
    O = k3cuda.DevBuf(T * H * dv * 4)
    k3cuda.check(k3.k3d_kda_prefill(bufs[0].ptr, O.ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                    bufs[4].ptr, bufs[5].ptr, T, H, dk, dv, chunk))
    k3cuda.check(k3.k3d_sync())
    return bufs[0].download(np.float32, S.shape), O.download(np.float32, (T, H, dv))


def _oracle_sequence(oracle, S, q, k, v, al, be):
    So = S.copy()
    oo = np.zeros((q.shape[0], q.shape[1], v.shape[2]), np.float32)
    for t in range(q.shape[0]):
        So2, o2 = oracle.kda_decode(So[None], q[t][None], k[t][None], v[t][None], al[t][None],
                                    be[t][None])
        So = So2[0]
        oo[t] = o2[0]
    return So, oo


@pytest.mark.parametrize("T,H,dk,dv,decay", [
    (200, 4, 128, 128, (0.9, 1.0)),     # config-3 gates: the product path for L and M
    (150, 3, 128, 128, (0.05, 0.5)),    # strong decay: |G| > 60, one exponential per pair
    (520, 2, 128, 128, (0.9, 1.0)),     # 9 chunks: crosses the 8-chunk segment boundary
    (64, 2, 64, 64, (0.5, 1.0)),        # exactly one chunk, smaller head
    (37, 2, 128, 32, (0.9, 1.0)),       # one ragged chunk, dv = 32
    (1, 1, 8, 32, (0.9, 1.0)),          # one step, the smallest supported head
])
def test_kda_chunked_matches_sequential_oracle(k3, oracle, T, H, dk, dv, decay):
    S, q, k, v, al, be = _inputs(31 + T, T, H, dk, dv, decay)
    Sg, og = _prefill(k3, S, q, k, v, al, be, 64)
    So, oo = _oracle_sequence(oracle, S, q, k, v, al, be)
    assert np.isfinite(og).all() and np.isfinite(Sg).all()
    assert max_rel_err(og, oo) <= TOL, max_rel_err(og, oo)
    assert max_rel_err(Sg, So) <= TOL, max_rel_err(Sg, So)


def test_kda_chunked_zero_decay(k3, oracle):
    """A decay of exactly 0 forgets the state; the chunked form treats it as 2^-126."""
    S, q, k, v, al, be = _inputs(5, 130, 2, 128, 128, (0.9, 1.0))
    al[17, :, ::3] = 0.0
    al[90, 1, :] = 0.0
    Sg, og = _prefill(k3, S, q, k, v, al, be, 64)
    So, oo = _oracle_sequence(oracle, S, q, k, v, al, be)
    assert max_rel_err(og, oo) <= TOL and max_rel_err(Sg, So) <= TOL


def test_kda_chunked_config3_full_size_vs_sequential(k3):
    """8192 tokens x 64 heads x 128x128 (BASELINE config 3 prefill) against the sequential
    kernel, which is bit-identical to the reference step."""
    T, H, D = 8192, 64, 128
    S, q, k, v, al, be = _inputs(77, T, H, D, D, (0.9, 1.0))
    Sc, oc = _prefill(k3, S, q, k, v, al, be, 64)
    Ss, os_ = _prefill(k3, S, q, k, v, al, be, 0)
    assert max_rel_err(oc, os_) <= TOL, max_rel_err(oc, os_)
    assert max_rel_err(Sc, Ss) <= TOL, max_rel_err(Sc, Ss)


def test_kda_prefill_rejects_other_chunks_and_shapes(k3):
    S, q, k, v, al, be = _inputs(1, 8, 1, 128, 128, (0.9, 1.0))
    bufs = [k3cuda.DevBuf.from_array(a) for a in (S, q, k, v, al, be)]
    O = k3cuda.DevBuf(8 * 128 * 4)
    for chunk, dk, dv in ((32, 128, 128), (64, 100, 128), (64, 128, 48)):
        rc = k3.k3d_kda_prefill(bufs[0].ptr, O.ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                bufs[4].ptr, bufs[5].ptr, 8, 1, dk, dv, chunk)
        assert rc == k3cuda.K3D_EINVAL
        k3.k3d_clear_status()
    # q, k and the decay are read as float4 rows: a pointer off a 16-byte boundary is refused
    rc = k3.k3d_kda_prefill(bufs[0].ptr, O.ptr, bufs[1].ptr + 4, bufs[2].ptr, bufs[3].ptr,
                            bufs[4].ptr, bufs[5].ptr, 4, 1, 128, 128, 64)
    assert rc == k3cuda.K3D_EINVAL
    k3.k3d_clear_status()
