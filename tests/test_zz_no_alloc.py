"""k3d_router_bf16_noalloc (fixed scratch compiled into the library, no device
allocation) against k3d_router_bf16 (library workspace). The router is bit-exact, so the
tolerance is zero: indices equal, weights equal bit for bit. The file name sorts last so
the test also runs after every other test has used the library in the same process."""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def _route(k3, fn, bufs, T, hidden, E, topk):
    import k3cuda
    X, Wd, B, I, Wt = bufs
    I.zero()
    Wt.zero()
    k3cuda.check(fn(I.ptr, Wt.ptr, X.ptr, Wd.ptr, B.ptr, T, hidden, E, topk, 1, 2.5))
    k3cuda.check(k3.k3d_sync())
    return I.download(np.int32, (T, topk)), Wt.download(np.float32, (T, topk))


@pytest.mark.parametrize("T", [1, 64])
def test_noalloc_router_matches_workspace_router(k3, T):
    import k3cuda
    hidden, E, topk = 7168, 384, 8
    x, W, bias = synth.router_inputs(seed=900 + T, T=T, hidden=hidden, n_experts=E)
    bufs = [k3cuda.DevBuf.from_array(a) for a in (x, W, bias)]
    bufs += [k3cuda.DevBuf(T * topk * 4), k3cuda.DevBuf(T * topk * 4)]
    want_i, want_w = _route(k3, k3.k3d_router_bf16, bufs, T, hidden, E, topk)
    # two calls in a row: the second reuses the scratch the first left behind
    for _ in range(2):
        got_i, got_w = _route(k3, k3.k3d_router_bf16_noalloc, bufs, T, hidden, E, topk)
        assert np.array_equal(got_i, want_i)
        assert np.array_equal(got_w.view(np.uint32), want_w.view(np.uint32))


def test_noalloc_router_rejects_oversize(k3):
    import k3cuda
    T, E = 86, 384                     # 33024 scores > K3D_ROUTER_NOALLOC_MAX (32768)
    bufs = [k3cuda.DevBuf(16) for _ in range(5)]
    rc = k3.k3d_router_bf16_noalloc(bufs[3].ptr, bufs[4].ptr, bufs[0].ptr, bufs[1].ptr,
                                    bufs[2].ptr, T, 7168, E, 8, 1, 2.5)
    assert rc == k3cuda.K3D_EBOUND
    assert "fixed scratch" in k3.k3d_last_message().decode()
    k3.k3d_clear_status()
