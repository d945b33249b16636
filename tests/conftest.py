import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "kimi-k3-in-c_b200")
for p in (PKG, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


def _ensure_built():
    lib = os.path.join(PKG, "lib", "libk3cuda.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)
    if not os.path.exists(os.path.join(REPO, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle")], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref/libk3ref.so not built (reference tree absent at build time)")
    return Reference()


@pytest.fixture(scope="session")
def k3():
    """libk3cuda on cuda:0. Only requested by tests marked gpu."""
    import k3cuda
    lib = k3cuda.init(0)
    return lib


@pytest.fixture(autouse=True)
def _clear_status(request):
    if request.node.get_closest_marker("gpu"):
        import k3cuda
        lib = k3cuda.load()
        lib.k3d_clear_status()
        yield
        st = lib.k3d_status()
        # a test that expects an error clears it itself; anything left is a failure
        assert st == 0, f"k3cuda status {st}: {lib.k3d_last_message().decode()}"
    else:
        yield


def load_npz(name):
    d = np.load(os.path.join(GOLDEN, name))
    meta = {}
    if "__meta__" in d:
        import json
        meta = json.loads(bytes(d["__meta__"]).decode())
    return {k: d[k] for k in d.files if k != "__meta__"}, meta


def manifest_tol():
    import json
    m = json.load(open(os.path.join(GOLDEN, "ref_ops", "MANIFEST.json")))
    return m["tolerance"]["fp32_abs"], m["tolerance"]["fp32_rel"]


def assert_close_elementwise(got, want, atol, rtol, what=""):
    """test_ops.c's criterion: |got - want| <= atol + rtol * |want| for every element."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want) / (atol + rtol * np.abs(want))
    worst = float(err.max()) if err.size else 0.0
    assert worst <= 1.0, f"{what}: worst {worst:.3f}x tolerance at {int(err.argmax())}"


def max_rel_err(got, want):
    """Normwise max relative error: max|got - want| / max|want| (the 1e-3 contract)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = float(np.abs(want).max())
    return float(np.abs(got - want).max()) / (den if den > 0 else 1.0)
