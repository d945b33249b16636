"""The C-ABI library loads and exports everything include/k3/*.h declares (CPU only: no
compute runs here)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import REPO

import k3cuda

HEADERS = [os.path.join(REPO, "include", "k3", h) for h in ("k3.h", "k3_cuda.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        # drop static inline bodies: they are header-only
        src = re.sub(r"static inline[^{]*\{(?:[^{}]|\{[^{}]*\})*\}", "", src)
        for m in re.finditer(r"\b([a-z_][a-z0-9_]*)\s*\(", src):
            name = m.group(1)
            if name.startswith(("k3_", "k3d_")):
                names.add(name)
    return names


def test_library_exports_every_declared_symbol():
    lib = k3cuda.load()
    want = declared_functions()
    assert len(want) > 60
    missing = [n for n in sorted(want) if not hasattr(lib, n)]
    assert not missing, missing
    # the expert-drop counter is a data symbol
    assert ctypes.c_long.in_dll(lib, "k3_expert_drops").value == 0
    # the Python binding declares prototypes for all of them
    undeclared = sorted(want - set(k3cuda.exported_names()))
    assert not undeclared, undeclared


def test_layer_map_is_host_logic():
    lib = k3cuda.load()
    full = (ctypes.c_int * 4)(4, 8, 12, 13)
    cfg = k3cuda.K3Cfg(n_full_attn=4, full_attn=full, first_dense=1)
    # one-based full_attn: zero-based MLA layers are 3, 7, 11, 12
    mla = [i for i in range(13) if lib.k3_is_mla(ctypes.byref(cfg), i)]
    assert mla == [3, 7, 11, 12]
    assert lib.k3_is_dense(ctypes.byref(cfg), 0) and not lib.k3_is_dense(ctypes.byref(cfg), 1)
    assert lib.k3_is_kda(ctypes.byref(cfg), 0) and not lib.k3_is_kda(ctypes.byref(cfg), 3)


@pytest.mark.skipif(bool(glob.glob("/dev/nvidia[0-9]*")), reason="checks the no-GPU failure path")
def test_without_a_gpu_calls_fail_loudly():
    """No CPU fallback: with no CUDA device every entry point records K3D_ENODEV."""
    lib = k3cuda.load()
    assert lib.k3d_init(0) == k3cuda.K3D_ENODEV
    import numpy as np
    y = np.full(4, 7.0, np.float32)
    x = np.ones(8, np.float32)
    W = np.ones(32, np.float32)
    lib.k3d_clear_status()
    lib.k3_matmul(y.ctypes.data, x.ctypes.data, W.ctypes.data, 8, 4)
    assert lib.k3d_status() == k3cuda.K3D_ENODEV
    assert np.all(y == 7.0), "output must be left untouched"
    lib.k3d_clear_status()
