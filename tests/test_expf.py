"""The router's exp (kimi-k3-in-c_b200/csrc/k3_expf.h) against the host libm's expf, which
the reference's router calls (k3_ops.c:451). CPU only: the header is compiled for the host
here; the GPU copy of the same source is checked by test_gpu_router.py."""
import ctypes
import os
import subprocess
import tempfile
from decimal import Decimal, getcontext
import struct

import numpy as np
import pytest

from conftest import PKG

SHIM = r"""
#include <math.h>
#include <stdint.h>
#include <string.h>
#include "k3_expf.h"
/* compares k3_expf with libm expf on every float whose bit pattern is lo + i*stride */
long long sweep(uint32_t lo, uint32_t hi, uint32_t stride, long long *tested)
{
    long long bad = 0, n = 0;
    for (uint64_t u = lo; u <= hi; u += stride) {
        uint32_t b = (uint32_t)u; float x; memcpy(&x, &b, 4);
        if (!(x > -103.9f && x < 88.7f)) continue;
        float a = expf(x), c = k3_expf(x);
        n++;
        if (memcmp(&a, &c, 4)) bad++;
    }
    *tested = n;
    return bad;
}
unsigned long long tab(int i) { return k3_exp2_tab_h[i]; }
"""


@pytest.fixture(scope="module")
def shim():
    d = tempfile.mkdtemp()
    src = os.path.join(d, "s.c")
    so = os.path.join(d, "s.so")
    open(src, "w").write(SHIM)
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-shared", "-fPIC", "-I",
                    os.path.join(PKG, "csrc"), src, "-o", so, "-lm"], check=True)
    lib = ctypes.CDLL(so)
    lib.sweep.restype = ctypes.c_longlong
    lib.sweep.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                          ctypes.POINTER(ctypes.c_longlong)]
    lib.tab.restype = ctypes.c_ulonglong
    return lib


def test_table_is_correctly_rounded(shim):
    getcontext().prec = 60
    for i in range(32):
        v = float(Decimal(2) ** (Decimal(i) / Decimal(32)))
        assert struct.unpack("<Q", struct.pack("<d", v))[0] == shim.tab(i)


def test_matches_libm_on_a_dense_sample(shim):
    n = ctypes.c_longlong()
    # positive and negative halves of the float line, every 97th pattern (~44M floats)
    bad = shim.sweep(0x00000000, 0x7F7FFFFF, 97, ctypes.byref(n))
    bad += shim.sweep(0x80000000, 0xFF7FFFFF, 97, ctypes.byref(n))
    assert bad == 0


def test_matches_libm_on_inputs_where_libm_is_not_correctly_rounded(shim):
    # glibc's expf is not correctly rounded: these are inputs where it differs from
    # (float)exp((double)x); the restatement must follow glibc, not the true value
    n = ctypes.c_longlong()
    for xs in ("0x1.fefe02p-16", "0x1.5b3c52p-14", "0x1.cd3982p-14", "0x1.dfb8fap-14"):
        b = struct.unpack("<I", struct.pack("<f", float.fromhex(xs)))[0]
        assert shim.sweep(b, b, 1, ctypes.byref(n)) == 0 and n.value == 1
