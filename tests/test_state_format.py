"""The K3ST header reader (k3d_state_peek) on files written by the CPU engine's layout
(src/cli/k3_run.c:175-300) in Python: fields, the device trailer flag, and refusal of files
that are not version-1 K3ST. Host code only: runs without a GPU."""
import ctypes

import numpy as np
import pytest

import k3cuda
import k3st


@pytest.fixture(scope="module")
def lib():
    return k3cuda.load()


def _write(tmp_path, name, data):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p).encode()


def _sample(latent):
    g = np.random.default_rng(3)
    fp = k3st.fingerprint(512, 8, 1024, 4, 64, 4, 8, 32, 16, 32, 16, 4)
    ks = g.standard_normal((8, 100)).astype(np.float32)
    kvc = g.standard_normal((2, 5, 8 * 64)).astype(np.float32)
    ropec = g.standard_normal((2, 5, 16)).astype(np.float32)
    lat = g.integers(0, 65535, (2, 5, 144), dtype=np.uint16) if latent else None
    return k3st.pack(fp, [1, 2, 3], ks, kvc, ropec, lat)


@pytest.mark.parametrize("latent", [False, True])
def test_peek_reads_the_header(lib, tmp_path, latent):
    path = _write(tmp_path, "s.k3st", _sample(latent))
    info = k3cuda.K3dStateInfo()
    assert lib.k3d_state_peek(path, ctypes.byref(info)) == 0
    assert (info.version, info.n_bound, info.n_mla, info.cached, info.nseq) == (1, 8, 2, 5, 3)
    assert info.has_latent == int(latent)


def test_unpack_round_trip():
    d = k3st.unpack(_sample(True))
    assert d["magic"] == b"K3ST" and d["cached"] == 5 and d["latent"].shape == (2, 5, 144)
    assert list(d["seq"]) == [1, 2, 3]


def test_peek_refuses_other_files(lib, tmp_path):
    info = k3cuda.K3dStateInfo()
    bad_magic = b"XXXX" + _sample(False)[4:]
    assert lib.k3d_state_peek(_write(tmp_path, "a", bad_magic), ctypes.byref(info)) == k3cuda.K3D_EINVAL
    v2 = bytearray(_sample(False))
    v2[4:8] = (2).to_bytes(4, "little")
    assert lib.k3d_state_peek(_write(tmp_path, "b", bytes(v2)), ctypes.byref(info)) == k3cuda.K3D_EINVAL
    assert lib.k3d_state_peek(_write(tmp_path, "c", b"K3ST"), ctypes.byref(info)) == k3cuda.K3D_EINVAL
    assert lib.k3d_state_peek(str(tmp_path / "missing").encode(), ctypes.byref(info)) == k3cuda.K3D_EINVAL
