"""The safetensors checkpoint index (k3d_ckpt_*: the device loader's counterpart of
src/io/k3_st.c) against Python's own json parse of the same shards, as the reference checks
its scanner (tools/verify_st.py): every tensor's dtype, shape, absolute offset and size,
the bytes read back, and the refusal of malformed or inconsistent headers. Host code only."""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

import k3cuda
from safetensors_io import read_header, write_shard

DT = {"U8": 1, "BF16": 2, "F16": 3, "F32": 4}


@pytest.fixture(scope="module")
def lib():
    return k3cuda.load()


def _shards(tmp_path, seed=0):
    g = np.random.default_rng(seed)
    d = tmp_path / "ck"
    d.mkdir()
    specs = []
    for s in range(3):
        t = {}
        for i in range(40):
            dt = ["U8", "BF16", "F16", "F32"][(i + s) % 4]
            shape = [int(x) for x in g.integers(1, 9, size=int(g.integers(0, 4)))]
            n = int(np.prod(shape)) if shape else 1
            arr = (g.integers(0, 250, n).astype(np.uint8) if dt == "U8" else
                   g.integers(0, 65535, n).astype(np.uint16) if dt == "BF16" else
                   g.standard_normal(n).astype(np.float16 if dt == "F16" else np.float32))
            t[f"language_model.model.layers.{s}.t{i}.weight"] = (dt, shape, arr)
        write_shard(d / f"model-{s + 1:05d}-of-00003.safetensors", t,
                    metadata={"format": "pt", "note": 'a "quoted" {value}'} if s == 1 else None)
        specs.append(t)
    (d / "README.txt").write_text("not a shard")
    return d, specs


def test_index_matches_python_json(lib, tmp_path):
    d, specs = _shards(tmp_path)
    lib_ck = lib.k3d_ckpt_open(str(d).encode())
    assert lib_ck, lib.k3d_ckpt_error().decode()
    try:
        assert lib.k3d_ckpt_count(lib_ck) == sum(len(t) for t in specs)
        files = sorted(os.listdir(d))
        files = [f for f in files if f.endswith(".safetensors")]
        for shard, fname in enumerate(files):
            hdr, base = read_header(d / fname)
            raw = (d / fname).read_bytes()
            for name, ent in hdr.items():
                if name == "__metadata__":
                    continue
                t = k3cuda.K3dCkptTensor()
                assert lib.k3d_ckpt_find(lib_ck, name.encode(), ctypes.byref(t)) == 0, name
                assert (t.shard, t.dtype, t.ndim) == (shard, DT[ent["dtype"]], len(ent["shape"]))
                assert list(t.shape[:t.ndim]) == ent["shape"]
                s0, s1 = ent["data_offsets"]
                assert (t.off, t.nbytes) == (base + s0, s1 - s0)
                buf = ctypes.create_string_buffer(max(t.nbytes, 1))
                assert lib.k3d_ckpt_read(lib_ck, t.shard, t.off, t.nbytes, buf) == t.nbytes
                assert buf.raw[:t.nbytes] == raw[base + s0: base + s1]
        t = k3cuda.K3dCkptTensor()
        assert lib.k3d_ckpt_find(lib_ck, b"language_model.model.layers.9.t0.weight", ctypes.byref(t)) == k3cuda.K3D_EINVAL
    finally:
        lib.k3d_ckpt_close(lib_ck)


def _one(tmp_path, name, header_obj=None, raw_header=None, data=b"\0" * 64):
    d = tmp_path / name
    d.mkdir()
    h = raw_header if raw_header is not None else json.dumps(header_obj).encode()
    (d / "m.safetensors").write_bytes(struct.pack("<Q", len(h)) + h + data)
    return str(d).encode()


@pytest.mark.parametrize("case", ["span", "outside", "dtype", "order", "syntax", "length", "dup"])
def test_bad_headers_are_refused(lib, tmp_path, case):
    ok = {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}
    hdrs = {
        "span": {"a": {"dtype": "F32", "shape": [5], "data_offsets": [0, 16]}},
        "outside": {"a": {"dtype": "U8", "shape": [100], "data_offsets": [0, 100]}},
        "dtype": {"a": {"dtype": "F64", "shape": [2], "data_offsets": [0, 16]}},
        "order": {"a": {"dtype": "F32", "shape": [0], "data_offsets": [16, 0]}},
    }
    if case in hdrs:
        path = _one(tmp_path, case, hdrs[case])
    elif case == "syntax":
        path = _one(tmp_path, case, raw_header=b'{"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]')
    elif case == "length":
        d = tmp_path / case
        d.mkdir()
        (d / "m.safetensors").write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
        path = str(d).encode()
    else:
        d = tmp_path / case
        d.mkdir()
        write_shard(d / "a.safetensors", {"x": ("F32", [4], np.zeros(4, np.float32))})
        write_shard(d / "b.safetensors", {"x": ("F32", [4], np.zeros(4, np.float32))})
        path = str(d).encode()
    ck = lib.k3d_ckpt_open(path)
    assert not ck, case
    assert lib.k3d_ckpt_error().decode()
    good = _one(tmp_path, case + "_ok", {"a": ok})
    ck = lib.k3d_ckpt_open(good)
    assert ck
    lib.k3d_ckpt_close(ck)


def test_missing_directory_or_no_shards(lib, tmp_path):
    assert not lib.k3d_ckpt_open(str(tmp_path / "nope").encode())
    (tmp_path / "empty").mkdir()
    assert not lib.k3d_ckpt_open(str(tmp_path / "empty").encode())
