"""Conversation state in the CPU engine's K3ST format (k3d_model_state_save/_load against
src/cli/k3_run.c:158-300) on the reduced-width decode stack: the file's sections read as the
CPU engine reads them hold the KDA states, the expanded keys and values (kv_b times the
latent) and the rope slots; a save/load round trip restores the caches bit for bit and the
next step decodes identically; a file without the device trailer (what the CPU engine
writes) is restored through the least-squares latent recovery; files of another model or
larger than the cache are refused."""
import contextlib
import ctypes

import numpy as np
import pytest

import k3cuda
import k3st
from conftest import max_rel_err
from test_gpu_stack import CFG, make_cfg, download

pytestmark = pytest.mark.gpu

CAP = 64


def bf16_f32(u):
    return (np.asarray(u, np.uint16).astype(np.uint32) << 16).view(np.float32)


@contextlib.contextmanager
def model(k3, seed=77, batch=1, cap=CAP, **over):
    c = dict(CFG, **over)
    m = k3.k3d_model_create(ctypes.byref(make_cfg(c, batch=batch, cap=cap, layout=1)), seed)
    assert m, k3.k3d_last_message()
    try:
        yield m
    finally:
        k3.k3d_model_destroy(m)


def step(k3, m, toks):
    toks = np.asarray(toks, np.int32)
    nxt = np.zeros(len(toks), np.int32)
    k3cuda.check(k3.k3d_model_step_host(m, toks.ctypes.data, nxt.ctypes.data))
    return nxt, download(k3, m, "logits", np.float32).reshape(len(toks), -1).copy()


def advance(k3, m, batch=1):
    """Context of 6 synthetic positions, then two decoded tokens (eager, then the graph)."""
    k3cuda.check(k3.k3d_model_fill_context(m, 6, 31))
    toks = np.arange(batch, dtype=np.int32) * 7 + 5
    seq = [int(toks[0])]
    for _ in range(2):
        toks, _ = step(k3, m, toks)
        seq.append(int(toks[0]))
    return seq


def caches(k3, m, cached, b=0, batch=1):
    """(MLA layer -> cache rows [cached][kvw] uint16 of sequence b, KDA layer -> state)."""
    c = CFG
    mla, kda = {}, {}
    kvw = c["mla"]["kv_lora"] + c["mla"]["qr"]
    for l in range(c["n_layers"]):
        if l in c["mla_layers"]:
            a = download(k3, m, f"layer{l}.mla.cache", np.uint16).reshape(batch, CAP, kvw)
            mla[l] = a[b, :cached].copy()
        else:
            a = download(k3, m, f"layer{l}.kda.state", np.float32).reshape(batch, -1)
            kda[l] = a[b].copy()
    return mla, kda


def save(k3, m, path, seq, b=0):
    s = np.asarray(seq, np.int32)
    k3cuda.check(k3.k3d_model_state_save(m, str(path).encode(), s.ctypes.data, len(s), b), "save")


def load(k3, m, path, cap=64, b=0):
    s = np.zeros(cap, np.int32)
    r = k3.k3d_model_state_load(m, str(path).encode(), s.ctypes.data, cap, b)
    return r, s


def test_save_writes_the_cpu_engine_layout(k3, tmp_path):
    c, ml = CFG, CFG["mla"]
    with model(k3) as a:
        seq = advance(k3, a)
        pos = int(download(k3, a, "pos", np.int32)[0])
        save(k3, a, tmp_path / "a.k3st", seq)
        mla, kda = caches(k3, a, pos)
        d = k3st.unpack((tmp_path / "a.k3st").read_bytes())
        assert d["magic"] == b"K3ST" and d["version"] == 1
        assert d["fp"] == k3st.fingerprint(c["hidden"], c["n_layers"], c["vocab"], c["kda_heads"],
                                           c["kda_head_dim"], c["conv_k"], ml["H"], ml["qn"], ml["qr"],
                                           ml["vh"], c["moe"]["n_experts"], c["moe"]["topk"])
        assert (d["n_bound"], d["n_mla"], d["cached"]) == (c["n_layers"], 2, pos)
        assert list(d["seq"]) == seq
        assert d["kvpp"] == ml["H"] * (ml["qn"] + ml["vh"]) and d["ropepp"] == ml["qr"]
        for l in range(c["n_layers"]):
            if l in kda:
                assert np.array_equal(d["ks"][l], kda[l]), l
            else:
                assert not d["ks"][l].any(), l
        for mi, l in enumerate(c["mla_layers"]):
            kv_b = bf16_f32(download(k3, a, f"layer{l}.mla.kv_b", np.uint16)).reshape(-1, ml["kv_lora"])
            lat = bf16_f32(mla[l][:, :ml["kv_lora"]]).astype(np.float64)
            want = lat @ kv_b.astype(np.float64).T
            assert max_rel_err(d["kvc"][mi], want) <= 1e-5, l
            assert np.array_equal(d["ropec"][mi], bf16_f32(mla[l][:, ml["kv_lora"]:])), l
            assert np.array_equal(d["latent"][mi], mla[l]), l


def test_round_trip_restores_caches_and_decoding(k3, tmp_path):
    with model(k3) as a, model(k3) as b:
        seq = advance(k3, a)
        pos = int(download(k3, a, "pos", np.int32)[0])
        save(k3, a, tmp_path / "s.k3st", seq)
        info = k3cuda.K3dStateInfo()
        k3cuda.check(k3.k3d_state_peek(str(tmp_path / "s.k3st").encode(), ctypes.byref(info)))
        assert (info.cached, info.nseq, info.has_latent) == (pos, len(seq), 1)
        r, s = load(k3, b, tmp_path / "s.k3st")
        assert r == 0, k3.k3d_last_message()
        assert list(s[:len(seq)]) == seq
        assert int(download(k3, b, "pos", np.int32)[0]) == pos
        ma, ka = caches(k3, a, pos)
        mb, kb = caches(k3, b, pos)
        for l in ma:
            assert np.array_equal(ma[l], mb[l]), l
        for l in ka:
            assert np.array_equal(ka[l], kb[l]), l
        for _ in range(2):
            na, la = step(k3, a, [seq[-1]])
            nb, lb = step(k3, b, [seq[-1]])
            assert np.array_equal(la, lb)
            assert np.array_equal(na, nb)
            seq.append(int(na[0]))


def test_cpu_engine_file_without_trailer_recovers_the_latent(k3, tmp_path):
    with model(k3) as a, model(k3) as b, model(k3) as cpu:
        seq = advance(k3, a)
        pos = int(download(k3, a, "pos", np.int32)[0])
        save(k3, a, tmp_path / "s.k3st", seq)
        data = (tmp_path / "s.k3st").read_bytes()
        d = k3st.unpack(data)
        (tmp_path / "cpu.k3st").write_bytes(data[:d["payload_end"]])
        info = k3cuda.K3dStateInfo()
        k3cuda.check(k3.k3d_state_peek(str(tmp_path / "cpu.k3st").encode(), ctypes.byref(info)))
        assert info.has_latent == 0
        assert load(k3, b, tmp_path / "s.k3st")[0] == 0
        r, _ = load(k3, cpu, tmp_path / "cpu.k3st")
        assert r == 0, k3.k3d_last_message()
        ma, ka = caches(k3, a, pos)
        mc, kc = caches(k3, cpu, pos)
        for l in ka:
            assert np.array_equal(ka[l], kc[l]), l
        kv_lora = CFG["mla"]["kv_lora"]
        for l in ma:
            va, vc = bf16_f32(ma[l]), bf16_f32(mc[l])
            assert np.array_equal(va[:, kv_lora:], vc[:, kv_lora:]), l     # rope slots: exact
            rel = np.abs(va[:, :kv_lora] - vc[:, :kv_lora]) / np.maximum(np.abs(va[:, :kv_lora]), 1e-30)
            assert rel.max() <= 2.0 ** -7, (l, float(rel.max()))           # within one bf16 step
            assert (ma[l] == mc[l]).mean() >= 0.99, l
        nb, lb = step(k3, b, [seq[-1]])
        nc, lc = step(k3, cpu, [seq[-1]])
        assert max_rel_err(lc, lb) <= 1e-3
        top2 = np.sort(lb[0])[-2:]
        if top2[1] - top2[0] > 1e-3 * np.abs(lb).max():
            assert nb[0] == nc[0]


def test_sequence_of_a_batch_and_refusals(k3, tmp_path):
    with model(k3, batch=2) as a2, model(k3) as b:
        seq = advance(k3, a2, batch=2)
        pos = int(download(k3, a2, "pos", np.int32)[0])
        save(k3, a2, tmp_path / "b1.k3st", seq, b=1)
        assert load(k3, b, tmp_path / "b1.k3st")[0] == 0
        m1, k1 = caches(k3, a2, pos, b=1, batch=2)
        mb, kb = caches(k3, b, pos)
        for l in m1:
            assert np.array_equal(m1[l], mb[l]), l
        for l in k1:
            assert np.array_equal(k1[l], kb[l]), l
        assert k3.k3d_model_state_save(a2, str(tmp_path / "x").encode(), None, 0, 2) == k3cuda.K3D_EINVAL
    path = tmp_path / "b1.k3st"
    with model(k3, vocab=2048) as other:
        assert load(k3, other, path)[0] == k3cuda.K3D_EINVAL           # another architecture
    with model(k3, cap=pos - 1) as small:
        assert load(k3, small, path)[0] == k3cuda.K3D_EBOUND           # more positions than the cache
    with model(k3) as m:
        assert load(k3, m, path, cap=2)[0] == k3cuda.K3D_EBOUND         # more ids than seq_cap
        k3.k3d_clear_status()
