"""Config 4 at full width: the exact model bench.py times (bench.stack_cfg: hidden 7168, 384
MXFP4 experts top-8 + bf16 shared expert, 64-head KDA and MLA, dense layer 18432, vocab
163840, tiled experts on the tcgen05 path), stepped eagerly, then captured and replayed as a
CUDA graph, against the oracle stepping the same weights and context on the host.

The trunk (about 10 GB of bf16) is copied to the host once; the routed experts stay on the
device and only those the oracle's router selects are downloaded (DeviceExperts). MLA runs
in the oracle's absorbed form, which the CPU tests pin to the expanded form and that to the
reference's k3_mla_cached.
"""
import ctypes
import os
import sys

import numpy as np
import pytest

import k3cuda
from conftest import REPO, max_rel_err
import oracle as orc_mod
from test_gpu_stack import download, host_copy, sequence_state

sys.path.insert(0, REPO)
import bench  # noqa: E402  (the benchmark's own model configuration)

pytestmark = pytest.mark.gpu

FULL = dict(hidden=7168, vocab=163840, n_layers=8, eps=1e-6, kda_heads=64, kda_head_dim=128,
            conv_k=4, gate_lb=-5.0, first_dense=1, dense_inter=18432, mla_layers=[3, 7],
            mla=dict(hidden=7168, H=64, q_lora=1536, kv_lora=512, qn=128, qr=64, vh=128,
                     theta=50000.0, eps=1e-6),
            moe=dict(inter=2048, n_experts=384, topk=8, routed_scale=2.5, shared_inter=2048),
            mla_absorbed=True)


def check_cfg_matches_bench(sc):
    """The test's host-side description must be the benchmark's model."""
    c = FULL
    assert (sc.hidden, sc.vocab, sc.n_layers) == (c["hidden"], c["vocab"], c["n_layers"])
    assert (sc.kda_heads, sc.kda_head_dim, sc.conv_k) == (c["kda_heads"], c["kda_head_dim"],
                                                          c["conv_k"])
    assert (sc.mla.n_heads, sc.mla.q_lora, sc.mla.kv_lora) == (64, 1536, 512)
    assert (sc.moe.inter, sc.moe.n_experts, sc.moe.topk) == (2048, 384, 8)
    assert (sc.first_dense, sc.dense_inter) == (1, 18432)
    assert [sc.mla_layers[i] for i in range(2)] == c["mla_layers"]
    assert sc.moe.expert_layout == 1


def make_model(k3, batch, ctx):
    cap = ctx + 8
    sc = bench.stack_cfg(1, 0, batch, cap)
    check_cfg_matches_bench(sc)
    model = k3.k3d_model_create(ctypes.byref(sc), 2024)
    assert model, k3.k3d_last_message()
    k3cuda.check(k3.k3d_model_fill_context(model, ctx, 77))
    k3cuda.check(k3.k3d_sync())
    return model, cap


def test_full_width_stack_batch1_matches_oracle(k3, oracle):
    ctx = 64
    model, cap = make_model(k3, 1, ctx)
    try:
        W, S = host_copy(k3, model, FULL, layout=1, batch=1, cap=cap, lazy_experts=True)
        assert S["pos"] == ctx
        tok = 12345
        for step in range(3):           # step 0 eager, step 1 captures the graph, 2 replays
            ids = np.array([tok], np.int32)
            nxt = np.zeros(1, np.int32)
            k3cuda.check(k3.k3d_model_step_host(model, ids.ctypes.data, nxt.ctypes.data),
                         f"step {step}")
            got = download(k3, model, "logits", np.float32)
            want = orc_mod.stack_step(oracle, FULL, W, S, tok)
            err = max_rel_err(got, want)
            assert err <= 1e-3, (step, err)
            top2 = np.sort(want)[-2:]
            if top2[1] - top2[0] > 1e-3 * np.abs(want).max():
                assert nxt[0] == int(np.argmax(want)), step
            tok = int(nxt[0])
        assert int(download(k3, model, "pos", np.int32)[0]) == ctx + 3
    finally:
        k3.k3d_model_destroy(model)


def test_full_width_stack_batch64_matches_oracle_per_sequence(k3, oracle):
    """Batch 64 (every projection on the tensor-core GEMM, the grouped expert pass over
    ~280 distinct experts per layer): three of the 64 sequences, first, middle and last,
    each stepped alone by the oracle from its own cache and state."""
    B, ctx = 64, 32
    model, cap = make_model(k3, B, ctx)
    try:
        W, S = host_copy(k3, model, FULL, layout=1, batch=B, cap=cap, lazy_experts=True)
        picks = (0, 29, 63)
        seqs = {b: sequence_state(FULL, S, b, B) for b in picks}
        del S
        toks = ((np.arange(B) * 2557 + 11) % FULL["vocab"]).astype(np.int32)
        for step in range(2):           # eager, then the captured graph
            nxt = np.zeros(B, np.int32)
            k3cuda.check(k3.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data),
                         f"step {step}")
            got = download(k3, model, "logits", np.float32).reshape(B, FULL["vocab"])
            for b in picks:
                want = orc_mod.stack_step(oracle, FULL, W, seqs[b], int(toks[b]))
                err = max_rel_err(got[b], want)
                assert err <= 1e-3, (step, b, err)
                top2 = np.sort(want)[-2:]
                if top2[1] - top2[0] > 1e-3 * np.abs(want).max():
                    assert nxt[b] == int(np.argmax(want)), (step, b)
            toks = nxt.copy()
    finally:
        k3.k3d_model_destroy(model)
