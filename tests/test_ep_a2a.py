"""Mode A expert parallelism (all-to-all dispatch and combine of data-parallel tokens) on
the CPU: the host dispatch plan (k3d_a2a_plan, no device work) and the whole protocol on
two gloo ranks, each with its own batch, whose experts run in the oracle; the result must
equal the single-process oracle MoE bit for bit."""
import socket

import numpy as np
import pytest

import k3cuda


def test_a2a_plan_groups_rows_by_rank_in_assignment_order():
    rng = np.random.default_rng(5)
    for nranks in (1, 2, 4, 8):
        E = 32
        idx = rng.integers(0, E, size=(37, 6)).astype(np.int32)
        cnt, off, pos = k3cuda.a2a_plan(idx, E, nranks)
        per = E // nranks
        owner = idx.reshape(-1) // per
        assert cnt.sum() == idx.size
        assert np.array_equal(cnt, np.bincount(owner, minlength=nranks))
        assert np.array_equal(off, np.concatenate([[0], np.cumsum(cnt)[:-1]]))
        assert np.array_equal(np.sort(pos), np.arange(idx.size))       # a permutation
        for r in range(nranks):
            rows = pos[owner == r]
            assert np.array_equal(rows, np.arange(off[r], off[r] + cnt[r]))   # in order


def test_a2a_plan_rejects_bad_input():
    lib = k3cuda.load()
    with pytest.raises(RuntimeError):
        k3cuda.a2a_plan(np.array([0, 9], np.int32), 8, 2, lib)        # id out of range
    with pytest.raises(RuntimeError):
        k3cuda.a2a_plan(np.array([0, 1], np.int32), 9, 2, lib)        # 9 experts over 2 ranks
    lib.k3d_clear_status()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_a2a_protocol_two_gloo_ranks_matches_oracle():
    # ranks are fresh interpreters (spawn) that import torch before libk3cuda; this process
    # may already hold libk3cuda (and the system NCCL it links), so it does not import torch
    import multiprocessing as mp
    import ep_a2a_worker
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=ep_a2a_worker.run, args=(r, 2, port, 17)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes
