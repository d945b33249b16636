"""One rank (one GPU) of the two-GPU tests of the NVLink push combine (test_gpu_ep_combine.py).

run_combine: k3d_ep_combine_add on seeded partials of several lengths, repeated (the
parity of the receive slots alternates), with both protocols (k3d_set_ep_combine), against
the rank-order sum computed on the host; every rank must hold the same result.
run_stack: the reduced-width decode stack under expert parallelism (routed experts split
by rank, shared expert split by intermediate rows, the KDA heads, MLA heads (when they
split into multiples of 8) and dense rows split by rank, vocabulary-split LM head, the push
combine after every attention layer, dense MLP and MoE layer; eager, graph capture, replay), then rank 0 alone steps the same
seeded model on one GPU with the same tokens: logits (the ranks' vocabulary slices put
together) within 1e-5 and the same greedy tokens."""
import ctypes
import datetime
import os

import numpy as np


def _setup(rank, world, port):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    import k3cuda
    lib = k3cuda.init(rank)
    idb = np.zeros(128, np.uint8)
    if rank == 0:
        k3cuda.check(lib.k3d_ep_unique_id(idb.ctypes.data))
    t = torch.from_numpy(idb)
    dist.broadcast(t, 0)
    idb = t.numpy().copy()
    k3cuda.check(lib.k3d_ep_init(rank, world, idb.ctypes.data), "ep init")
    return lib, dist, torch


def run_combine(rank, world, port, seed):
    lib, dist, torch = _setup(rank, world, port)
    import k3cuda
    try:
        nmax = 64 * 7168
        k3cuda.check(lib.k3d_ep_peer_init(nmax), "peer init")
        sizes = [7168, 7168, 3 * 7168, nmax, 7168, 1000]
        # the tagged-word protocol, then the flag protocol, then back (both keep the
        # per-slice call counts in step)
        kinds = [0] * len(sizes) + [1] * len(sizes) + [0] * 3
        for call, (kind, n) in enumerate(zip(kinds, sizes * 2 + sizes[:3])):
            k3cuda.check(lib.k3d_set_ep_combine(kind))
            parts = [np.random.default_rng(seed * 100 + call * 10 + r).standard_normal(n).astype(np.float32)
                     for r in range(world)]
            h0 = np.random.default_rng(seed * 100 + call).standard_normal(n).astype(np.float32)
            H = k3cuda.DevBuf.from_array(h0, lib)
            P = k3cuda.DevBuf.from_array(parts[rank], lib)
            k3cuda.check(lib.k3d_ep_combine_add(H.ptr, P.ptr, n, 1), f"combine {call}")
            k3cuda.check(lib.k3d_sync(), f"combine {call} sync")
            got = H.download(np.float32, n)
            v = parts[0].copy()
            for r in range(1, world):
                v = (v + parts[r]).astype(np.float32)
            want = (h0 + v).astype(np.float32)
            assert np.array_equal(got, want), (call, float(np.abs(got - want).max()))
            allg = [torch.zeros(n, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(allg, torch.from_numpy(got))
            assert all(np.array_equal(a.numpy(), got) for a in allg), "ranks disagree"
        k3cuda.check(lib.k3d_ep_finalize())
    finally:
        dist.destroy_process_group()


def run_stack(rank, world, port, seed, batch, mla_heads=None):
    lib, dist, torch = _setup(rank, world, port)
    import k3cuda
    from test_gpu_stack import CFG, make_cfg, download
    try:
        c = CFG
        if mla_heads:      # 16 heads split over 2 ranks: the MLA layers run tensor-parallel too
            c = dict(CFG, mla=dict(CFG["mla"], H=mla_heads))
        E = c["moe"]["n_experts"]

        def model_cfg(lo, hi, add_shared):
            sc = make_cfg(c, batch=batch, layout=1)
            sc.moe.expert_lo, sc.moe.expert_hi, sc.moe.add_shared = lo, hi, add_shared
            return sc

        V = c["vocab"]

        def full_logits(raw, nr):
            """Under expert parallelism each rank's logits buffer holds its vocabulary slice,
            [batch][vshard] from the start; the slices of all ranks make the whole row."""
            if nr == 1:
                return raw.reshape(batch, V).copy()
            allg = [torch.zeros(raw.size, dtype=torch.float32) for _ in range(nr)]
            dist.all_gather(allg, torch.from_numpy(raw))
            parts = []
            for r in range(nr):
                v0, v1 = r * V // nr, (r + 1) * V // nr
                parts.append(allg[r].numpy()[:batch * (v1 - v0)].reshape(batch, v1 - v0))
            return np.concatenate(parts, axis=1)

        def steps(model, toks, nr):
            out, logs = [], []
            for step in range(3):            # eager, graph capture, replay
                nxt = np.zeros(batch, np.int32)
                k3cuda.check(lib.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data), f"step {step}")
                logs.append(full_logits(download(lib, model, "logits", np.float32), nr))
                out.append(nxt.copy())
                toks = nxt.copy()
            return out, logs

        toks0 = ((np.arange(batch) * 37 + 5) % c["vocab"]).astype(np.int32)
        lo, hi = rank * E // world, (rank + 1) * E // world
        model = lib.k3d_model_create(ctypes.byref(model_cfg(lo, hi, 1 if rank == 0 else 0)), seed)
        assert model, lib.k3d_last_message()
        k3cuda.check(lib.k3d_model_fill_context(model, 6, 17))
        toks_ep, logs_ep = steps(model, toks0, world)
        lib.k3d_model_destroy(model)           # releases the graph (it holds an NCCL call)
        k3cuda.check(lib.k3d_sync())
        for t in toks_ep:
            allg = [torch.zeros(batch, dtype=torch.int32) for _ in range(world)]
            dist.all_gather(allg, torch.from_numpy(t))
            assert all(np.array_equal(a.numpy(), t) for a in allg), "ranks disagree on tokens"
        k3cuda.check(lib.k3d_ep_finalize())
        if rank == 0:
            assert lib.k3d_ep_size() == 1
            model = lib.k3d_model_create(ctypes.byref(model_cfg(0, E, 1)), seed)
            assert model, lib.k3d_last_message()
            k3cuda.check(lib.k3d_model_fill_context(model, 6, 17))
            toks_1, logs_1 = steps(model, toks0, 1)
            lib.k3d_model_destroy(model)
            for s in range(3):
                a, b = logs_ep[s], logs_1[s]
                err = float(np.abs(a - b).max() / np.abs(b).max())
                assert err <= 1e-5, (s, err)
                for q in range(batch):
                    top2 = np.sort(b[q])[-2:]
                    if top2[1] - top2[0] > 1e-4 * np.abs(b[q]).max():
                        assert toks_ep[s][q] == toks_1[s][q], (s, q)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def run_stack_mode_a(rank, world, port, seed, batch):
    """Mode A: the batch split over the ranks (rank r steps the global sequences
    [r b, (r + 1) b), b = batch / world, with its own caches), experts split, every MoE layer
    through the device-planned all-to-all; eager, captured, replayed. Rank 0 then steps the
    whole batch on one GPU: the ranks' logits put together within 1e-5 and the same tokens."""
    lib, dist, torch = _setup(rank, world, port)
    import k3cuda
    from test_gpu_stack import CFG, make_cfg, download
    try:
        c = CFG
        E, V = c["moe"]["n_experts"], c["vocab"]
        b = batch // world

        def steps(model, toks, nb):
            out, logs = [], []
            for step in range(3):
                nxt = np.zeros(nb, np.int32)
                k3cuda.check(lib.k3d_model_step_host(model, toks.ctypes.data, nxt.ctypes.data), f"step {step}")
                logs.append(download(lib, model, "logits", np.float32)[:nb * V].reshape(nb, V).copy())
                out.append(nxt.copy())
                toks = nxt.copy()
            return out, logs

        toks_all = ((np.arange(batch) * 37 + 5) % V).astype(np.int32)
        sc = make_cfg(c, batch=b, layout=1)
        sc.moe.expert_lo, sc.moe.expert_hi = rank * E // world, (rank + 1) * E // world
        sc.ep_tokens = 1
        model = lib.k3d_model_create(ctypes.byref(sc), seed)
        assert model, lib.k3d_last_message()
        k3cuda.check(lib.k3d_model_fill_context(model, 6, 17))
        toks_ep, logs_ep = steps(model, toks_all[rank * b:(rank + 1) * b].copy(), b)
        lib.k3d_model_destroy(model)           # releases the graph (it holds NCCL calls)
        k3cuda.check(lib.k3d_sync())
        gathered = []
        for s in range(3):
            tl = [torch.zeros(b, dtype=torch.int32) for _ in range(world)]
            dist.all_gather(tl, torch.from_numpy(toks_ep[s]))
            ll = [torch.zeros(b * V, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(ll, torch.from_numpy(logs_ep[s].reshape(-1)))
            gathered.append((np.concatenate([t.numpy() for t in tl]),
                             np.concatenate([x.numpy().reshape(b, V) for x in ll])))
        k3cuda.check(lib.k3d_ep_finalize())
        if rank == 0:
            sc1 = make_cfg(c, batch=batch, layout=1)
            model = lib.k3d_model_create(ctypes.byref(sc1), seed)
            assert model, lib.k3d_last_message()
            k3cuda.check(lib.k3d_model_fill_context(model, 6, 17))
            toks_1, logs_1 = steps(model, toks_all.copy(), batch)
            lib.k3d_model_destroy(model)
            for s in range(3):
                t_ep, l_ep = gathered[s]
                err = float(np.abs(l_ep - logs_1[s]).max() / np.abs(logs_1[s]).max())
                assert err <= 1e-5, (s, err)
                for q in range(batch):
                    top2 = np.sort(logs_1[s][q])[-2:]
                    if top2[1] - top2[0] > 1e-4 * np.abs(logs_1[s][q]).max():
                        assert t_ep[q] == toks_1[s][q], (s, q)
        dist.barrier()
    finally:
        dist.destroy_process_group()
