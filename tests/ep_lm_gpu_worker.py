"""One rank (one GPU) of the two-GPU vocabulary-split LM head test (test_gpu_ep_a2a.py):
this rank's rows of a seeded [vocab][hidden] matrix, the keys combined by an NCCL max."""
import datetime
import os

import numpy as np


def run(rank, world, port, seed):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    import k3cuda
    import synth
    lib = k3cuda.init(rank)
    try:
        idb = np.zeros(128, np.uint8)
        if rank == 0:
            k3cuda.check(lib.k3d_ep_unique_id(idb.ctypes.data))
        t = torch.from_numpy(idb)
        dist.broadcast(t, 0)
        idb = t.numpy().copy()
        k3cuda.check(lib.k3d_ep_init(rank, world, idb.ctypes.data), "ep init")
        vocab, hidden = 5000, 512
        g = synth.rng(seed)
        W = synth.bf16_normal(g, (vocab, hidden), 0.02)
        v0, v1 = rank * vocab // world, (rank + 1) * vocab // world
        Wd = k3cuda.DevBuf.from_array(np.ascontiguousarray(W[v0:v1]), lib)
        nw = np.ones(hidden, np.float32)
        NW = k3cuda.DevBuf.from_array(nw, lib)
        for B in (3, 6):
            x = g.standard_normal((B, hidden)).astype(np.float32)
            X = k3cuda.DevBuf.from_array(x, lib)
            nxt = k3cuda.DevBuf(B * 4, lib)
            key = k3cuda.DevBuf(B * 8, lib)
            k3cuda.check(lib.k3d_lm_head_argmax_shard_normed(nxt.ptr, None, X.ptr, NW.ptr, 1e-6, Wd.ptr, v0,
                                                             v1 - v0, hidden, B, key.ptr), "shard lm head")
            k3cuda.check(lib.k3d_sync())
            got = nxt.download(np.int32, B)
            xn = x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-6)
            logits = xn @ synth.bf16_to_f32(W).astype(np.float64).T
            for b in range(B):
                top2 = np.sort(logits[b])[-2:]
                if top2[1] - top2[0] > 1e-4 * np.abs(logits[b]).max():
                    assert got[b] == int(np.argmax(logits[b])), (B, b, got[b])
            allg = [torch.zeros(B, dtype=torch.int32) for _ in range(world)]
            dist.all_gather(allg, torch.from_numpy(got))
            assert all(np.array_equal(a.numpy(), got) for a in allg), "ranks disagree"
        k3cuda.check(lib.k3d_ep_finalize())
    finally:
        dist.destroy_process_group()
