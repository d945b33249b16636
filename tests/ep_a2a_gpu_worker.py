"""One rank (one GPU) of the two-GPU Mode A test (test_gpu_ep_a2a.py): NCCL through
k3d_ep_init (the id travels over a gloo group), this rank's experts only, its own tokens,
k3d_moe_swiglu_a2a (or, with dev, k3d_moe_swiglu_a2a_dev eagerly and as a captured
graph) against the oracle."""
import datetime
import os

import numpy as np


def run(rank, world, port, seed, tiled, dev=False):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    import k3cuda
    import synth
    from oracle import Oracle
    lib = k3cuda.init(rank)
    try:
        idb = (np.zeros(128, np.uint8))
        if rank == 0:
            k3cuda.check(lib.k3d_ep_unique_id(idb.ctypes.data))
        t = torch.from_numpy(idb)
        dist.broadcast(t, 0)
        idb = t.numpy().copy()
        k3cuda.check(lib.k3d_ep_init(rank, world, idb.ctypes.data), "ep init")
        hidden, inter, E, K, SI = 1024, 512, 16, 8, 256
        g = synth.rng(seed)
        experts = [synth.mxfp4_expert(g, hidden, inter) for _ in range(E)]
        W = synth.bf16_normal(g, (E, hidden), 0.02)
        bias = g.uniform(-0.1, 0.1, E).astype(np.float32)
        sh = (synth.bf16_normal(g, (SI, hidden), 0.02), synth.bf16_normal(g, (SI, hidden), 0.02),
              synth.bf16_normal(g, (hidden, SI), 0.02))
        per = E // world
        mw = k3cuda.MoeWeights(hidden, inter, E, K, W, bias, shared=sh, experts=experts,
                               lo=rank * per, hi=(rank + 1) * per, add_shared=1, tiled=tiled, lib=lib)
        t_max = 24
        T = 12 if dev else 5 + 19 * rank   # the host-planned form takes different batch sizes
        x = synth.bf16_to_f32(synth.bf16_normal(synth.rng(seed * 100 + rank), (T, hidden), 1.0))
        X = k3cuda.DevBuf.from_array(x, lib)
        O = k3cuda.DevBuf(T * hidden * 4, lib)
        I = k3cuda.DevBuf(T * K * 4, lib)
        n = mw.a2a_ws_bytes(T if dev else t_max, world)
        WS = k3cuda.DevBuf(n, lib)
        for _ in range(2):                 # repeated calls give the same result
            O.zero()
            if dev:
                k3cuda.check(mw.run_a2a_dev(O.ptr, X.ptr, T, WS.ptr, n, 0, I.ptr, None), "moe a2a dev")
            else:
                k3cuda.check(mw.run_a2a(O.ptr, X.ptr, T, t_max, WS.ptr, n, 0, I.ptr, None), "moe a2a")
            k3cuda.check(lib.k3d_sync(), "sync")
        y = O.download(np.float32, (T, hidden))
        if dev:
            # the same call captured into a graph (NCCL inside) and replayed twice
            k3cuda.check(lib.k3d_graph_begin())
            r = mw.run_a2a_dev(O.ptr, X.ptr, T, WS.ptr, n, 0, I.ptr, None)
            graph = lib.k3d_graph_end()
            k3cuda.check(r, "capture")
            assert graph, lib.k3d_last_message()
            for _ in range(2):
                O.zero()
                k3cuda.check(lib.k3d_graph_launch(graph), "replay")
                k3cuda.check(lib.k3d_sync(), "sync")
                assert np.array_equal(O.download(np.float32, (T, hidden)), y)
            lib.k3d_graph_destroy(graph)      # before the communicator goes
        idx = I.download(np.int32, (T, K))
        want, oi, _ = Oracle().moe_swiglu(x, T, hidden, inter, E, K, 1, 2.5, W, bias, experts, SI, *sh)
        assert np.array_equal(idx, oi)
        err = np.abs(y - want).max() / max(np.abs(want).max(), 1e-30)
        assert err <= 1e-4, err
        k3cuda.check(lib.k3d_ep_finalize())
    finally:
        dist.destroy_process_group()
