"""One gloo rank of the Mode A protocol test (test_ep_a2a.py): the rank's own tokens are
routed by the oracle, dispatched with libk3cuda's host plan (k3d_a2a_plan) over
all_to_all_single, run through the oracle's experts on the owning rank, sent back and
summed in top-k order with the shared expert, exactly as k3d_moe_swiglu_a2a orders it."""
import datetime
import os

import numpy as np

# torch is imported inside the rank functions only: the parent test process may already
# hold libk3cuda and the system NCCL it links, which torch's own CUDA library must not meet

HIDDEN, INTER, E, K, SI = 128, 64, 8, 3, 64


def layer(seed):
    import synth
    g = synth.rng(seed)
    experts = [synth.mxfp4_expert(g, HIDDEN, INTER) for _ in range(E)]
    W = synth.bf16_normal(g, (E, HIDDEN), 0.02)
    bias = g.uniform(-0.1, 0.1, E).astype(np.float32)
    sh = (synth.bf16_normal(g, (SI, HIDDEN), 0.02), synth.bf16_normal(g, (SI, HIDDEN), 0.02),
          synth.bf16_normal(g, (HIDDEN, SI), 0.02))
    return experts, W, bias, sh


def tokens(seed, rank):
    import synth
    T = 3 + 2 * rank                      # ranks hold different batch sizes
    return synth.bf16_to_f32(synth.bf16_normal(synth.rng(seed * 100 + rank), (T, HIDDEN), 1.0))


def exchange(send, scnt, rcnt, tail=()):
    import torch
    import torch.distributed as dist
    out = torch.empty((int(sum(rcnt)),) + tuple(tail), dtype=send.dtype)
    dist.all_to_all_single(out, send, output_split_sizes=[int(c) for c in rcnt],
                           input_split_sizes=[int(c) for c in scnt])
    return out


def run(rank, world, port, seed):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        import k3cuda
        from oracle import Oracle
        orc = Oracle()
        lib = k3cuda.load()
        experts, W, bias, sh = layer(seed)
        x = tokens(seed, rank)
        T = x.shape[0]
        routes = [orc.router_bf16(x[t], W, bias, K, 1, 2.5) for t in range(T)]
        idx = np.stack([r[0] for r in routes]).astype(np.int32)
        wts = np.stack([r[1] for r in routes]).astype(np.float32)
        cnt, off, pos = k3cuda.a2a_plan(idx, E, world, lib)
        rcnt = exchange(torch.from_numpy(cnt.astype(np.int64)), [1] * world, [1] * world).numpy()
        send = np.empty((T * K, HIDDEN), np.float32)
        sid = np.empty(T * K, np.int32)
        for a in range(T * K):
            send[pos[a]] = x[a // K]
            sid[pos[a]] = idx.flat[a]
        recv = exchange(torch.from_numpy(send), cnt, rcnt, (HIDDEN,)).numpy()
        rid = exchange(torch.from_numpy(sid), cnt, rcnt).numpy()
        per = E // world
        y = np.empty_like(recv)
        for j in range(recv.shape[0]):
            assert rid[j] // per == rank, "row sent to the wrong rank"
            y[j] = orc.expert_swiglu(recv[j], experts[rid[j]], HIDDEN, INTER)
        back = exchange(torch.from_numpy(y), rcnt, cnt, (HIDDEN,)).numpy()
        out = np.zeros((T, HIDDEN), np.float32)
        for t in range(T):
            for k in range(K):
                out[t] = out[t] + np.float32(wts[t, k]) * back[pos[t * K + k]]
        # the shared expert alone: the oracle layer with no routed expert in range
        shared_only, _, _ = orc.moe_swiglu(x, T, HIDDEN, INTER, E, K, 1, 2.5, W, bias, experts, SI,
                                           *sh, lo=0, hi=0)
        out = out + shared_only
        want, oi, ow = orc.moe_swiglu(x, T, HIDDEN, INTER, E, K, 1, 2.5, W, bias, experts, SI, *sh)
        assert np.array_equal(idx, oi)
        assert np.array_equal(wts.view(np.uint32), ow.view(np.uint32))
        assert np.array_equal(out, want), float(np.abs(out - want).max())
    finally:
        dist.destroy_process_group()
