"""Benchmark of the B200 decode hot path (libk3cuda) and of the reference's CPU path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload moe|expert|stack]

One JSON line on rank 0. Under torchrun (N > 1) every rank owns 1/N of the routed experts
(expert parallelism), the partial MoE outputs are summed over NCCL, and the reported time
is the max over ranks of the device-timed steps.

workload "moe" (T = 1): one MoE layer decode step = bit-exact router over
384 experts, the 8 selected MXFP4 SwiGLU experts (7168 -> 2048 -> 7168) and the bf16 shared
expert. A step's input is one of 64 resident token activations, so consecutive steps route
to different experts; L2 is flushed (256 MB write) between timed steps, outside the events.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "kimi-k3-in-c_b200"))
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))

HIDDEN, INTER, N_EXPERTS, TOPK, SHARED = 7168, 2048, 384, 8, 2048
EXPERT_BYTES = 3 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 32)   # 23,396,352
METRIC = "decode tok/s at 1/2/4/8 B200; MXFP4 expert GEMV HBM GB/s vs peak"


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) > 8:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def load_traffic(name):
    p = os.path.join(REPO, "profiles", name)
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("traffic_bytes_per_launch")
        except (OSError, ValueError):
            return None
    return None


# ------------------------------------------------------------------ CPU baseline ----
def cpu_moe_sample(seconds=12.0, max_tokens=2000):
    """The reference's own k3_ops.c (oracle/_ref, else the C restatement) on one MoE layer
    decode per token: k3_router over 384 experts, 8 x (3 k3_matmul_mxfp4 + SiLU*mul) in
    top-k order, bf16 shared expert via k3_matmul_bf16. Expert bytes come from a 16-expert
    host pool (expert e uses pool[e % 16]); the arithmetic per token is the same."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as orc
    import synth
    if orc.Reference.available():
        impl, kind = orc.Reference(), "reference"
    else:
        impl, kind = orc.Oracle(), "port"
    g = synth.rng(555)
    pool = [synth.mxfp4_expert(g, HIDDEN, INTER) for _ in range(16)]
    Wr = synth.bf16_to_f32(synth.bf16_normal(g, (N_EXPERTS, HIDDEN), 0.02))
    bias = g.uniform(-0.1, 0.1, N_EXPERTS).astype(np.float32)
    sg, su = (synth.bf16_normal(g, (SHARED, HIDDEN), 0.02) for _ in range(2))
    sd = synth.bf16_normal(g, (HIDDEN, SHARED), 0.02)
    xs = synth.bf16_to_f32(synth.bf16_normal(g, (64, HIDDEN), 1.0))

    def token(x):
        idx, w = impl.router(x, Wr, bias, TOPK, 1, 2.5)
        acc = np.zeros(HIDDEN, np.float32)
        for j in range(TOPK):
            e = pool[int(idx[j]) % 16]
            gg = impl.matmul_mxfp4(x, e["p1"], e["s1"], INTER)
            uu = impl.matmul_mxfp4(x, e["p3"], e["s3"], INTER)
            act = (gg / (np.float32(1) + np.exp(-gg))).astype(np.float32) * uu
            acc += w[j] * impl.matmul_mxfp4(act, e["p2"], e["s2"], HIDDEN)
        a = impl.matmul_bf16(x, sg)
        b = impl.matmul_bf16(x, su)
        act = (a / (np.float32(1) + np.exp(-a))).astype(np.float32) * b
        return acc + impl.matmul_bf16(act, sd)

    token(xs[0])
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < max_tokens:
        token(xs[n % 64])
        n += 1
    dt = time.perf_counter() - t0
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count()))
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"{n} tokens through one config-1 MoE layer (router + 8 MXFP4 experts + "
                      f"bf16 shared expert) in {dt:.1f} s; AVX2 k3_ops.c, OpenMP"}


# --------------------------------------------------------------------- GPU arm ----
def bench_moe(args, rank, world):
    import k3cuda
    lib = k3cuda.init(0)
    per = N_EXPERTS // world
    lo, hi = rank * per, (rank + 1) * per
    import synth
    g = synth.rng(4242)
    W = synth.bf16_normal(g, (N_EXPERTS, HIDDEN), 0.02)
    bias = g.uniform(-0.1, 0.1, N_EXPERTS).astype(np.float32)
    sh = (synth.bf16_normal(g, (SHARED, HIDDEN), 0.02), synth.bf16_normal(g, (SHARED, HIDDEN), 0.02),
          synth.bf16_normal(g, (HIDDEN, SHARED), 0.02))
    mw = k3cuda.MoeWeights(HIDDEN, INTER, N_EXPERTS, TOPK, W, bias, shared=sh, seed=7, lo=lo, hi=hi,
                           add_shared=1 if rank == 0 else 0, lib=lib)
    P = 64
    xs = synth.bf16_to_f32(synth.bf16_normal(g, (P, HIDDEN), 1.0))
    X = k3cuda.DevBuf.from_array(xs, lib)
    Y = k3cuda.DevBuf(HIDDEN * 4, lib)
    nws = mw.ws_bytes(1)
    WS = k3cuda.DevBuf(nws, lib)
    FL = k3cuda.DevBuf(256 << 20, lib)
    ev = [lib.k3d_event_create() for _ in range(2)]

    def step(i):
        k3cuda.check(mw.run(Y.ptr, X.ptr + (i % P) * HIDDEN * 4, 1, WS.ptr, nws), "moe step")
        if world > 1:
            k3cuda.check(lib.k3d_ep_allreduce_f32(Y.ptr, HIDDEN), "ep combine")

    for i in range(args.warmup):
        step(i)
    k3cuda.check(lib.k3d_sync())
    barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
    lib.k3d_prof_reset()
    lib.k3d_prof_enable(1)
    lib.k3d_launch_count_reset()
    step_ms = []
    uniq = []
    for i in range(args.steps):
        lib.k3d_memset(FL.ptr, i & 0xff, FL.nbytes)      # L2 flush, outside the events
        lib.k3d_event_record(ev[0])
        step(args.warmup + i)
        lib.k3d_event_record(ev[1])
        step_ms.append(lib.k3d_event_elapsed_ms(ev[0], ev[1]))
        uniq.append(lib.k3d_moe_last_unique())
    k3cuda.check(lib.k3d_sync())
    launches = lib.k3d_launch_count() - args.steps        # minus the flush memsets
    cnt = C.c_long()
    exp_ms = lib.k3d_prof_ms(b"moe.experts", C.byref(cnt))
    n_exp = cnt.value
    lib.k3d_prof_enable(0)
    clk = clocks.stop()
    barrier()
    tot_ms = sum(step_ms)
    tot_ms = reduce_max(tot_ms)
    exp_ms_avg = exp_ms / max(1, n_exp)
    u_avg = float(np.mean(uniq))
    alg_bytes = u_avg * (EXPERT_BYTES + INTER * 8 + HIDDEN * 4) + HIDDEN * 4
    hbm, peak_kind = measured_peaks()
    achieved = alg_bytes / (exp_ms_avg * 1e-3) / 1e9
    # end to end through the public API with host buffers
    hx = lib.k3d_host_alloc(HIDDEN * 4)
    hy = lib.k3d_host_alloc(HIDDEN * 4)
    C.memmove(hx, xs[0].ctypes.data, HIDDEN * 4)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        k3cuda.check(lib.k3d_upload(X.ptr, hx, HIDDEN * 4))
        k3cuda.check(mw.run(Y.ptr, X.ptr, 1, WS.ptr, nws))
        if world > 1:
            k3cuda.check(lib.k3d_ep_allreduce_f32(Y.ptr, HIDDEN))
        k3cuda.check(lib.k3d_download(hy, Y.ptr, HIDDEN * 4))
    e2e_s = reduce_max(time.perf_counter() - t0)
    lib.k3d_host_free(hx)
    lib.k3d_host_free(hy)
    res = {
        "metric": METRIC, "value": args.steps / (tot_ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded MXFP4 experts, E8M0 117..121; bf16 ~N(0,0.02) router and "
                "shared expert; bf16 ~N(0,1) tokens)",
        "config": {"workload": "config1 MoE layer decode, T=1", "hidden": HIDDEN,
                   "n_experts": N_EXPERTS, "topk": TOPK, "inter": INTER, "shared_inter": SHARED,
                   "parallelism": f"ep{world}", "l2": "flushed between steps (256 MB write)"},
        "roofline": {"kernel": "MXFP4 expert GEMV (k_moe_gate_up + k_moe_down)", "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind,
                     "traffic": load_traffic("moe_experts_traffic.json"),
                     "alg_bytes_per_launch": alg_bytes, "unique_experts": u_avg,
                     "kernel_ms": exp_ms_avg},
        "e2e": {"value": args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": HIDDEN * 4,
                "d2h_bytes_per_step": HIDDEN * 4},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    return res


# ---------------------------------------------------------------- distributed ----
_PG = None


def barrier():
    if _PG is not None:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(v):
    if _PG is None:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def setup_dist(world, rank, local):
    global _PG
    if world <= 1:
        return
    import datetime
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    _PG = True
    # one process per GPU: the library uses the device torchrun assigned
    os.environ["CUDA_VISIBLE_DEVICES"] = str(local)
    import k3cuda
    lib = k3cuda.init(0)
    uid = (C.c_ubyte * 128)()
    if rank == 0:
        k3cuda.check(lib.k3d_ep_unique_id(uid))
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
    k3cuda.check(lib.k3d_ep_init(rank, world, uid), "ep init")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="moe", choices=["moe"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return
        cb = cpu_moe_sample(seconds=args.cpu_seconds)
        res = {"metric": METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / cb["value"],
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "fp64-accumulate/fp32", "data": "synthetic",
               "config": {"workload": "config1 MoE layer decode, T=1", "hidden": HIDDEN,
                          "n_experts": N_EXPERTS, "topk": TOPK, "parallelism": "cpu"},
               "impl": "reference", "cpu_baseline": cb,
               "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(res), flush=True)
        return
    setup_dist(world, rank, local)
    res = bench_moe(args, rank, world)
    if rank == 0:
        if world == 1:
            res["cpu_baseline"] = cpu_moe_sample(seconds=args.cpu_seconds)
        print(json.dumps(res), flush=True)
    if world > 1:
        import k3cuda
        k3cuda.load().k3d_ep_finalize()
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
