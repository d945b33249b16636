"""Benchmark of the B200 decode hot path (libk3cuda) and of the reference's CPU path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload stack|moe|moe_a2a|kda_prefill]

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
EXPERT_KERNEL = {0: "MXFP4 expert GEMV, tcgen05 kind::mxf4 block-scaled MMA (k_mxfp4_umma gate/up + down)",
                 1: "MXFP4 expert GEMV, mma.sync m16n8k16 (k_mxfp4_mma gate/up + down)",
                 2: "MXFP4 expert GEMV, CUDA cores (k_moe_gate_up + k_moe_down)",
                 3: "MXFP4 expert GEMV, tcgen05 kind::mxf4 block-scaled MMA, one token per item",
                 4: "MXFP4 expert GEMV, tcgen05 kind::mxf4 block-scaled MMA, gate/up + act split + down "
                    "in one launch (k_mxfp4_fused)"}


def expert_kernel_ms(lib, sections=None):
    """Device time per MoE layer of the expert launches from the section timers: the fused
    launch when it ran, else the gate/up and down launches (the act split between them is
    not counted, as before)."""
    out = {}
    for name in ("experts.fused", "experts.gateup", "experts.down"):
        c = C.c_long()
        ms = lib.k3d_prof_ms(name.encode(), C.byref(c))
        if c.value:
            out[name] = ms / c.value
    if "experts.fused" in out:
        return out["experts.fused"], out
    return out.get("experts.gateup", float("nan")) + out.get("experts.down", float("nan")), out


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
    """nvidia-smi clocks and throttle reasons sampled every 100 ms by rank 0 on its own
    GPU. Under several ranks any query during the timed steps stalls the push combines
    (the caller then samples a second pass of the same steps instead)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu=None):
        rank, world, local = dist_env()
        self.active = rank == 0
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        me = local if gpu is None else gpu
        self.gpus = [vis[me] if me < len(vis) else str(me)]
        self.rows = []
        self.proc = None

    def start(self):
        if not self.active:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(self.gpus), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0:   # first sample before timing
                time.sleep(0.02)
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if not self.active:
            return None
        t0 = time.time()
        n0 = len(self.rows)
        while self.proc and len(self.rows) < n0 + 2 * len(self.gpus) and time.time() - t0 < 2.0:
            time.sleep(0.02)                                     # a sample after the region
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
                "samples": len(sm), "gpus": len(self.gpus)}


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

    cores, cpu_model, _ = cpu_threads(impl.lib)
    token(xs[0])
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < max_tokens:
        token(xs[n % 64])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": kind, "cpu_model": cpu_model,
            "sample": f"{n} tokens through one config-1 MoE layer (router + 8 MXFP4 experts + "
                      f"bf16 shared expert) in {dt:.1f} s; AVX2 k3_ops.c, OpenMP"}


def cpu_threads(lib):
    """Sets the OpenMP thread count of the CPU arm explicitly, whatever the launcher put in
    OMP_NUM_THREADS (torchrun exports 1): one thread per physical core the process may run
    on. Returns (threads in force, CPU model)."""
    import psutil
    aff = len(os.sched_getaffinity(0))
    phys = psutil.cpu_count(logical=False) or aff
    n = max(1, min(aff, phys))
    gomp = C.CDLL("libgomp.so.1")              # the instance libk3ref.so is linked with
    gomp.omp_set_num_threads(C.c_int(n))
    got = int(gomp.omp_get_max_threads())
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return got, model, gomp


def fnv1a(a):
    """FNV-1a over the bytes of an array (the reference bench_kernels.c output hash)."""
    h = 1469598103934665603
    for b in np.ascontiguousarray(a).view(np.uint8).tobytes():
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


def cpu_stack_run(context=4096, reps=5, one_thread_reps=2):
    """The reference's own k3_ops.c (oracle/_ref/libk3ref.so; the C restatement when absent)
    running whole config-4 decode tokens at full width on the host cores: 8 layers (KDA at
    0-based 0,1,2,4,5,6 through k3_kda_layer with all 64 heads; MLA at 3 and 7 through
    k3_mla_cached over `context` cached positions in its fp32 expanded cache), the dense
    SwiGLU layer and the seven config-1 MoE layers composed from k3_rmsnorm, k3_matmul_bf16,
    k3_router and k3_matmul_mxfp4 (SURVEY's per-config composition), then the final norm and
    the 163840-row LM head with argmax. bf16 weights ~N(0, 0.02) (a 32 MB seeded block tiled
    over each matrix: the bytes read per token are the full model's), MXFP4 experts from a
    pool of 32 distinct experts (expert e reads pool[e % 32], 749 MB). One warm-up token,
    then `reps` timed tokens on all physical cores and `one_thread_reps` on one core."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as orc
    import synth
    if orc.Reference.available():
        impl, kind, pre = orc.Reference(), "reference", "k3_"
    else:
        impl, kind, pre = orc.Oracle(), "port", "orc_"
    lib = impl.lib
    threads, cpu_model, gomp = cpu_threads(lib)
    g = synth.rng(2029)
    E, V, P, H, D = HIDDEN, 163840, 64 * 128, 64, 128
    block = synth.bf16_normal(g, (1 << 24,), 0.02)

    def bf16(shape):
        a = np.empty(shape, np.uint16)
        f = a.reshape(-1)
        for o in range(0, f.size, block.size):
            n = min(block.size, f.size - o)
            f[o:o + n] = block[:n]
        return a

    vp = C.c_void_p
    fn = {}
    for name, args in (("rmsnorm", [vp, vp, vp, C.c_int, C.c_float]),
                       ("matmul_bf16", [vp, vp, vp, C.c_int, C.c_int]),
                       ("matmul_mxfp4", [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int]),
                       ("router", [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float])):
        f = getattr(lib, pre + name)
        f.argtypes, f.restype = args, None
        fn[name] = f
    kda = getattr(lib, pre + "kda_layer")
    kda.argtypes = [vp, vp, C.POINTER(orc.K3KdaW), C.POINTER(orc.K3Cfg), C.c_int, vp, vp]
    kda.restype = None
    ksz = getattr(lib, pre + "kda_scratch")
    ksz.argtypes, ksz.restype = [C.POINTER(orc.K3Cfg), C.c_int], C.c_size_t
    mla = getattr(lib, pre + "mla_cached")
    mla.argtypes = [vp, vp, C.POINTER(orc.K3MlaW), C.POINTER(orc.K3Cfg), C.c_int, vp, vp, vp,
                    C.c_int, C.c_int]
    mla.restype = None
    msz = getattr(lib, pre + "mla_scratch_cached")
    msz.argtypes, msz.restype = [C.POINTER(orc.K3Cfg), C.c_int, C.c_int, C.c_int], C.c_size_t

    kcfg = orc.K3Cfg(hidden=E, kda_heads=H, kda_head_dim=D, conv_k=4, gate_lb=-5.0, rms_eps=1e-6)
    mcfg = orc.K3Cfg(hidden=E, n_heads=64, q_lora=1536, kv_lora=512, qk_nope=128, qk_rope=64,
                     v_head=128, mla_out_gate=1, rms_eps=1e-6)
    cap = context + 1
    layers = []
    keep = []
    for l in range(8):
        L = {"in_norm": np.ones(E, np.float32), "post_norm": np.ones(E, np.float32)}
        if l in (3, 7):
            w = {"q_a": bf16((1536, E)), "q_b": bf16((64 * 192, 1536)), "kv_a": bf16((576, E)),
                 "kv_b": bf16((64 * 256, 512)), "o": bf16((E, 64 * 128)), "g": bf16((64 * 128, E)),
                 "q_a_norm": np.ones(1536, np.float32), "kv_a_norm": np.ones(512, np.float32)}
            keep.append(w)
            L["mla"] = orc.K3MlaW(*(w[k].ctypes.data for k in ("q_a", "q_b", "kv_a", "kv_b", "o",
                                                                 "g", "q_a_norm", "kv_a_norm")), 1)
            kvc = np.empty((cap, 64 * 256), np.float32)
            kvc.reshape(-1)[:] = np.resize(synth.bf16_to_f32(block), kvc.size) * np.float32(50.0)
            L["kvc"], L["ropec"] = kvc, g.standard_normal((cap, 64), dtype=np.float32)
        else:
            w = {k: bf16(shp) for k, shp in (("q", (P, E)), ("k", (P, E)), ("v", (P, E)),
                                            ("g", (P, E)), ("b", (H, E)), ("f_a", (D, E)),
                                            ("f_b", (P, D)), ("o", (E, P)))}
            for k in ("q_conv", "k_conv", "v_conv"):
                w[k] = g.standard_normal(P * 4, dtype=np.float32) * np.float32(0.5)
            w["A_log"] = g.uniform(0, 1.5, H).astype(np.float32)
            w["dt_bias"] = g.standard_normal(P, dtype=np.float32) * np.float32(0.5)
            w["o_norm"] = np.ones(D, np.float32)
            keep.append(w)
            L["kda"] = orc.K3KdaW(*(w[k].ctypes.data for k in (
                "q", "k", "v", "q_conv", "k_conv", "v_conv", "f_a", "f_b", "A_log", "dt_bias",
                "b", "g", "o_norm", "o")), 1)
            L["state"] = g.standard_normal(H * D * D + 3 * P * 3, dtype=np.float32) * np.float32(0.01)
        if l == 0:
            L["dense"] = (bf16((18432, E)), bf16((18432, E)), bf16((E, 18432)))
        else:
            L["router"] = synth.bf16_to_f32(bf16((N_EXPERTS, E)))
            L["bias"] = g.uniform(-0.1, 0.1, N_EXPERTS).astype(np.float32)
            L["shared"] = (bf16((SHARED, E)), bf16((SHARED, E)), bf16((E, SHARED)))
        layers.append(L)
    pool = [synth.mxfp4_expert(g, E, INTER) for _ in range(32)]
    lm_head = bf16((V, E))
    final_norm = np.ones(E, np.float32)
    kscr = np.empty(ksz(C.byref(kcfg), 1) + 64, np.float32)
    mscr = np.empty(msz(C.byref(mcfg), 1, cap, 1) + 64, np.float32)
    x0 = synth.bf16_to_f32(block[:E].copy()) * np.float32(50.0)
    buf = {k: np.empty(n, np.float32) for k, n in (("xn", E), ("out", E), ("g", 18432),
                                                   ("u", 18432), ("e", E), ("lg", V))}
    idx, wt = np.empty(TOPK, np.int32), np.empty(TOPK, np.float32)

    def mm(y, x, W):
        fn["matmul_bf16"](y.ctypes.data, x.ctypes.data, W.ctypes.data, W.shape[1], W.shape[0])
        return y

    def swiglu(x, Wg, Wu, Wd, out):
        n = Wg.shape[0]
        a = mm(buf["g"][:n], x, Wg)
        b = mm(buf["u"][:n], x, Wu)
        act = ((a / (np.float32(1) + np.exp(-a))) * b).astype(np.float32)
        return mm(out, act, Wd)

    def token():
        h = x0.copy()
        xn, out = buf["xn"], buf["out"]
        for l, L in enumerate(layers):
            fn["rmsnorm"](xn.ctypes.data, h.ctypes.data, L["in_norm"].ctypes.data, E, C.c_float(1e-6))
            if "mla" in L:
                mla(out.ctypes.data, xn.ctypes.data, C.byref(L["mla"]), C.byref(mcfg), 1,
                    mscr.ctypes.data, L["kvc"].ctypes.data, L["ropec"].ctypes.data, context, cap)
            else:
                kda(out.ctypes.data, xn.ctypes.data, C.byref(L["kda"]), C.byref(kcfg), 1,
                    L["state"].ctypes.data, kscr.ctypes.data)
            h += out
            fn["rmsnorm"](xn.ctypes.data, h.ctypes.data, L["post_norm"].ctypes.data, E, C.c_float(1e-6))
            if "dense" in L:
                h += swiglu(xn, *L["dense"], out)
                continue
            fn["router"](idx.ctypes.data, wt.ctypes.data, xn.ctypes.data, L["router"].ctypes.data,
                         L["bias"].ctypes.data, E, N_EXPERTS, TOPK, 1, C.c_float(2.5))
            acc = np.zeros(E, np.float32)
            for j in range(TOPK):
                e = pool[int(idx[j]) % len(pool)]
                a, b = buf["g"][:INTER], buf["u"][:INTER]
                fn["matmul_mxfp4"](a.ctypes.data, xn.ctypes.data, e["p1"].ctypes.data,
                                   e["s1"].ctypes.data, E, INTER, 32)
                fn["matmul_mxfp4"](b.ctypes.data, xn.ctypes.data, e["p3"].ctypes.data,
                                   e["s3"].ctypes.data, E, INTER, 32)
                act = ((a / (np.float32(1) + np.exp(-a))) * b).astype(np.float32)
                fn["matmul_mxfp4"](buf["e"].ctypes.data, act.ctypes.data, e["p2"].ctypes.data,
                                   e["s2"].ctypes.data, INTER, E, 32)
                acc += wt[j] * buf["e"]
            h += acc + swiglu(xn, *L["shared"], out)
        fn["rmsnorm"](xn.ctypes.data, h.ctypes.data, final_norm.ctypes.data, E, C.c_float(1e-6))
        mm(buf["lg"], xn, lm_head)
        return int(np.argmax(buf["lg"]))

    def timed(n):
        ts = []
        for _ in range(n):
            t0 = time.perf_counter()
            token()
            ts.append(time.perf_counter() - t0)
        return ts

    token()                                               # warm-up
    ts = timed(reps)
    digest = fnv1a(buf["lg"])
    gomp.omp_set_num_threads(1)
    ts1 = timed(one_thread_reps)
    gomp.omp_set_num_threads(threads)
    best, med = min(ts), statistics.median(ts)
    return {"value": 1.0 / med, "unit": "tok/s", "cores": threads, "kind": kind,
            "best_tok_s": 1.0 / best, "median_tok_s": 1.0 / med,
            "one_thread_tok_s": 1.0 / statistics.median(ts1), "reps": reps,
            "one_thread_reps": one_thread_reps, "cpu_model": cpu_model,
            "logits_fnv1a": digest,
            "sample": f"{reps} whole config-4 tokens (8 layers at full width, context {context}, "
                      f"LM head 163840 x 7168) after one warm-up, median {med * 1e3:.0f} ms, best "
                      f"{best * 1e3:.0f} ms on {threads} threads; one thread "
                      f"{statistics.median(ts1) * 1e3:.0f} ms; AVX2 k3_ops.c (-mavx2 -mfma: the "
                      "path -march=native selects on an AVX-512 host), OpenMP"}


# --------------------------------------------------------------------- GPU arm ----
def bench_moe(args, rank, world):
    import k3cuda
    lib = k3cuda.init(0)
    k3cuda.check(lib.k3d_set_expert_kernel(args.expert_kernel))
    n_exp = args.n_experts
    per = n_exp // world
    lo, hi = rank * per, (rank + 1) * per
    import synth
    g = synth.rng(4242)
    W = synth.bf16_normal(g, (n_exp, HIDDEN), 0.02)
    bias = g.uniform(-0.1, 0.1, n_exp).astype(np.float32)
    sh = (synth.bf16_normal(g, (SHARED, HIDDEN), 0.02), synth.bf16_normal(g, (SHARED, HIDDEN), 0.02),
          synth.bf16_normal(g, (HIDDEN, SHARED), 0.02))
    mw = k3cuda.MoeWeights(HIDDEN, INTER, n_exp, TOPK, W, bias, shared=sh, seed=7, lo=lo, hi=hi,
                           add_shared=1 if rank == 0 else 0, tiled=args.expert_kernel in (0, 3, 4),
                           lib=lib)
    T = max(1, args.tokens)
    P = 64 if T == 1 else 8
    xs = synth.bf16_to_f32(synth.bf16_normal(g, (P * T, HIDDEN), 1.0))
    X = k3cuda.DevBuf.from_array(xs, lib)
    Y = k3cuda.DevBuf(T * HIDDEN * 4, lib)
    nws = mw.ws_bytes(T)
    WS = k3cuda.DevBuf(nws, lib)
    FL = k3cuda.DevBuf(256 << 20, lib)
    ev = [lib.k3d_event_create() for _ in range(2)]

    def step(i):
        k3cuda.check(mw.run(Y.ptr, X.ptr + (i % P) * T * HIDDEN * 4, T, WS.ptr, nws), "moe step")
        if world > 1:
            k3cuda.check(lib.k3d_ep_allreduce_f32(Y.ptr, T * HIDDEN), "ep combine")

    for i in range(args.warmup):
        step(i)
    k3cuda.check(lib.k3d_sync())
    barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
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
    clk = clocks.stop()
    # per-kernel device times from a separate pass with the section timers on (they run
    # the shared expert in line instead of on the side stream); same kernels, same inputs
    lib.k3d_prof_reset()
    lib.k3d_prof_enable(1)
    for i in range(min(args.steps, 20)):
        lib.k3d_memset(FL.ptr, i & 0xff, FL.nbytes)
        step(args.warmup + i)
    k3cuda.check(lib.k3d_sync())
    cnt = C.c_long()
    exp_ms = lib.k3d_prof_ms(b"moe.experts", C.byref(cnt))
    n_prof = cnt.value
    kern_ms, _ = expert_kernel_ms(lib)
    lib.k3d_prof_enable(0)
    barrier()
    tot_ms = sum(step_ms)
    tot_ms = reduce_max(tot_ms)
    exp_ms_avg = exp_ms / max(1, n_prof)
    u_avg = float(np.mean(uniq))
    alg_bytes = u_avg * EXPERT_BYTES + T * TOPK * (INTER * 8 + HIDDEN * 4) + T * HIDDEN * 4
    hbm, peak_kind = measured_peaks()
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    # end to end through the public API with host buffers
    hx = lib.k3d_host_alloc(T * HIDDEN * 4)
    hy = lib.k3d_host_alloc(T * HIDDEN * 4)
    C.memmove(hx, xs[:T].ctypes.data, T * HIDDEN * 4)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        k3cuda.check(lib.k3d_upload(X.ptr, hx, T * HIDDEN * 4))
        k3cuda.check(mw.run(Y.ptr, X.ptr, T, WS.ptr, nws))
        if world > 1:
            k3cuda.check(lib.k3d_ep_allreduce_f32(Y.ptr, T * HIDDEN))
        k3cuda.check(lib.k3d_download(hy, Y.ptr, T * HIDDEN * 4))
    e2e_s = reduce_max(time.perf_counter() - t0)
    lib.k3d_host_free(hx)
    lib.k3d_host_free(hy)
    res = {
        "metric": METRIC, "value": T * args.steps / (tot_ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded MXFP4 experts, E8M0 117..121; bf16 ~N(0,0.02) router and "
                "shared expert; bf16 ~N(0,1) tokens)",
        "config": {"workload": f"config1 MoE layer decode, T={T}", "hidden": HIDDEN,
                   "n_experts": n_exp, "topk": TOPK, "inter": INTER, "shared_inter": SHARED,
                   "parallelism": f"ep{world}", "l2": "flushed between steps (256 MB write)"},
        "roofline": {"kernel": EXPERT_KERNEL[args.expert_kernel], "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind,
                     "traffic": load_traffic("moe_experts_traffic.json"),
                     "alg_bytes_per_launch": alg_bytes, "unique_experts": u_avg,
                     "kernel_ms": kern_ms, "expert_section_ms": exp_ms_avg},
        "e2e": {"value": T * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": T * HIDDEN * 4,
                "d2h_bytes_per_step": T * HIDDEN * 4},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    return res


# -------------------------------------------------- MoE layer, Mode A (all-to-all EP) ----
def bench_moe_a2a(args, rank, world):
    """Config 1 MoE layer for a batch of args.batch tokens split over the ranks
    (data-parallel tokens): each rank routes its own tokens and k3d_moe_swiglu_a2a sends
    every (token, slot) row to its expert's rank and back (grouped NCCL send/recv). A step
    is one layer call on every rank; the step time is the max over ranks."""
    import k3cuda
    import synth
    lib = k3cuda.init(0)
    n_exp = args.n_experts
    per = n_exp // world
    T = max(1, args.batch // world)
    g = synth.rng(4242)
    W = synth.bf16_normal(g, (n_exp, HIDDEN), 0.02)
    bias = g.uniform(-0.1, 0.1, n_exp).astype(np.float32)
    sh = (synth.bf16_normal(g, (SHARED, HIDDEN), 0.02), synth.bf16_normal(g, (SHARED, HIDDEN), 0.02),
          synth.bf16_normal(g, (HIDDEN, SHARED), 0.02))
    mw = k3cuda.MoeWeights(HIDDEN, INTER, n_exp, TOPK, W, bias, shared=sh, seed=7, lo=rank * per,
                           hi=(rank + 1) * per, add_shared=1, tiled=True, lib=lib)
    P = 16
    xs = synth.bf16_to_f32(synth.bf16_normal(synth.rng(5000 + rank), (P * T, HIDDEN), 1.0))
    X = k3cuda.DevBuf.from_array(xs, lib)
    Y = k3cuda.DevBuf(T * HIDDEN * 4, lib)
    nws = mw.a2a_ws_bytes(T, world)
    WS = k3cuda.DevBuf(nws, lib)
    FL = k3cuda.DevBuf(256 << 20, lib)
    ev = [lib.k3d_event_create() for _ in range(2)]

    def step(i):
        k3cuda.check(mw.run_a2a(Y.ptr, X.ptr + (i % P) * T * HIDDEN * 4, T, T, WS.ptr, nws), "moe a2a step")

    for i in range(args.warmup):
        step(i)
    k3cuda.check(lib.k3d_sync())
    barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
    lib.k3d_launch_count_reset()
    step_ms = []
    for i in range(args.steps):
        lib.k3d_memset(FL.ptr, i & 0xff, FL.nbytes)      # L2 flush, outside the events
        barrier()
        lib.k3d_event_record(ev[0])
        step(args.warmup + i)
        lib.k3d_event_record(ev[1])
        step_ms.append(lib.k3d_event_elapsed_ms(ev[0], ev[1]))
    k3cuda.check(lib.k3d_sync())
    launches = lib.k3d_launch_count() - args.steps
    clk = clocks.stop()
    tot_ms = reduce_max(sum(step_ms))
    # end to end through the public API with host buffers (this rank's tokens in and out)
    hx = lib.k3d_host_alloc(T * HIDDEN * 4)
    hy = lib.k3d_host_alloc(T * HIDDEN * 4)
    C.memmove(hx, xs[:T].ctypes.data, T * HIDDEN * 4)
    barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        k3cuda.check(lib.k3d_upload(X.ptr, hx, T * HIDDEN * 4))
        step(0)
        k3cuda.check(lib.k3d_download(hy, Y.ptr, T * HIDDEN * 4))
    e2e_s = reduce_max(time.perf_counter() - t0)
    lib.k3d_host_free(hx)
    lib.k3d_host_free(hy)
    B = T * world
    return {
        "metric": METRIC, "value": B * args.steps / (tot_ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded MXFP4 experts, E8M0 117..121; bf16 ~N(0,0.02) router and "
                "shared expert; bf16 ~N(0,1) tokens, different on every rank)",
        "config": {"workload": f"config1 MoE layer, Mode A all-to-all EP, batch {B} "
                               f"({T} tokens per rank)", "hidden": HIDDEN, "n_experts": n_exp,
                   "topk": TOPK, "inter": INTER, "shared_inter": SHARED, "parallelism": f"ep{world}-a2a",
                   "l2": "flushed between steps (256 MB write)"},
        "e2e": {"value": B * args.steps / e2e_s, "unit": "tok/s",
                "h2d_bytes_per_step": T * HIDDEN * 4, "d2h_bytes_per_step": T * HIDDEN * 4},
        "gpu_launches": int(launches),
        "clocks": clk,
    }


# ------------------------------------------------------------ KDA prefill (config 3) ----
KDA_H, KDA_D = 64, 128


def kda_prefill_bytes(T):
    """Algorithmic bytes of one prefill: q, k, v, decay and o (fp32 [T][64][128] each),
    beta [T][64], and the 64 fp32 128x128 states read and written once."""
    return 5 * T * KDA_H * KDA_D * 4 + T * KDA_H * 4 + 2 * KDA_H * KDA_D * KDA_D * 4


def kda_prefill_inputs(T, seed):
    g = np.random.default_rng(seed)

    def unit(x):
        x /= np.linalg.norm(x, axis=-1, keepdims=True)
        return x

    shp = (T, KDA_H, KDA_D)
    q = unit(g.standard_normal(shp, dtype=np.float32))
    k = unit(g.standard_normal(shp, dtype=np.float32))
    v = g.standard_normal(shp, dtype=np.float32)
    al = g.uniform(0.9, 1.0, shp).astype(np.float32)
    be = g.uniform(0, 1, (T, KDA_H)).astype(np.float32)
    S = (g.standard_normal((KDA_H, KDA_D, KDA_D), dtype=np.float32) * np.float32(0.01))
    return S, q, k, v, al, be


def cpu_kda_prefill_sample(seconds=12.0, max_tokens=4096):
    """The reference's k3_kda_step (k3_ops.c:186-243, compiled in oracle/_ref) over the 64
    heads of a config-3 prefill, token after token on one core, for about `seconds`."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as orc
    if orc.Reference.available():
        impl, kind = orc.Reference(), "reference"
    else:
        impl, kind = orc.Oracle(), "port"
    S, q, k, v, al, be = kda_prefill_inputs(64, 11)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < max_tokens:
        t = n % 64
        for h in range(KDA_H):
            S[h] = impl.kda_step(S[h], q[t, h], k[t, h], v[t, h], al[t, h], float(be[t, h]))[0]
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": 1, "kind": kind,
            "sample": f"{n} prefill tokens x 64 heads of k3_kda_step (128x128 state) in {dt:.1f} s "
                      f"on one core; the reference runs heads in parallel under OpenMP"}


def bench_kda_prefill(args, rank, world):
    """BASELINE config 3 prefill: one step = k3d_kda_prefill(chunk = 64) over T = 8192 tokens
    x 64 heads x 128x128 fp32 states, the state carried from step to step. The inputs
    (1.35 GB) exceed L2, so no flush is needed. Ranks run independent sequences (weak)."""
    import k3cuda
    lib = k3cuda.init(0)
    T = args.prefill_tokens
    S, q, k, v, al, be = kda_prefill_inputs(T, 3303 + rank)
    bufs = [k3cuda.DevBuf.from_array(a, lib) for a in (S, q, k, v, al, be)]
    O = k3cuda.DevBuf(T * KDA_H * KDA_D * 4, lib)
    ev = [lib.k3d_event_create() for _ in range(2)]

    def step(chunk=64):
        k3cuda.check(lib.k3d_kda_prefill(bufs[0].ptr, O.ptr, bufs[1].ptr, bufs[2].ptr, bufs[3].ptr,
                                         bufs[4].ptr, bufs[5].ptr, T, KDA_H, KDA_D, KDA_D, chunk),
                     "kda prefill")

    for _ in range(args.warmup):
        step()
    k3cuda.check(lib.k3d_sync())
    barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0)))
    clocks.start()
    lib.k3d_launch_count_reset()
    step_ms = []
    for _ in range(args.steps):
        barrier()
        lib.k3d_event_record(ev[0])
        step()
        lib.k3d_event_record(ev[1])
        step_ms.append(lib.k3d_event_elapsed_ms(ev[0], ev[1]))
    k3cuda.check(lib.k3d_sync())
    launches = lib.k3d_launch_count()
    clk = clocks.stop()
    tot_ms = reduce_max(sum(step_ms))
    # the sequential recurrence (chunk = 0, bit-identical to k3_kda_step) once, for scale
    lib.k3d_event_record(ev[0])
    step(0)
    lib.k3d_event_record(ev[1])
    k3cuda.check(lib.k3d_sync())
    seq_ms = lib.k3d_event_elapsed_ms(ev[0], ev[1])
    # end to end with host buffers: inputs up, prefill, o down
    names = ("q", "k", "v", "al", "be")
    host = {}
    for n_, a in zip(names, (q, k, v, al, be)):
        host[n_] = (lib.k3d_host_alloc(a.nbytes), a.nbytes)
        C.memmove(host[n_][0], a.ctypes.data, a.nbytes)
    ho = lib.k3d_host_alloc(O.nbytes)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for b, n_ in zip(bufs[1:], names):
            k3cuda.check(lib.k3d_upload(b.ptr, host[n_][0], host[n_][1]))
        step()
        k3cuda.check(lib.k3d_download(ho, O.ptr, O.nbytes))
    e2e_s = reduce_max(time.perf_counter() - t0)
    for p_, _ in host.values():
        lib.k3d_host_free(p_)
    lib.k3d_host_free(ho)
    h2d = sum(a.nbytes for a in (q, k, v, al, be))
    alg = kda_prefill_bytes(T)
    ms = tot_ms / args.steps
    peak, pk = measured_peaks()
    ach = alg / (ms * 1e-3) / 1e9
    nch = (T + 63) // 64
    fma = KDA_H * nch * (3 * 64 * KDA_D * KDA_D + 64 * 64 * KDA_D // 2 + 64 * KDA_D * KDA_D)
    return {
        "metric": "KDA prefill tok/s (config 3: 64 heads, 128x128 fp32 state, chunk 64)",
        "value": world * T * args.steps / (tot_ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (q, k L2-normalised N(0,1); v N(0,1); decay U(0.9,1); beta U(0,1); "
                "state N(0,0.01)), one sequence per rank",
        "config": {"workload": f"config3 KDA chunked prefill, {T} tokens", "heads": KDA_H,
                   "head_dim": KDA_D, "chunk": 64, "parallelism": f"replicas{world}",
                   "l2": "inputs 1.35 GB > L2", "sequential_ms": seq_ms,
                   "scan_fp32_fma_per_step": fma},
        "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                     "frac": ach / peak, "peak_kind": pk, "traffic": None,
                     "note": "whole step (prep + scan kernels); the scan is fp32-FMA bound on "
                             "CUDA cores, the bytes are the algorithmic floor"},
        "e2e": {"value": world * T * args.steps / e2e_s, "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": O.nbytes},
        "gpu_launches": int(launches),
        "clocks": clk,
    }


# ----------------------------------------------------------------- stack (config 4) ----
def stack_cfg(world, rank, batch, cap, layout=1, ep_tokens=0):
    import k3cuda
    sc = k3cuda.K3dStackCfg()
    sc.hidden, sc.vocab, sc.n_layers, sc.eps = HIDDEN, 163840, 8, 1e-6
    sc.kda_heads, sc.kda_head_dim, sc.conv_k, sc.gate_lb = 64, 128, 4, -5.0
    sc.mla = k3cuda.K3dMlaShape(HIDDEN, 64, 1536, 512, 128, 64, 128, 50000.0, 1e-6, 1)
    per = N_EXPERTS // world
    sc.moe = k3cuda.K3dMoeShape(HIDDEN, INTER, N_EXPERTS, TOPK, 1, 2.5, SHARED, rank * per,
                                (rank + 1) * per, 1 if rank == 0 else 0, layout)
    sc.first_dense, sc.dense_inter = 1, 18432
    for i in range(16):
        sc.mla_layers[i] = (3, 7)[i] if i < 2 else -1
    sc.batch, sc.ctx_cap = batch, cap
    sc.ep_tokens = ep_tokens
    return sc


def stack_config(args, world):
    """The workload description both arms print (the reference arm times the same model)."""
    mode_a = stack_mode_a(args, world)
    return {"workload": "config4 8-layer K3 stack decode", "batch": args.batch,
            "context": args.context, "hidden": HIDDEN,
            "layers": "KDA x6 + MLA x2 (one-based 4, 8); layer 0 dense 18432, layers 1-7 MoE "
                      "384x top-8 + shared", "vocab": 163840,
            "parallelism": f"ep{world}" + (f" mode A: {args.batch // world} sequences per rank, "
                                           "device-planned all-to-all" if mode_a else ""),
            "l2": "per-step weight stream of GBs >> 126 MB L2 (no flush needed)"}


def stack_mode_a(args, world):
    """Mode A (each rank its own share of the batch, all-to-all MoE) for a batch split over
    several ranks; Mode R (the batch replicated, experts split, NVLink push combine)
    otherwise or when asked."""
    if args.ep_mode == "r" or world == 1:
        return False
    if args.ep_mode == "auto" and args.batch == 1:
        return False
    if args.batch % world:
        raise SystemExit(f"--batch {args.batch} does not split over {world} ranks")
    return True


def bench_stack(args, rank, world):
    import k3cuda
    lib = k3cuda.init(0)
    k3cuda.check(lib.k3d_set_expert_kernel(args.expert_kernel))
    ctx = args.context
    n_prof = max(3, min(args.steps, 10))
    e2e_steps = max(args.steps, 200)
    # the timed and profiled steps, then (from a refilled context) the end-to-end ones
    # the timed steps (twice under several ranks: see the clocks below) and the profiled
    # steps, then (from a refilled context) the end-to-end ones
    cap = ctx + max(args.warmup + 2 * args.steps + n_prof, 3 + e2e_steps) + 16
    # the tcgen05 kernel streams experts stored in the tiled layout; the other two
    # kernels read the checkpoint layout
    mode_a = stack_mode_a(args, world)
    B = args.batch // world if mode_a else args.batch      # this rank's sequences
    cfg = stack_cfg(world, rank, B, cap, 1 if args.expert_kernel in (0, 3, 4) else 0, 1 if mode_a else 0)
    t0 = time.time()
    model = lib.k3d_model_create(C.byref(cfg), 2024)
    if not model:
        raise k3cuda.K3Error("k3d_model_create failed: " + lib.k3d_last_message().decode())
    k3cuda.check(lib.k3d_model_fill_context(model, ctx, 77))
    k3cuda.check(lib.k3d_sync())
    init_s = time.time() - t0
    ids = k3cuda.DevBuf(B * 4, lib)
    nxt = k3cuda.DevBuf(B * 4, lib)
    k3cuda.check(lib.k3d_fill_i32_uniform(ids.ptr, B, 5, 0, 163839))
    logits_p = lib.k3d_model_tensor(model, b"logits", None)
    ev = [lib.k3d_event_create() for _ in range(2)]
    # warm-up: the first step runs eagerly, the second captures the graph
    for i in range(args.warmup):
        k3cuda.check(lib.k3d_model_step_dev(model, ids.ptr, nxt.ptr, logits_p), "warmup step")
        k3cuda.check(lib.k3d_copy(ids.ptr, nxt.ptr, B * 4))
    k3cuda.check(lib.k3d_sync())
    barrier()
    def timed_steps(sample):
        """K steps between one event pair on the library stream, no host synchronisation
        inside the region (the host enqueues graph replays back to back); the device time
        as the max over ranks, and the clocks when sampled."""
        clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0)))
        if sample:
            clocks.start()
        lib.k3d_launch_count_reset()
        lib.k3d_event_record(ev[0])
        for i in range(args.steps):
            k3cuda.check(lib.k3d_model_step_dev(model, ids.ptr, nxt.ptr, logits_p), "step")
            k3cuda.check(lib.k3d_copy(ids.ptr, nxt.ptr, B * 4))   # greedy: next token in
        lib.k3d_event_record(ev[1])
        k3cuda.check(lib.k3d_sync())
        clk = clocks.stop() if sample else None
        barrier()
        return reduce_max(lib.k3d_event_elapsed_ms(ev[0], ev[1])), clk

    # One GPU: the clocks are sampled during the timed steps. Several: an nvidia-smi query
    # during the steps stalls the ranks' push combines (two B200, 50 steps: 775 tok/s
    # unsampled, 667 with an NVML clock and throttle-reason poll, 175-475 with nvidia-smi),
    # so the K timed steps run unsampled and the same K steps run again right after,
    # sampled by rank 0; the line reports that pass's rate beside its clocks.
    if world == 1:
        tot_ms, clk = timed_steps(True)
    else:
        tot_ms, _ = timed_steps(False)
        s_ms, clk = timed_steps(True)
        if clk is not None:
            clk["window"] = "the same K steps run again right after the timed ones, sampled"
            clk["window_tok_s"] = (B * world if mode_a else B) * args.steps / (s_ms * 1e-3)
    step_bytes = lib.k3d_model_last_step_bytes(model)
    hbm, peak_kind = measured_peaks()
    # per-kernel device times from an eager pass with the section timers on (graph
    # replays carry no per-kernel events); same kernels, same inputs
    k3cuda.check(lib.k3d_model_use_graph(model, 0))
    lib.k3d_prof_reset()
    lib.k3d_prof_enable(1)
    lib.k3d_launch_count_reset()
    for i in range(n_prof):
        k3cuda.check(lib.k3d_model_step_dev(model, ids.ptr, nxt.ptr, logits_p), "profiled step")
    k3cuda.check(lib.k3d_sync())
    launches_per_step = lib.k3d_launch_count() / n_prof
    sections = {}
    exp_ms, _ = expert_kernel_ms(lib)
    for name in ("moe.experts", "experts.fused", "experts.gateup", "experts.down", "moe.shared", "moe.router",
                 "kda.proj_in", "kda.core",
                 "kda.proj_out", "mla.proj_in", "mla.core", "mla.proj_out", "dense.mlp", "lm_head",
                 "ep.combine"):
        cnt = C.c_long()
        ms = lib.k3d_prof_ms(name.encode(), C.byref(cnt))
        if cnt.value:
            sections[name] = {"ms_per_call": ms / cnt.value, "calls_per_step": cnt.value / n_prof}
    lib.k3d_prof_enable(0)
    k3cuda.check(lib.k3d_model_use_graph(model, 1))
    # algorithmic bytes: the weights of the distinct experts the step routed to (measured:
    # the last MoE layer's count), read once, plus the activation and output rows
    uniq = lib.k3d_moe_last_unique()
    if uniq <= 0:
        uniq = TOPK * B
    alg_exp = uniq * EXPERT_BYTES + TOPK * B * (INTER * 8 + HIDDEN * 4) + HIDDEN * 4 * B
    if world > 1 and not mode_a:
        alg_exp /= world
    achieved = alg_exp / (exp_ms * 1e-3) / 1e9
    # end to end through the public API with host buffers: token ids in from host memory,
    # next ids out to host memory, every step (greedy decoding); a few untimed steps first,
    # then at least 200 timed steps so that host jitter averages out. The context is filled
    # again and sequence b starts from token (37 b + 5) mod vocab (b the global sequence
    # index), so the generated tokens, and their hash, do not depend on how many steps ran
    # before or on how many ranks share the job.
    k3cuda.check(lib.k3d_model_fill_context(model, ctx, 77))
    g0 = rank * B if mode_a else 0
    hid = ((np.arange(g0, g0 + B) * 37 + 5) % 163840).astype(np.int32)
    hnx = np.zeros(B, np.int32)
    for i in range(3):
        k3cuda.check(lib.k3d_model_step_host(model, hid.ctypes.data, hnx.ctypes.data), "e2e warm-up")
        hid[:] = hnx
    gen = np.zeros((e2e_steps, B), np.int32)
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        k3cuda.check(lib.k3d_model_step_host(model, hid.ctypes.data, hnx.ctypes.data), "e2e step")
        hid[:] = hnx
        gen[i] = hnx
    e2e_s = reduce_max(time.perf_counter() - t0)
    k3cuda.check(lib.k3d_sync(), "after the e2e steps")      # device errors of the steps
    lib.k3d_model_destroy(model)
    if mode_a:
        gen = gather_cols(gen)                                # every rank's sequences
    ms = tot_ms / args.steps
    res = {
        "metric": METRIC, "value": (B * world if mode_a else B) * args.steps / (tot_ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic random-init weights (bf16 ~N(0,0.02), MXFP4 experts E8M0 117..121); "
                f"MLA latent caches ~N(0,1) and KDA states ~N(0,0.01) filled as after {ctx} tokens",
        "config": stack_config(args, world),
        "roofline": {"kernel": EXPERT_KERNEL[args.expert_kernel], "bound": "hbm",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": peak_kind, "traffic": load_traffic("moe_experts_traffic.json"),
                     "alg_bytes_per_launch": alg_exp, "unique_experts": uniq, "kernel_ms": exp_ms},
        "roofline_step": {"bound": "hbm", "alg_bytes_per_step": step_bytes,
                          "achieved": step_bytes / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                          "frac": step_bytes / (ms * 1e-3) / 1e9 / hbm},
        "sections_ms": sections,
        "e2e": {"value": (B * world if mode_a else B) * e2e_steps / e2e_s, "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B, "steps": e2e_steps,
                "tokens_fnv1a": fnv1a(gen), "first_tokens": gen[:8, 0].tolist()},
        "gpu_launches": int(round(launches_per_step * args.steps)),
        "clocks": clk,
        "init_s": init_s,
    }
    return res


# ---------------------------------------------------------------- distributed ----
_PG = None


def barrier():
    if _PG is not None:
        import torch.distributed as dist
        dist.barrier()


def gather_cols(a):
    """The ranks' [steps][B] arrays side by side, in rank order (a copy on one rank)."""
    if _PG is None:
        return a
    import torch
    import torch.distributed as dist
    t = torch.from_numpy(np.ascontiguousarray(a))
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return np.concatenate([p.numpy() for p in parts], axis=1)


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
    # stdout carries the one JSON line: NCCL's version banner (printed at NCCL_DEBUG=VERSION)
    # stays off and NCCL's own log goes to stderr
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
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
    ap.add_argument("--workload", default="stack", choices=["stack", "moe", "moe_a2a", "kda_prefill"],
                    help="moe_a2a: the MoE layer for a --batch split over the ranks (Mode A); "
                         "kda_prefill: config 3 chunked prefill")
    ap.add_argument("--prefill-tokens", type=int, default=8192,
                    help="kda_prefill workload: tokens per step (config 3: 8192)")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ep-mode", choices=("auto", "r", "a"), default="auto",
                    help="stack under expert parallelism: r = the batch replicated on every rank "
                         "(push combine), a = the batch split over the ranks (device-planned "
                         "all-to-all); auto = a when the batch is above 1")
    ap.add_argument("--tokens", type=int, default=1,
                    help="moe workload: tokens per step (config 1 lists T = 1, 8, 64, 512)")
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="bounded CPU-baseline sample length; 0 skips it")
    ap.add_argument("--expert-kernel", type=int, default=0, choices=[0, 1, 2, 3, 4],
                    help="0 tcgen05 block-scaled (default), 1 mma.sync, 2 CUDA cores, 3 tcgen05 with "
                         "one token per work item, 4 tcgen05 with gate/up, act split and down as "
                         "one launch at decode sizes")
    ap.add_argument("--n-experts", type=int, default=N_EXPERTS,
                    help="routed experts resident per layer (384 = config 1; fewer only for "
                         "profiling captures that must stay small)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_env()
    if args.impl == "reference":
        if rank != 0:
            return
        metric = METRIC
        if args.workload == "stack":
            cb = cpu_stack_run(args.context, reps=max(5, min(args.steps, 10)))
            wl = stack_config(args, world)
        elif args.workload == "kda_prefill":
            cb = cpu_kda_prefill_sample(args.cpu_seconds)
            metric = "KDA prefill tok/s (config 3: 64 heads, 128x128 fp32 state, chunk 64)"
            wl = {"workload": f"config3 KDA chunked prefill, {args.prefill_tokens} tokens",
                  "heads": KDA_H, "head_dim": KDA_D, "chunk": 64, "parallelism": "cpu"}
        else:
            cb = cpu_moe_sample(seconds=args.cpu_seconds)
            wl = {"workload": "config1 MoE layer decode, T=1", "hidden": HIDDEN,
                  "n_experts": N_EXPERTS, "topk": TOPK, "parallelism": "cpu"}
        res = {"metric": metric, "value": cb["value"], "unit": "tok/s", "n_gpus": world,
               "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / cb["value"],
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "fp64-accumulate/fp32", "data": "synthetic",
               "config": wl,
               "impl": "reference", "cpu_baseline": cb,
               "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                       "d2h_bytes_per_step": 0}}
        print(json.dumps(res), flush=True)
        return
    if args.workload == "moe_a2a" and args.batch == 1:
        args.batch = 64
    setup_dist(world, rank, local)
    if args.workload == "stack":
        res = bench_stack(args, rank, world)
    elif args.workload == "moe":
        res = bench_moe(args, rank, world)
    elif args.workload == "kda_prefill":
        res = bench_kda_prefill(args, rank, world)
    else:
        res = bench_moe_a2a(args, rank, world)
    if rank == 0:
        if world == 1 and args.cpu_seconds > 0 and args.workload != "moe_a2a":
            res["cpu_baseline"] = (cpu_stack_run(args.context) if args.workload == "stack"
                                   else cpu_kda_prefill_sample(args.cpu_seconds)
                                   if args.workload == "kda_prefill"
                                   else cpu_moe_sample(seconds=args.cpu_seconds))
        print(json.dumps(res), flush=True)
    if world > 1:
        import k3cuda
        k3cuda.load().k3d_ep_finalize()
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
