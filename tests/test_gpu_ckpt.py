"""Loading a checkpoint in the released naming (k3d_model_load_checkpoint; names from
src/model/k3_bind.c:167-241 and src/io/k3_load.c:11) into the reduced-width decode stack.
Model A's weights are exported into three safetensors shards, the way the released
checkpoint stores them (bf16 matrices, fp32 vectors, conv weights as [H*D][1][conv_k], A_log
padded to head_dim with zeros, U8 MXFP4 experts as six contiguous tensors, one expert
written non-contiguously); model B (another seed) loads them and then holds A's tensors bit
for bit and decodes exactly as A. A checkpoint that does not fit (a missing tensor, a wrong
element count, an fp32 matrix, a wrong scale count) is refused before anything is read."""
import contextlib
import ctypes

import numpy as np
import pytest

import k3cuda
from safetensors_io import write_shard
from test_gpu_stack import CFG, make_cfg, download, host_copy

pytestmark = pytest.mark.gpu

PRE = "language_model.model."


@contextlib.contextmanager
def model(k3, seed):
    m = k3.k3d_model_create(ctypes.byref(make_cfg(CFG, batch=1, cap=64, layout=1)), seed)
    assert m, k3.k3d_last_message()
    try:
        yield m
    finally:
        k3.k3d_model_destroy(m)


def export(W, c):
    """The model's weights as released-checkpoint tensors: name -> (dtype, shape, array)."""
    E, V = c["hidden"], c["vocab"]
    H, D, K = c["kda_heads"], c["kda_head_dim"], c["conv_k"]
    P = H * D
    ml, mo = c["mla"], c["moe"]
    T = {}

    def bf(name, key, shape):
        T[name] = ("BF16", shape, W[key].reshape(-1))

    def f32(name, key, shape):
        T[name] = ("F32", shape, W[key].reshape(-1))

    bf(PRE + "embed_tokens.weight", "embed", [V, E])
    bf("language_model.lm_head.weight", "lm_head", [V, E])
    f32(PRE + "norm.weight", "final_norm", [E])
    for l in range(c["n_layers"]):
        p, n = f"layer{l}.", f"{PRE}layers.{l}."
        f32(n + "input_layernorm.weight", p + "in_norm", [E])
        f32(n + "post_attention_layernorm.weight", p + "post_norm", [E])
        if l in c["mla_layers"]:
            qh, kvw, kvd = ml["qn"] + ml["qr"], ml["kv_lora"] + ml["qr"], ml["qn"] + ml["vh"]
            for k, nm, shp in (("q_a", "q_a_proj", [ml["q_lora"], E]), ("q_b", "q_b_proj", [ml["H"] * qh, ml["q_lora"]]),
                               ("kv_a", "kv_a_proj_with_mqa", [kvw, E]), ("kv_b", "kv_b_proj", [ml["H"] * kvd, ml["kv_lora"]]),
                               ("o", "o_proj", [E, ml["H"] * ml["vh"]]), ("g", "g_proj", [ml["H"] * ml["vh"], E])):
                bf(n + f"self_attn.{nm}.weight", p + "mla." + k, shp)
            f32(n + "self_attn.q_a_layernorm.weight", p + "mla.q_a_norm", [ml["q_lora"]])
            f32(n + "self_attn.kv_a_layernorm.weight", p + "mla.kv_a_norm", [ml["kv_lora"]])
        else:
            for k, shp in (("q", [P, E]), ("k", [P, E]), ("v", [P, E]), ("g", [P, E]), ("o", [E, P]),
                           ("f_a", [D, E]), ("f_b", [P, D]), ("b", [H, E])):
                bf(n + f"self_attn.{k}_proj.weight", p + "kda." + k, shp)
            for k in ("q", "k", "v"):
                f32(n + f"self_attn.{k}_conv1d.weight", p + f"kda.{k}_conv", [P, 1, K])
            a = np.zeros(D, np.float32)
            a[:H] = W[p + "kda.A_log"]
            T[n + "self_attn.A_log"] = ("F32", [D], a)
            f32(n + "self_attn.dt_bias", p + "kda.dt_bias", [P])
            f32(n + "self_attn.o_norm.weight", p + "kda.o_norm", [D])
        if l < c["first_dense"]:
            I = c["dense_inter"]
            bf(n + "mlp.gate_proj.weight", p + "dense.gate", [I, E])
            bf(n + "mlp.up_proj.weight", p + "dense.up", [I, E])
            bf(n + "mlp.down_proj.weight", p + "dense.down", [E, I])
            continue
        m, SI, I = n + "block_sparse_moe.", mo["shared_inter"], mo["inter"]
        bf(m + "gate.weight", p + "moe.router_w", [mo["n_experts"], E])
        f32(m + "gate.e_score_correction_bias", p + "moe.router_bias", [mo["n_experts"]])
        bf(m + "shared_experts.gate_proj.weight", p + "moe.sh_gate", [SI, E])
        bf(m + "shared_experts.up_proj.weight", p + "moe.sh_up", [SI, E])
        bf(m + "shared_experts.down_proj.weight", p + "moe.sh_down", [E, SI])
        ex = W[p + "moe.experts"]
        for e in range(mo["n_experts"]):
            x = ex.get(e)
            for w, pk, sk, rows, cin in (("w1", "p1", "s1", I, E), ("w3", "p3", "s3", I, E), ("w2", "p2", "s2", E, I)):
                T[m + f"experts.{e}.{w}.weight_packed"] = ("U8", [rows, cin // 2], x[pk])
                T[m + f"experts.{e}.{w}.weight_scale"] = ("U8", [rows, cin // 32], x[sk])
    return T


def write_checkpoint(d, T, shuffle_expert=None):
    """Three shards by layer range; each expert's six tensors contiguous, except
    shuffle_expert = (layer, e), whose tensors are split by the names of other tensors."""
    d.mkdir()
    names = list(T)
    shards = [[], [], []]
    for nm in names:
        l = int(nm.split("layers.")[1].split(".")[0]) if "layers." in nm else 0
        shards[min(2, l // 3)].append(nm)
    if shuffle_expert:
        l, e = shuffle_expert
        key = f"{PRE}layers.{l}.block_sparse_moe.experts.{e}."
        lst = shards[min(2, l // 3)]
        mine = [n for n in lst if n.startswith(key)]
        rest = [n for n in lst if not n.startswith(key)]
        lst[:] = [v for pair in zip(mine, rest) for v in pair] + rest[len(mine):]
    for i, lst in enumerate(shards):
        write_shard(d / f"model-{i + 1:05d}-of-00003.safetensors", {n: T[n] for n in lst}, order=lst,
                    metadata={"format": "pt"})
    return str(d).encode()


def load(k3, m, path):
    ck = k3.k3d_ckpt_open(path)
    assert ck, k3.k3d_ckpt_error().decode()
    try:
        return k3.k3d_model_load_checkpoint(m, ck)
    finally:
        k3.k3d_ckpt_close(ck)


def test_checkpoint_round_trip(k3, tmp_path):
    with model(k3, 11) as a, model(k3, 12) as b:
        Wa, _ = host_copy(k3, a, CFG, layout=1, batch=1, cap=64, lazy_experts=True)
        path = write_checkpoint(tmp_path / "ck", export(Wa, CFG), shuffle_expert=(4, 3))
        r = load(k3, b, path)
        assert r == 0, k3.k3d_ckpt_error().decode()
        Wb, _ = host_copy(k3, b, CFG, layout=1, batch=1, cap=64, lazy_experts=True)
        for key, va in Wa.items():
            vb = Wb[key]
            if key.endswith("moe.experts"):
                for e in range(CFG["moe"]["n_experts"]):
                    xa, xb = va.get(e), vb.get(e)
                    for k in xa:
                        assert np.array_equal(xa[k], xb[k]), (key, e, k)
            else:
                assert np.array_equal(np.asarray(va), np.asarray(vb)), key
        for m_ in (a, b):
            k3cuda.check(k3.k3d_model_fill_context(m_, 5, 3))
        toks = np.array([17], np.int32)
        for _ in range(3):
            na, nb = np.zeros(1, np.int32), np.zeros(1, np.int32)
            k3cuda.check(k3.k3d_model_step_host(a, toks.ctypes.data, na.ctypes.data))
            la = download(k3, a, "logits", np.float32).copy()
            k3cuda.check(k3.k3d_model_step_host(b, toks.ctypes.data, nb.ctypes.data))
            lb = download(k3, b, "logits", np.float32).copy()
            assert np.array_equal(la, lb)
            assert na[0] == nb[0]
            toks = na


@pytest.mark.parametrize("case", ["missing", "count", "f32_matrix", "scales"])
def test_checkpoint_that_does_not_fit_is_refused(k3, tmp_path, case):
    with model(k3, 21) as a, model(k3, 22) as b:
        Wa, _ = host_copy(k3, a, CFG, layout=1, batch=1, cap=64, lazy_experts=True)
        T = export(Wa, CFG)
        q = f"{PRE}layers.1.self_attn.q_proj.weight"
        sc = f"{PRE}layers.2.block_sparse_moe.experts.5.w2.weight_scale"
        if case == "missing":
            del T[f"{PRE}layers.5.self_attn.dt_bias"]
        elif case == "count":
            dt, shp, arr = T[q]
            T[q] = (dt, [shp[0] - 1, shp[1]], arr[: (shp[0] - 1) * shp[1]])
        elif case == "f32_matrix":
            dt, shp, arr = T[q]
            T[q] = ("F32", shp, (arr.astype(np.uint32) << 16).view(np.float32))
        else:
            dt, shp, arr = T[sc]
            T[sc] = (dt, [shp[0], shp[1] * 2], np.concatenate([arr.reshape(shp), arr.reshape(shp)], 1).reshape(-1))
        path = write_checkpoint(tmp_path / "ck", T)
        before = download(k3, b, "layer1.kda.q", np.uint16).copy()
        assert load(k3, b, path) == k3cuda.K3D_EINVAL
        assert k3.k3d_ckpt_error().decode()
        assert np.array_equal(download(k3, b, "layer1.kda.q", np.uint16), before)   # nothing read
