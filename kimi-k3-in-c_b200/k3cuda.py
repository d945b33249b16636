"""k3cuda -- Python ctypes binding of libk3cuda.so (include/k3/k3.h, include/k3/k3_cuda.h).

The library is the product: sm_100a kernels behind a C ABI. This module only loads it,
declares the C prototypes and offers small helpers (device buffers, numpy transfers) for
the tests and bench.py. There is no Python or CPU implementation of any operator here;
if the shared object or a CUDA device is missing, load() raises.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libk3cuda.so")

K3D_OK = 0
K3D_ENODEV, K3D_EINVAL, K3D_ENOMEM, K3D_ECUDA, K3D_EDEVICE = 1, 2, 3, 4, 5
K3D_EUNSUPPORTED, K3D_ENCCL, K3D_EBOUND, K3D_ETIMEOUT = 6, 7, 8, 9

vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t
u64 = C.c_uint64


class K3Cfg(C.Structure):
    _fields_ = [
        ("hidden", i32), ("n_layers", i32), ("vocab", i32), ("rms_eps", f32),
        ("kda_heads", i32), ("kda_head_dim", i32), ("conv_k", i32), ("gate_lb", f32),
        ("n_heads", i32), ("q_lora", i32), ("kv_lora", i32), ("qk_nope", i32),
        ("qk_rope", i32), ("v_head", i32), ("mla_out_gate", i32),
        ("n_experts", i32), ("topk", i32), ("n_shared", i32), ("latent", i32),
        ("moe_inter", i32), ("routed_scale", f32), ("moe_renorm", i32), ("latent_norm", i32),
        ("first_dense", i32), ("dense_inter", i32), ("attn_res_block", i32),
        ("situ_b1", f32), ("situ_b2", f32), ("n_full_attn", i32), ("full_attn", C.POINTER(i32)),
    ]


class K3MlaW(C.Structure):
    _fields_ = [("q_a", vp), ("q_b", vp), ("kv_a", vp), ("kv_b", vp), ("o", vp), ("g", vp),
                ("q_a_norm", vp), ("kv_a_norm", vp), ("wdt", i32)]


class K3ExpertQ(C.Structure):
    _fields_ = [("p1", vp), ("s1", vp), ("p3", vp), ("s3", vp), ("p2", vp), ("s2", vp)]


class K3MoeW(C.Structure):
    _fields_ = [("gate", vp), ("bias", vp), ("w1", vp), ("w3", vp), ("w2", vp),
                ("latent_norm", vp), ("down", vp), ("up", vp), ("sh1", vp), ("sh3", vp),
                ("sh2", vp), ("wdt", i32), ("src", vp), ("layer", i32), ("cache_only", i32)]


class K3KdaW(C.Structure):
    _fields_ = [("q", vp), ("k", vp), ("v", vp), ("q_conv", vp), ("k_conv", vp),
                ("v_conv", vp), ("f_a", vp), ("f_b", vp), ("A_log", vp), ("dt_bias", vp),
                ("b", vp), ("g", vp), ("o_norm", vp), ("o", vp), ("wdt", i32)]


class K3LayerW(C.Structure):
    _fields_ = [("in_norm", vp), ("post_norm", vp), ("attn_res_norm", vp),
                ("attn_res_proj", vp), ("mlp_res_norm", vp), ("mlp_res_proj", vp),
                ("kda", C.POINTER(K3KdaW)), ("mla", C.POINTER(K3MlaW)),
                ("moe", C.POINTER(K3MoeW)), ("dense_gate", vp), ("dense_up", vp),
                ("dense_down", vp), ("wdt", i32)]


class K3dMoeShape(C.Structure):
    _fields_ = [("hidden", i32), ("inter", i32), ("n_experts", i32), ("topk", i32),
                ("renorm", i32), ("routed_scale", f32), ("shared_inter", i32),
                ("expert_lo", i32), ("expert_hi", i32), ("add_shared", i32),
                ("expert_layout", i32)]


class K3dMoeW(C.Structure):
    _fields_ = [("router_w", vp), ("router_bias", vp), ("experts", vp), ("sh_gate", vp),
                ("sh_up", vp), ("sh_down", vp)]


class K3dMlaShape(C.Structure):
    _fields_ = [("hidden", i32), ("n_heads", i32), ("q_lora", i32), ("kv_lora", i32),
                ("qk_nope", i32), ("qk_rope", i32), ("v_head", i32), ("rope_theta", f32),
                ("eps", f32), ("out_gate", i32)]


class K3dMlaW(C.Structure):
    _fields_ = [("q_a", vp), ("q_b", vp), ("kv_a", vp), ("kv_b", vp), ("o", vp), ("g", vp),
                ("q_a_norm", vp), ("kv_a_norm", vp)]


class K3dKdaShape(C.Structure):
    _fields_ = [("hidden", i32), ("heads", i32), ("head_dim", i32), ("conv_k", i32),
                ("gate_lb", f32), ("eps", f32)]


class K3dKdaW(C.Structure):
    _fields_ = [("q", vp), ("k", vp), ("v", vp), ("g", vp), ("b", vp), ("f_a", vp), ("f_b", vp),
                ("o", vp), ("q_conv", vp), ("k_conv", vp), ("v_conv", vp), ("A_log", vp),
                ("dt_bias", vp), ("o_norm", vp)]


class K3dStateInfo(C.Structure):
    _fields_ = [("version", i32), ("n_bound", i32), ("n_mla", i32), ("cached", i32), ("nseq", i32),
                ("has_latent", i32)]


class K3dCkptTensor(C.Structure):
    _fields_ = [("shard", i32), ("dtype", i32), ("ndim", i32), ("shape", C.c_int64 * 4),
                ("off", C.c_int64), ("nbytes", C.c_int64)]


class K3dStackCfg(C.Structure):
    _fields_ = [("hidden", i32), ("vocab", i32), ("n_layers", i32), ("eps", f32),
                ("kda_heads", i32), ("kda_head_dim", i32), ("conv_k", i32), ("gate_lb", f32),
                ("mla", K3dMlaShape), ("moe", K3dMoeShape), ("first_dense", i32),
                ("dense_inter", i32), ("mla_layers", i32 * 16), ("batch", i32),
                ("ctx_cap", i32), ("ep_tokens", i32)]


# name -> (restype, argtypes)
_PROTOS = {
    # k3.h
    "k3_is_mla": (i32, [C.POINTER(K3Cfg), i32]),
    "k3_is_kda": (i32, [C.POINTER(K3Cfg), i32]),
    "k3_is_dense": (i32, [C.POINTER(K3Cfg), i32]),
    "k3_rmsnorm": (None, [vp, vp, vp, i32, f32]),
    "k3_situ_glu": (None, [vp, vp, i32, f32, f32]),
    "k3_shortconv": (None, [vp, vp, vp, vp, i32, i32, i32]),
    "k3_kda_decay": (None, [vp, vp, vp, vp, vp, i32, i32, f32]),
    "k3_kda_step": (None, [vp, vp, vp, vp, vp, vp, f32, i32, i32]),
    "k3_matmul": (None, [vp, vp, vp, i32, i32]),
    "k3_mla_scratch": (sz, [C.POINTER(K3Cfg), i32]),
    "k3_mla_scratch_cached": (sz, [C.POINTER(K3Cfg), i32, i32, i32]),
    "k3_mla_cached": (None, [vp, vp, C.POINTER(K3MlaW), C.POINTER(K3Cfg), i32, vp, vp, vp, i32, i32]),
    "k3_mla": (None, [vp, vp, C.POINTER(K3MlaW), C.POINTER(K3Cfg), i32, vp]),
    "k3_router": (None, [vp, vp, vp, vp, vp, i32, i32, i32, i32, f32]),
    "k3_attn_res": (None, [vp, vp, vp, i32, i32, f32]),
    "k3_matmul_bf16": (None, [vp, vp, vp, i32, i32]),
    "k3_matmul_q8": (None, [vp, vp, vp, i32, i32]),
    "k3_moe_scratch": (sz, [C.POINTER(K3Cfg)]),
    "k3_moe": (None, [vp, vp, C.POINTER(K3MoeW), C.POINTER(K3Cfg), i32, vp, vp, vp]),
    "k3_moe_prefill": (None, [vp, vp, C.POINTER(K3MoeW), C.POINTER(K3Cfg), i32, vp, vp, vp]),
    "k3_kda_scratch": (sz, [C.POINTER(K3Cfg), i32]),
    "k3_kda_layer": (None, [vp, vp, C.POINTER(K3KdaW), C.POINTER(K3Cfg), i32, vp, vp]),
    "k3_layer_scratch": (sz, [C.POINTER(K3Cfg), i32]),
    "k3_decoder_layer": (None, [vp, vp, vp, C.POINTER(K3LayerW), C.POINTER(K3Cfg), i32, i32, vp, vp]),
    "k3_decoder_layer_inc": (None, [vp, vp, vp, C.POINTER(K3LayerW), C.POINTER(K3Cfg), i32, i32,
                                    vp, vp, vp, vp, i32, i32]),
    "k3_mxfp4_dequant": (None, [vp, vp, vp, i32, i32, i32]),
    "k3_matmul_mxfp4": (None, [vp, vp, vp, vp, i32, i32, i32]),
    # k3_cuda.h: context
    "k3d_init": (i32, [i32]),
    "k3d_device": (i32, []),
    "k3d_status": (i32, []),
    "k3d_clear_status": (None, []),
    "k3d_strerror": (C.c_char_p, [i32]),
    "k3d_last_message": (C.c_char_p, []),
    "k3d_set_abort_on_error": (None, [i32]),
    "k3d_device_error": (i32, [C.POINTER(i32), C.POINTER(i32)]),
    "k3d_set_wait_limit": (i32, [C.c_longlong]),
    "k3d_alloc": (vp, [sz]),
    "k3d_free": (None, [vp]),
    "k3d_upload": (i32, [vp, vp, sz]),
    "k3d_download": (i32, [vp, vp, sz]),
    "k3d_memset": (i32, [vp, i32, sz]),
    "k3d_copy": (i32, [vp, vp, sz]),
    "k3d_copy2d": (i32, [vp, C.c_size_t, vp, C.c_size_t, C.c_size_t, C.c_size_t]),
    "k3d_set_weight_cache": (None, [i32]),
    "k3d_forget": (None, [vp]),
    "k3d_forget_all": (None, []),
    "k3d_weight_cache_bytes": (sz, []),
    "k3d_sync": (i32, []),
    "k3d_stream": (vp, []),
    "k3d_set_stream": (i32, [vp]),
    "k3d_event_create": (vp, []),
    "k3d_event_record": (i32, [vp]),
    "k3d_event_elapsed_ms": (f32, [vp, vp]),
    "k3d_event_destroy": (None, [vp]),
    "k3d_graph_begin": (i32, []),
    "k3d_graph_end": (vp, []),
    "k3d_set_graph_priorities": (i32, [i32]),
    "k3d_graph_launch": (i32, [vp]),
    "k3d_graph_destroy": (None, [vp]),
    "k3d_host_alloc": (vp, [sz]),
    "k3d_host_free": (None, [vp]),
    "k3d_prof_enable": (None, [i32]),
    "k3d_prof_reset": (None, []),
    "k3d_prof_ms": (C.c_double, [C.c_char_p, C.POINTER(C.c_long)]),
    "k3d_launch_count": (C.c_long, []),
    "k3d_launch_count_reset": (None, []),
    "k3d_sm_count": (i32, []),
    # fills
    "k3d_fill_bf16_normal": (i32, [vp, sz, u64, f32]),
    "k3d_fill_bf16_normal_at": (i32, [vp, sz, u64, f32, sz]),
    "k3d_fill_f32_normal": (i32, [vp, sz, u64, f32]),
    "k3d_fill_f32_uniform": (i32, [vp, sz, u64, f32, f32]),
    "k3d_fill_mxfp4": (i32, [vp, sz, vp, sz, u64, i32, i32]),
    "k3d_fill_i32_uniform": (i32, [vp, sz, u64, i32, i32]),
    # experts / MoE
    "k3d_expert_ws_bytes": (sz, [i32, i32]),
    "k3d_expert_swiglu": (i32, [vp, vp, C.POINTER(K3ExpertQ), i32, i32, vp, sz]),
    "k3d_moe_ws_bytes": (sz, [C.POINTER(K3dMoeShape), i32]),
    "k3d_moe_swiglu": (i32, [vp, vp, C.POINTER(K3dMoeW), C.POINTER(K3dMoeShape), i32, i32, vp, vp,
                             vp, sz]),
    "k3d_router_bf16": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32]),
    "k3d_set_expert_kernel": (i32, [i32]),
    "k3d_expert_pretile": (i32, [C.POINTER(K3ExpertQ), C.POINTER(K3ExpertQ), i32, i32]),
    "k3d_router_bf16_noalloc": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32]),
    "k3d_moe_last_unique": (i32, []),
    "k3d_router_fallbacks": (C.c_longlong, []),
    "k3d_gemv_bf16": (i32, [vp, vp, vp, i32, i32, i32, i32]),
    # KDA / MLA / small
    "k3d_kda_decode": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]),
    "k3d_kda_prefill": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32]),
    "k3d_mla_ws_bytes": (sz, [C.POINTER(K3dMlaShape), i32, i32]),
    "k3d_mla_decode": (i32, [vp, vp, C.POINTER(K3dMlaW), C.POINTER(K3dMlaShape), i32, vp, i32, vp,
                             i32, vp, sz]),
    "k3d_mla_decode_normed": (i32, [vp, vp, vp, f32, C.POINTER(K3dMlaW), C.POINTER(K3dMlaShape), i32, vp,
                                    i32, vp, i32, vp, sz]),
    "k3d_rmsnorm": (i32, [vp, vp, vp, i32, i32, f32]),
    "k3d_embed_bf16": (i32, [vp, vp, vp, i32, i32, i32]),
    "k3d_swiglu_mlp_bf16": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "k3d_lm_head_argmax": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
    "k3d_lm_head_argmax_normed": (i32, [vp, vp, vp, vp, f32, vp, i32, i32, i32, vp]),
    "k3d_lm_head_argmax_shard_normed": (i32, [vp, vp, vp, vp, f32, vp, i32, i32, i32, i32, vp]),
    "k3d_add_f32": (i32, [vp, vp, sz]),
    "k3d_add_i32": (i32, [vp, i32, i32]),
    "k3d_kda_layer_ws_bytes": (sz, [C.POINTER(K3dKdaShape), i32]),
    "k3d_kda_state_floats": (sz, [C.POINTER(K3dKdaShape)]),
    "k3d_set_kda_head_kernel": (i32, [i32]),
    "k3d_fill_f32_normal_at": (i32, [vp, sz, C.c_uint64, f32, sz]),
    "k3d_fill_f32_uniform_at": (i32, [vp, sz, C.c_uint64, f32, f32, sz]),
    "k3d_state_peek": (i32, [C.c_char_p, C.POINTER(K3dStateInfo)]),
    "k3d_ckpt_open": (vp, [C.c_char_p]),
    "k3d_ckpt_close": (None, [vp]),
    "k3d_ckpt_count": (i32, [vp]),
    "k3d_ckpt_find": (i32, [vp, C.c_char_p, C.POINTER(K3dCkptTensor)]),
    "k3d_ckpt_read": (C.c_int64, [vp, i32, C.c_int64, C.c_int64, vp]),
    "k3d_ckpt_elem_size": (i32, [i32]),
    "k3d_ckpt_error": (C.c_char_p, []),
    "k3d_model_load_checkpoint": (i32, [vp, vp]),
    "k3d_model_state_save": (i32, [vp, C.c_char_p, vp, i32, i32]),
    "k3d_model_state_load": (i32, [vp, C.c_char_p, vp, i32, i32]),
    "k3d_bf16_rows_to_f32": (i32, [vp, vp, sz, i32, i32]),
    "k3d_f32_rows_to_bf16": (i32, [vp, sz, vp, i32, i32]),
    "k3d_transpose_u16": (i32, [vp, vp, i32, i32]),
    "k3d_kda_layer_decode_normed_out": (i32, [vp, vp, vp, f32, C.POINTER(K3dKdaW), C.POINTER(K3dKdaShape), i32,
                                              vp, vp, sz, i32]),
    "k3d_kda_layer_decode": (i32, [vp, vp, C.POINTER(K3dKdaW), C.POINTER(K3dKdaShape), i32, vp, vp, sz]),
    "k3d_kda_layer_decode_normed": (i32, [vp, vp, f32, C.POINTER(K3dKdaW), C.POINTER(K3dKdaShape), i32,
                                          vp, vp, sz]),
    "k3d_silu_mul": (i32, [vp, vp, i32, i32]),
    # EP
    "k3d_ep_unique_id": (i32, [vp]),
    "k3d_ep_init": (i32, [i32, i32, vp]),
    "k3d_ep_finalize": (i32, []),
    "k3d_ep_rank": (i32, []),
    "k3d_ep_size": (i32, []),
    "k3d_ep_allreduce_f32": (i32, [vp, sz]),
    "k3d_ep_peer_init": (i32, [C.c_size_t]),
    "k3d_set_ep_combine": (i32, [i32]),
    "k3d_ep_combine_add": (i32, [vp, vp, C.c_size_t, i32]),
    "k3d_moe_a2a_ws_bytes": (sz, [C.POINTER(K3dMoeShape), i32, i32]),
    "k3d_moe_swiglu_a2a_dev": (i32, [vp, vp, C.POINTER(K3dMoeW), C.POINTER(K3dMoeShape), i32, i32, vp, vp, vp, sz]),
    "k3d_moe_swiglu_a2a": (i32, [vp, vp, C.POINTER(K3dMoeW), C.POINTER(K3dMoeShape), i32, i32, i32, vp,
                                 vp, vp, sz]),
    "k3d_a2a_plan": (i32, [vp, i32, i32, i32, vp, vp, vp]),
    # stack
    "k3d_model_create": (vp, [C.POINTER(K3dStackCfg), u64]),
    "k3d_model_destroy": (None, [vp]),
    "k3d_model_fill_context": (i32, [vp, i32, u64]),
    "k3d_model_step_dev": (i32, [vp, vp, vp, vp]),
    "k3d_model_step_host": (i32, [vp, vp, vp]),
    "k3d_model_use_graph": (i32, [vp, i32]),
    "k3d_model_tensor": (vp, [vp, C.c_char_p, C.POINTER(sz)]),
    "k3d_model_last_step_bytes": (C.c_double, [vp]),
}

_lib = None


def load(path=LIB_PATH):
    """Load libk3cuda.so and declare its prototypes. Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `make -C {HERE}` (or __graft_entry__.build()); "
            "there is no CPU implementation to fall back to")
    lib = C.CDLL(path)
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_names():
    return list(_PROTOS)


class K3Error(RuntimeError):
    pass


def check(code, what=""):
    if code:
        lib = load()
        msg = lib.k3d_last_message().decode(errors="replace")
        raise K3Error(f"{what}: k3cuda error {code} ({lib.k3d_strerror(code).decode()}): {msg}")


def init(device=0):
    lib = load()
    check(lib.k3d_init(device), "k3d_init")
    return lib


class DevBuf:
    """A device allocation from k3d_alloc with numpy transfer helpers."""

    def __init__(self, nbytes, lib=None):
        self.lib = lib or load()
        self.nbytes = int(nbytes)
        self.ptr = self.lib.k3d_alloc(max(self.nbytes, 16))
        if not self.ptr:
            raise K3Error(f"k3d_alloc({nbytes}) failed: {self.lib.k3d_last_message().decode()}")

    @classmethod
    def from_array(cls, arr, lib=None):
        arr = np.ascontiguousarray(arr)
        b = cls(arr.nbytes, lib)
        b.upload(arr)
        return b

    def upload(self, arr):
        arr = np.ascontiguousarray(arr)
        assert arr.nbytes <= self.nbytes
        check(self.lib.k3d_upload(self.ptr, arr.ctypes.data, arr.nbytes), "upload")

    def download(self, dtype, shape):
        out = np.empty(shape, dtype=dtype)
        assert out.nbytes <= self.nbytes
        check(self.lib.k3d_download(out.ctypes.data, self.ptr, out.nbytes), "download")
        return out

    def zero(self):
        check(self.lib.k3d_memset(self.ptr, 0, self.nbytes), "memset")

    def free(self):
        if self.ptr:
            self.lib.k3d_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def __int__(self):
        return self.ptr

    @property
    def value(self):
        return self.ptr


def _align(n, a=256):
    return (n + a - 1) // a * a


class MoeWeights:
    """Device-resident weights of one MoE layer at the benchmark shapes: an MXFP4 expert
    table (experts [lo, hi) only), a bf16 router and an optional bf16 shared expert.

    Either `experts` (a list of numpy dicts p1,s1,p3,s3,p2,s2 for every expert id, None for
    absent ones) or `seed` (device-side fill, E8M0 bytes in [s_lo, s_hi]) supplies the
    expert bytes."""

    def __init__(self, hidden, inter, n_experts, topk, router_w, router_bias, shared=None,
                 experts=None, seed=None, lo=0, hi=None, s_lo=117, s_hi=121, renorm=1,
                 routed_scale=2.5, add_shared=1, tiled=False, lib=None):
        self.lib = lib or load()
        hi = n_experts if hi is None else hi
        self.shape = K3dMoeShape(hidden, inter, n_experts, topk, renorm, routed_scale,
                                 shared[0].shape[0] if shared is not None else 0, lo, hi,
                                 add_shared, 1 if tiled else 0)
        gu = inter * hidden // 2
        gus = inter * hidden // 32
        sizes = [gu, gus, gu, gus, gu, gus]
        offs = []
        o = 0
        for s in sizes:
            offs.append(o)
            o += _align(s)
        self.per_expert = o
        n_local = hi - lo
        self.pool = DevBuf(max(1, n_local) * o, self.lib)
        # tiled: the checkpoint bytes go to a staging expert and k3d_expert_pretile writes
        # the pool slot as [gate/up codes 2*gu][gate/up scales 2*gus][down codes][down scales]
        tsizes = [2 * gu, 2 * gus, gu, gus]
        toffs = []
        o2 = 0
        for s_ in tsizes:
            toffs.append(o2)
            o2 += _align(s_)
        assert o2 <= o
        stage = DevBuf(o, self.lib) if tiled else None
        table = (K3ExpertQ * n_experts)()
        for e in range(lo, hi):
            base = self.pool.ptr + (e - lo) * o
            src_base = stage.ptr if tiled else base
            ptrs = [src_base + off for off in offs]
            if experts is not None:
                for key, p in zip(("p1", "s1", "p3", "s3", "p2", "s2"), ptrs):
                    a = np.ascontiguousarray(experts[e][key])
                    check(self.lib.k3d_upload(p, a.ctypes.data, a.nbytes), "expert upload")
            else:
                for j in range(3):
                    check(self.lib.k3d_fill_mxfp4(ptrs[2 * j], sizes[2 * j], ptrs[2 * j + 1],
                                                  sizes[2 * j + 1], seed * 7919 + e * 3 + j,
                                                  s_lo, s_hi), "expert fill")
            if tiled:
                tp = [base + off for off in toffs]
                dst = K3ExpertQ(tp[0], tp[1], None, None, tp[2], tp[3])
                check(self.lib.k3d_expert_pretile(C.byref(dst), C.byref(K3ExpertQ(*ptrs)),
                                                  hidden, inter), "expert pretile")
                check(self.lib.k3d_sync(), "pretile")     # the staging expert is reused
                table[e] = dst
            else:
                table[e] = K3ExpertQ(*ptrs)
        self.tiled = tiled
        self.table_host = table
        self.offs = offs
        self.sizes = sizes
        self.table = DevBuf(C.sizeof(table), self.lib)
        check(self.lib.k3d_upload(self.table.ptr, C.addressof(table), C.sizeof(table)))
        self.router_w = DevBuf.from_array(np.ascontiguousarray(router_w, np.uint16), self.lib)
        self.router_b = DevBuf.from_array(np.ascontiguousarray(router_bias, np.float32), self.lib)
        self.sh = [DevBuf.from_array(np.ascontiguousarray(a, np.uint16), self.lib)
                   for a in shared] if shared is not None else [None, None, None]
        self.w = K3dMoeW(self.router_w.ptr, self.router_b.ptr, self.table.ptr,
                         *(b.ptr if b is not None else None for b in self.sh))

    def expert_bytes(self):
        return sum(self.sizes)

    def download_expert(self, e):
        assert not self.tiled, "tiled experts hold no checkpoint-layout copy"
        q = self.table_host[e]
        out = {}
        for key, size in zip(("p1", "s1", "p3", "s3", "p2", "s2"), self.sizes):
            a = np.empty(size, np.uint8)
            check(self.lib.k3d_download(a.ctypes.data, getattr(q, key), size))
            out[key] = a
        return out

    def ws_bytes(self, T):
        return self.lib.k3d_moe_ws_bytes(C.byref(self.shape), T)

    def run(self, out, x, T, ws, ws_bytes, accumulate=0, idx=None, wts=None):
        return self.lib.k3d_moe_swiglu(out, x, C.byref(self.w), C.byref(self.shape), T,
                                       accumulate, idx, wts, ws, ws_bytes)

    def a2a_ws_bytes(self, t_max, nranks):
        return self.lib.k3d_moe_a2a_ws_bytes(C.byref(self.shape), t_max, nranks)

    def run_a2a(self, out, x, T, t_max, ws, ws_bytes, accumulate=0, idx=None, wts=None):
        """Mode A: this rank's own T tokens, experts dispatched to their ranks."""
        return self.lib.k3d_moe_swiglu_a2a(out, x, C.byref(self.w), C.byref(self.shape), T, t_max,
                                           accumulate, idx, wts, ws, ws_bytes)

    def run_a2a_dev(self, out, x, T, ws, ws_bytes, accumulate=0, idx=None, wts=None):
        """Mode A planned on the device (graph-capturable): every rank passes the same T."""
        return self.lib.k3d_moe_swiglu_a2a_dev(out, x, C.byref(self.w), C.byref(self.shape), T, accumulate,
                                               idx, wts, ws, ws_bytes)


def a2a_plan(idx, n_experts, nranks, lib=None):
    """k3d_a2a_plan on host arrays: (cnt[nranks], off[nranks], pos[len(idx)])."""
    lib = lib or load()
    idx = np.ascontiguousarray(idx, np.int32).reshape(-1)
    cnt = np.zeros(nranks, np.int32)
    off = np.zeros(nranks, np.int32)
    pos = np.zeros(idx.size, np.int32)
    check(lib.k3d_a2a_plan(idx.ctypes.data, idx.size, n_experts, nranks, cnt.ctypes.data,
                           off.ctypes.data, pos.ctypes.data), "k3d_a2a_plan")
    return cnt, off, pos
