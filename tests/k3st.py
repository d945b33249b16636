"""The conversation-state file of the CPU engine (K3ST version 1, src/cli/k3_run.c:175-300)
for the tests: header packing, and a reader that splits a file into its sections the way the
CPU engine's k3_state_load reads them, plus the device trailer ("K3LT") this library appends."""
import struct

import numpy as np

HDR = struct.Struct("<4si12i4iqqq")        # magic, version, fp[12], n_bound, n_mla, cached, nseq, kper, kvpp, ropepp
TRL = struct.Struct("<4s4i")               # magic, version, n_mla, cached, kvw
assert HDR.size == 96 and TRL.size == 20


def fingerprint(hidden, n_layers, vocab, kda_heads, kda_head_dim, conv_k, n_heads, qk_nope, qk_rope,
                v_head, n_experts, topk):
    return [hidden, n_layers, vocab, kda_heads, kda_head_dim, conv_k, n_heads, qk_nope, qk_rope, v_head,
            n_experts, topk]


def pack(fp, seq, ks, kvc, ropec, latent=None, version=1):
    """ks [n_bound][kper], kvc [n_mla][cached][kvpp], ropec [n_mla][cached][ropepp] (float32);
    latent [n_mla][cached][kvw] uint16 adds the trailer."""
    seq = np.asarray(seq, np.int32)
    n_bound, kper = ks.shape
    n_mla, cached, kvpp = kvc.shape
    ropepp = ropec.shape[2]
    out = [HDR.pack(b"K3ST", version, *fp, n_bound, n_mla, cached, len(seq), kper, kvpp, ropepp),
           seq.tobytes(), np.ascontiguousarray(ks, np.float32).tobytes(),
           np.ascontiguousarray(kvc, np.float32).tobytes(), np.ascontiguousarray(ropec, np.float32).tobytes()]
    if latent is not None:
        out.append(TRL.pack(b"K3LT", 1, n_mla, cached, latent.shape[2]))
        out.append(np.ascontiguousarray(latent, np.uint16).tobytes())
    return b"".join(out)


def unpack(data):
    h = HDR.unpack_from(data, 0)
    magic, version, fp = h[0], h[1], list(h[2:14])
    n_bound, n_mla, cached, nseq, kper, kvpp, ropepp = h[14:]
    o = HDR.size
    seq = np.frombuffer(data, np.int32, nseq, o); o += 4 * nseq
    ks = np.frombuffer(data, np.float32, n_bound * kper, o).reshape(n_bound, kper); o += 4 * n_bound * kper
    kvc = np.frombuffer(data, np.float32, n_mla * cached * kvpp, o).reshape(n_mla, cached, kvpp)
    o += 4 * n_mla * cached * kvpp
    ropec = np.frombuffer(data, np.float32, n_mla * cached * ropepp, o).reshape(n_mla, cached, ropepp)
    o += 4 * n_mla * cached * ropepp
    latent = None
    payload_end = o
    if len(data) >= o + TRL.size:
        t = TRL.unpack_from(data, o)
        if t[0] == b"K3LT":
            o += TRL.size
            latent = np.frombuffer(data, np.uint16, t[2] * t[3] * t[4], o).reshape(t[2], t[3], t[4])
    return dict(magic=magic, version=version, fp=fp, n_bound=n_bound, n_mla=n_mla, cached=cached, seq=seq,
                ks=ks, kvc=kvc, ropec=ropec, latent=latent, kper=kper, kvpp=kvpp, ropepp=ropepp,
                payload_end=payload_end)
