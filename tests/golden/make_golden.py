"""Regenerates the golden fixtures under tests/golden/ (run where the reference tree exists).

1. ref_ops/*.npz, mxfp4.npz: the reference engine's own golden vectors
   (tests/fixtures/ops/*.json and tests/fixtures/mxfp4.json of libxsmm/kimi-k3-in-c, made
   by its tools/emit_fixtures.py from the pure-torch model), converted to npz so the GPU
   hosts, which have no copy of the reference tree, can read them.
2. ref_*.npz: outputs of the reference's compiled k3_ops.c (oracle/_ref/libk3ref.so) on
   seeded synthetic inputs at the benchmark shapes (tests/golden/synth.py), with a digest
   of the inputs.

    python tests/golden/make_golden.py --reference <path of the reference source tree>
"""
import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(REPO, "oracle"))

import synth  # noqa: E402

INT_KEYS = {"topk_idx", "packed", "scales"}


def convert_fixture(path, out_path):
    d = json.load(open(path))
    arrays, meta = {}, {}
    for k, v in d.items():
        if isinstance(v, dict) and "first64" in v:
            arrays[k] = np.asarray(v["first64"], dtype=np.float32)
            meta[k + ".note"] = v.get("note", "")
        elif isinstance(v, dict) and "data" in v:
            shape = tuple(v.get("shape", [len(v["data"])]))
            if k in INT_KEYS:
                dt = np.uint8 if k in ("packed", "scales") else np.int32
            else:
                dt = np.float32
            arrays[k] = np.asarray(v["data"], dtype=dt).reshape(shape)
            if "note" in v:
                meta[k + ".note"] = v["note"]
        elif isinstance(v, list) and all(isinstance(t, (int, float)) for t in v):
            arrays[k] = np.asarray(v, dtype=np.float32)
        else:
            meta[k] = v
    arrays["__meta__"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(out_path, **arrays)


def reference_goldens():
    from oracle import Reference  # noqa: E402
    ref = Reference()
    # config 0: one MXFP4 SwiGLU expert at 7168 -> 2048 -> 7168, reference GEMVs + SiLU
    x, e = synth.config0_inputs()
    g = ref.matmul_mxfp4(x, e["p1"], e["s1"], 2048)
    u = ref.matmul_mxfp4(x, e["p3"], e["s3"], 2048)
    act = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u
    y = ref.matmul_mxfp4(act.astype(np.float32), e["p2"], e["s2"], 7168)
    np.savez_compressed(os.path.join(HERE, "ref_config0.npz"), gate=g, up=u, y=y,
                        digest=np.frombuffer(synth.digest(x, *e.values()).encode(), np.uint8))
    # router at the config-1 shape: bf16 W widened exactly to the fp32 the API takes
    x, W, bias = synth.router_inputs()
    Wf = synth.bf16_to_f32(W)
    idx, wts = [], []
    for t in range(x.shape[0]):
        i, w = ref.router(x[t], Wf, bias, 8, 1, 2.5)
        idx.append(i)
        wts.append(w)
    np.savez_compressed(os.path.join(HERE, "ref_router.npz"), idx=np.stack(idx), w=np.stack(wts),
                        digest=np.frombuffer(synth.digest(x, W, bias).encode(), np.uint8))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the reference source tree (read only)")
    args = ap.parse_args()
    fx = os.path.join(args.reference, "tests", "fixtures")
    os.makedirs(os.path.join(HERE, "ref_ops"), exist_ok=True)
    for name in sorted(os.listdir(os.path.join(fx, "ops"))):
        if name.endswith(".json") and name != "MANIFEST.json":
            convert_fixture(os.path.join(fx, "ops", name),
                            os.path.join(HERE, "ref_ops", name[:-5] + ".npz"))
    man = json.load(open(os.path.join(fx, "ops", "MANIFEST.json")))
    json.dump({"config": man["config"], "tolerance": man["tolerance"]},
              open(os.path.join(HERE, "ref_ops", "MANIFEST.json"), "w"), indent=1)
    convert_fixture(os.path.join(fx, "mxfp4.json"), os.path.join(HERE, "mxfp4.npz"))
    reference_goldens()
    print("golden fixtures written under", HERE)


if __name__ == "__main__":
    main()
