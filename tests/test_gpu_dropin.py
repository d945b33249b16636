"""The drop-in relink: the reference engine's own unit tests, compiled against this
repository's include/k3/k3.h and linked with libk3cuda.so in place of k3_ops.o
(oracle/Makefile, target `dropin`), run on the B200 with the reference's own fixtures and
pass criteria.

  test_ops  (tests/unit/test_ops.c:850-896 of the reference): every kernel against its
            fixture at the MANIFEST.json tolerance; the bar is "22 passed, 0 failed,
            0 skipped" and exit status 0.
  k3_model  (tests/unit/k3_model.c:323-430): the tiny 13-layer model's exact-token gates
            (teacher forcing, state reuse bit-identical, greedy and incremental decode);
            the bar is its VERDICT line and exit status 0.

The binaries and a copy of the fixtures live in oracle/_ref (built where the reference
tree exists; they travel with the repository to the GPU host)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(REPO, "oracle", "_ref")


def run(binary, arg):
    exe = os.path.join(REF, binary)
    if not os.path.exists(exe):
        pytest.skip(f"{binary} not built (oracle/Makefile target dropin needs the reference tree)")
    p = subprocess.run([exe, arg], capture_output=True, text=True, timeout=600)
    return p.returncode, p.stdout + p.stderr


def test_reference_test_ops_passes_on_libk3cuda():
    rc, out = run("test_ops_k3cuda", os.path.join(REF, "fixtures", "ops"))
    assert "22 passed, 0 failed, 0 skipped" in out, out[-3000:]
    assert rc == 0, out[-3000:]


def test_reference_k3_model_gates_pass_on_libk3cuda():
    rc, out = run("k3_model_k3cuda", os.path.join(REF, "fixtures"))
    assert "VERDICT: ENGINE MATCHES THE REFERENCE EXACTLY" in out, out[-3000:]
    assert rc == 0, out[-3000:]
