"""Expert parallelism's MoE combine over NVLink peer memory (k3d_ep_combine_add) and the
decode stack under expert parallelism (Mode R, and Mode A with the batch split), on two GPUs (one process per GPU, gloo for the
test's own bookkeeping, CUDA IPC for the peer buffers). On one GPU, the combine is the
plain residual add."""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import k3cuda
from test_gpu_ep_a2a import _gpu_count

pytestmark = pytest.mark.gpu


def test_combine_one_rank_is_the_residual_add(k3):
    g = np.random.default_rng(5)
    h0 = g.standard_normal(7168).astype(np.float32)
    p = g.standard_normal(7168).astype(np.float32)
    H, P = k3cuda.DevBuf.from_array(h0), k3cuda.DevBuf.from_array(p)
    k3cuda.check(k3.k3d_ep_combine_add(H.ptr, P.ptr, 7168, 1))
    k3cuda.check(k3.k3d_sync())
    assert np.array_equal(H.download(np.float32, 7168), (h0 + p).astype(np.float32))


def _run_two(target, *args):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=(r, 2, port) + args) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], codes


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_push_combine_two_gpus_equals_rank_order_sum():
    import ep_combine_gpu_worker
    _run_two(ep_combine_gpu_worker.run_combine, 7)


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("batch,mla_heads", [(1, None), (6, None), (1, 16)])
def test_stack_two_gpus_matches_one_gpu(batch, mla_heads):
    import ep_combine_gpu_worker
    _run_two(ep_combine_gpu_worker.run_stack, 99, batch, mla_heads)


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("batch", [12, 64])
def test_stack_mode_a_two_gpus_matches_one_gpu(batch):
    import ep_combine_gpu_worker
    _run_two(ep_combine_gpu_worker.run_stack_mode_a, 99, batch)
