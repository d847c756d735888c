"""Layer pipeline across GPUs over NCCL, natively in libxj_cuda.so (xj_cuda_pipeline_*): one process per
GPU, each holding the batch kernels on its layer range, activations and token ids sent by NCCL. Against
the same batch decoded on one GPU: a token's matrix-product column does not depend on the micro-batch
it shares a launch with, so the ids must be identical. The one-rank pipeline runs on any GPU; the
multi-rank cases need as many GPUs (skipped otherwise). The communicator identifier goes from rank 0 to
the other ranks through a multiprocessing queue (the host's choice of channel)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def worker(rank, world, path, prompts, n_gen, n_mb, steps_after, idq, outq):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import pathlib
    import sys
    sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
    from conftest import load_pkg
    load_pkg()
    from xjb200 import xjcuda
    torch.cuda.set_device(rank)
    if rank == 0:
        pid = xjcuda.pipeline_id()
        for _ in range(world - 1):
            idq.put(pid)
    else:
        pid = idq.get(timeout=120)
    m = xjcuda.Model(path)
    p = xjcuda.Pipeline(m, rank, world, pid, prompts.shape[0], 256, n_mb)
    out, _ = p.decode(prompts if rank == 0 else prompts.shape[1], n_gen)
    more = None
    if steps_after:
        # continuation: the last id as a one-token prompt (positions continue)
        more, _ = p.decode(out[:, -1:] if rank == 0 else 1, steps_after)
    if rank == 0:
        outq.put((out, more))
    p.close()


def run_ranks(world, path, prompts, n_gen, n_mb, steps_after=0):
    ctx = mp.get_context("spawn")
    idq, outq = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=worker, args=(r, world, str(path), prompts, n_gen, n_mb, steps_after, idq, outq))
             for r in range(world)]
    for pr in procs:
        pr.start()
    got = outq.get(timeout=600)
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    return got


def one_gpu(path, prompts, n_gen):
    from xjb200 import xjcuda
    m = xjcuda.Model(path)
    b = xjcuda.Batch(m, prompts.shape[0], 256)
    want, _, _ = b.decode(prompts, n_gen)
    b.close()
    return want


@pytest.mark.parametrize("n_mb", [1, 3])
def test_one_rank_pipeline_matches_batch(mid_path, n_mb):
    from xjb200 import xjcuda
    rng = np.random.default_rng(7)
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (6, 10)).astype(np.int32)
    want = one_gpu(mid_path, prompts, 12)
    p = xjcuda.Pipeline(m, 0, 1, None, 6, 256, n_mb)
    got, ms = p.decode(prompts, 12)
    p.close()
    assert np.array_equal(got, want) and ms > 0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("n_mb", [1, 2])
def test_two_gpu_pipeline_matches_one_gpu_batch(mid_path, n_mb):
    rng = np.random.default_rng(9)
    from xjb200 import xjcuda
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (6, 12)).astype(np.int32)
    want = one_gpu(mid_path, prompts, 16 + 8)
    got, more = run_ranks(2, mid_path, prompts, 16, n_mb, steps_after=8)
    assert np.array_equal(got, want[:, :16])
    assert np.array_equal(more, want[:, 16:])


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_four_gpu_pipeline_matches_one_gpu_batch(mid_path):
    rng = np.random.default_rng(10)
    from xjb200 import xjcuda
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (8, 9)).astype(np.int32)
    want = one_gpu(mid_path, prompts, 12)
    got, _ = run_ranks(4, mid_path, prompts, 12, 4)
    assert np.array_equal(got, want)
