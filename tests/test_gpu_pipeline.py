"""Two-GPU layer pipeline over NCCL (meta-work_b200/pipeline.py with CUDA stages) against the same batch
decoded on one GPU: every stage runs the single-GPU batch kernels on its layer range, and a token's
GEMV column does not depend on the micro-batch it shares a launch with, so the ids must be identical.
Needs two GPUs (skipped otherwise)."""
from __future__ import annotations

import datetime
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def worker(rank, world, port, path, prompts, n_gen, n_mb, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import sys
    import pathlib
    sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
    from conftest import load_pkg
    load_pkg()
    import torch.distributed as dist
    from xjb200 import pipeline as pl, xjcuda
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120), device_id=dev)
    gx, gt = dist.new_group(list(range(world))), dist.new_group(list(range(world)))
    m = xjcuda.Model(path)
    l0, l1 = pl.split_layers(m.n_layer, world)[rank]
    st = pl.CudaStage(m, l0, l1, rank == world - 1, prompts.shape[0], 256, dev)
    p = pl.Pipeline(st, rank, world, prompts.shape[0], n_mb, gx, gt)
    out = p.decode(prompts if rank == 0 else None, n_gen)
    if rank == 0:
        q.put(out)
    dist.barrier()
    st.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("n_mb", [1, 2])
def test_two_gpu_pipeline_matches_one_gpu_batch(mid_path, n_mb):
    from xjb200 import xjcuda
    rng = np.random.default_rng(9)
    m = xjcuda.Model(mid_path)
    prompts = rng.integers(0, m.n_vocab, (6, 12)).astype(np.int32)
    n_gen = 16
    b = xjcuda.Batch(m, 6, 256)
    want, _, _ = b.decode(prompts, n_gen)
    b.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + n_mb
    procs = [ctx.Process(target=worker, args=(r, 2, port, str(mid_path), prompts, n_gen, n_mb, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    got = q.get(timeout=300)
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    assert np.array_equal(got, want)
