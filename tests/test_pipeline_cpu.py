"""The layer-pipeline schedule (tests/pipeline_schedule.py, the step order of the native pipeline) on CPU: world-size-2 and -3 gloo process
groups, micro-batches, ids flowing back to rank 0, against the same stages run in one process.

The stand-in stage has the interface of the CUDA stage (embed / forward / pick on row ranges, each
sequence with its own position) and a cheap deterministic layer function, so the test checks the
schedule and the data movement, not the model.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, V, L = 8, 50, 6


class FakeStage:
    """Layers [l0, l1) of a toy model: x <- tanh(x * (1 + 0.1 l) + 0.01 pos); head: id = argmax(W x)."""

    def __init__(self, l0, l1, has_head, n_seq):
        self.l0, self.l1, self.has_head, self.first = l0, l1, has_head, l0 == 0
        self.pos = np.zeros(n_seq, np.int64)
        self.device = torch.device("cpu")
        rng = np.random.default_rng(3)
        self.emb = rng.standard_normal((V, E)).astype(np.float32)
        self.W = rng.standard_normal((V, E)).astype(np.float32)

    def new_x(self, n):
        return torch.zeros((n, E), dtype=torch.float32)

    def new_ids(self, n):
        return torch.zeros(n, dtype=torch.int32)

    def sync(self):
        pass

    def embed(self, ids, x):
        x.copy_(torch.from_numpy(self.emb[ids.numpy()]))

    def forward(self, x, r0, n):
        a = x.numpy()
        for l in range(self.l0, self.l1):
            a = np.tanh(a * (1 + 0.1 * l) + 0.01 * self.pos[r0:r0 + n, None])
        x.copy_(torch.from_numpy(a.astype(np.float32)))
        self.pos[r0:r0 + n] += 1

    def pick(self, x, r0, n, ids):
        ids.copy_(torch.from_numpy(np.argmax(x.numpy() @ self.W.T, axis=1).astype(np.int32)))


def reference(prompts, n_gen):
    import pipeline_schedule as pl  # noqa: F401  (same import path as the workers)
    st = FakeStage(0, L, True, prompts.shape[0])
    out = []
    ids = None
    for i in range(prompts.shape[1] + n_gen - 1):
        src = prompts[:, i] if i < prompts.shape[1] else ids
        x = st.new_x(prompts.shape[0])
        st.embed(torch.from_numpy(np.ascontiguousarray(src, np.int32)), x)
        st.forward(x, 0, prompts.shape[0])
        if i >= prompts.shape[1] - 1:
            t = st.new_ids(prompts.shape[0])
            st.pick(x, 0, prompts.shape[0], t)
            ids = t.numpy()
            out.append(ids.copy())
    return np.stack(out, axis=1)


def worker(rank, world, port, prompts, n_gen, n_mb, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    import pathlib
    sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))
    from conftest import load_pkg
    load_pkg()
    import pipeline_schedule as pl
    dist.init_process_group("gloo", rank=rank, world_size=world)
    gx, gt = dist.new_group(list(range(world))), dist.new_group(list(range(world)))
    l0, l1 = pl.split_layers(L, world)[rank]
    st = FakeStage(l0, l1, rank == world - 1, prompts.shape[0])
    p = pl.Pipeline(st, rank, world, prompts.shape[0], n_mb, gx, gt)
    out = p.decode(prompts if rank == 0 else None, n_gen)
    if rank == 0:
        q.put(out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,n_mb", [(2, 1), (2, 3), (3, 2)])
def test_pipeline_schedule_matches_single_process(world, n_mb):
    rng = np.random.default_rng(5)
    prompts = rng.integers(0, V, (7, 4)).astype(np.int32)
    n_gen = 6
    want = reference(prompts, n_gen)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + 10 * world + n_mb
    procs = [ctx.Process(target=worker, args=(r, world, port, prompts, n_gen, n_mb, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    got = q.get(timeout=120)
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    assert np.array_equal(got, want)


def test_split_helpers():
    import pipeline_schedule as pl
    assert pl.split_layers(28, 2) == [(0, 14), (14, 28)]
    assert pl.split_layers(7, 3) == [(0, 3), (3, 5), (5, 7)]
    assert pl.micro_batches(7, 3) == [(0, 3), (3, 2), (5, 2)]
    assert pl.micro_batches(2, 5) == [(0, 1), (1, 1)]
