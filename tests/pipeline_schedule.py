"""A host-side model of the layer pipeline's schedule, for CPU tests (tests/test_pipeline_cpu.py): the
same step order as the native pipeline in libxj_cuda.so (meta-work_b200/csrc/pipeline.cpp), driven over
torch.distributed process groups (gloo on CPU) with stand-in stages. TEST INFRASTRUCTURE: the product's
pipeline is the native one; this model checks the schedule and the data movement without GPUs.

The reference splits a model into stages by layer range (``xj_net.h:93-111``: a|r|b) and drives them
with ``xj_pipeline_eval`` over TCP. Here every rank holds one stage: a batch of ``n_seq`` sequences
over its layer range (``xj_cuda_batch_new_range``), the first stage also embeds and the last also
owns the LM head and the greedy pick. Per decode step and micro-batch of rows:

    rank 0:      ids -> embed -> layers [0, l1)   -> send x ------------\\
    rank i:      recv x -> layers [l0, l1) -> send x                    | activations: group gx
    rank N-1:    recv x -> layers [l0, L) -> head + argmax -> send ids -/  ids: group gt (to rank 0)

Micro-batches keep the stages busy at the same time: while the last stage works on micro-batch k of
step s, the first stage already runs micro-batch k+1. Activations ([rows][n_embd] fp32) and ids go
over gloo here (NCCL in the native pipeline); they travel on two process groups, one per direction,
so a send in one direction never waits behind a receive in the other on one communicator. The last
rank sends each micro-batch's picks as soon as they are made, without waiting
for the send; rank 0 receives them only when the next step's micro-batch needs them. So the first
stage starts micro-batch k of the next step as soon as that micro-batch's picks exist, and no stream
ever holds a receive of activations behind a send of ids (which could deadlock the two communicators).
KV caches and recurrent state stay on the rank that owns the layer.

The per-stage compute is behind a small interface (``embed``, ``forward``, ``pick``), provided here by a
stand-in stage.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass

import numpy as np


def split_layers(n_layer: int, world: int) -> list[tuple[int, int]]:
    """Contiguous layer ranges, as even as possible, first ranges one longer when uneven."""
    base, extra = divmod(n_layer, world)
    out, l0 = [], 0
    for r in range(world):
        l1 = l0 + base + (1 if r < extra else 0)
        out.append((l0, l1))
        l0 = l1
    return out


def micro_batches(n_seq: int, n_mb: int) -> list[tuple[int, int]]:
    """Row ranges (row0, nrows) of n_mb micro-batches covering n_seq rows."""
    n_mb = max(1, min(n_mb, n_seq))
    base, extra = divmod(n_seq, n_mb)
    out, r0 = [], 0
    for k in range(n_mb):
        n = base + (1 if k < extra else 0)
        out.append((r0, n))
        r0 += n
    return out


@dataclass
class PipelineStats:
    steps: int = 0
    sent_x_bytes: int = 0
    sent_id_bytes: int = 0


class Pipeline:
    """Runs the schedule for one rank. ``stage`` provides embed/forward/pick/new_x/new_ids; ``gx`` and
    ``gt`` are the process groups for activations and ids (both containing every rank)."""

    def __init__(self, stage, rank: int, world: int, n_seq: int, n_mb: int, gx=None, gt=None):
        import torch.distributed as dist
        self.dist, self.stage, self.rank, self.world = dist, stage, rank, world
        self.mbs = micro_batches(n_seq, n_mb)
        self.gx, self.gt = gx, gt
        self.stats = PipelineStats()
        self._pending = []           # last rank: (work, ids) of picks sent to rank 0
        self._local = None           # one rank only: the last step's picks

    def _send_x(self, x):
        self.dist.send(x, self.rank + 1, group=self.gx)
        self.stats.sent_x_bytes += x.numel() * x.element_size()

    def _recv_x(self, x):
        self.dist.recv(x, self.rank - 1, group=self.gx)
        self.stage.sync()

    def _recv_ids(self, n):
        ids = self.stage.new_ids(n)
        self.dist.recv(ids, self.world - 1, group=self.gt)
        return ids

    def step(self, ids_by_mb, pick: bool):
        """One token of every sequence. Rank 0 passes ids_by_mb (one id tensor per micro-batch), or None
        to feed the previous step's picks, each received from the last rank just before its micro-batch
        needs it. The last rank, when pick, sends each micro-batch's picks to rank 0 as soon as they are
        made (non-blocking; see finish). Returns the ids rank 0 fed, the picks on the last rank."""
        fed, out = [], []
        last = self.rank == self.world - 1
        for k, (r0, n) in enumerate(self.mbs):
            x = self.stage.new_x(n)
            if self.rank == 0:
                if ids_by_mb is not None:
                    ids = ids_by_mb[k]
                elif self.world > 1:
                    ids = self._recv_ids(n)
                else:
                    ids = self._local[k]
                fed.append(ids)
                self.stage.embed(ids, x)
            else:
                self._recv_x(x)
            self.stage.forward(x, r0, n)
            if not last:
                self._send_x(x)
            elif pick:
                ids = self.stage.new_ids(n)
                self.stage.pick(x, r0, n, ids)
                out.append(ids)
                if self.world > 1:
                    # to rank 0 right away, on its own group; nothing waits for it before finish(), so a
                    # device-ordered stream never holds a receive of activations behind this send
                    self._pending.append((self.dist.isend(ids, 0, group=self.gt), ids))
                    self.stats.sent_id_bytes += ids.numel() * ids.element_size()
        if last and pick:
            self._local = out
        self.stats.steps += 1
        return fed if self.rank == 0 else out

    def drain(self):
        """Rank 0: the picks of the last step (not fed to any step)."""
        if self.world == 1:
            return self._local
        return [self._recv_ids(n) for (r0, n) in self.mbs]

    def finish(self):
        """Last rank: wait for the picks sent to rank 0."""
        for w, _ in self._pending:
            w.wait()
        self._pending = []

    def decode(self, prompts, n_gen: int):
        """Greedy decode: prompts [n_seq][P] (numpy, used on rank 0). Returns ids [n_seq][n_gen] on rank 0
        (None elsewhere): the prompt goes through in P lockstep steps, the last of which picks out[:, 0];
        each generated id but the last is fed back."""
        ctx = getattr(self.stage, "context", None)
        with (ctx() if ctx else contextlib.nullcontext()):
            return self._decode(prompts, n_gen)

    def _decode(self, prompts, n_gen: int):
        P = int(prompts.shape[1]) if self.rank == 0 else None
        if self.world > 1:
            import torch
            t = torch.tensor([P if P is not None else 0], dtype=torch.int64, device=self.stage.device)
            self.dist.broadcast(t, 0, group=self.gx)
            P = int(t.item())
        gen = []
        for i in range(P + n_gen - 1):
            pick = i >= P - 1
            ids = None
            if self.rank == 0 and i < P:
                ids = [self._ids_from(prompts[r0:r0 + n, i]) for (r0, n) in self.mbs]
            got = self.step(ids, pick)
            if self.rank == 0 and i >= P:
                gen.append(got)          # the ids fed at step i are the picks of step i - 1 (on the device)
        if self.rank == 0:
            gen.append(self.drain())
        if self.rank == self.world - 1:
            self.finish()
        if self.rank != 0:
            return None
        gen = [np.concatenate([g.cpu().numpy() for g in got]) for got in gen]   # copies on the stage's stream
        return np.stack(gen, axis=1).astype(np.int32)

    def _ids_from(self, arr):
        import torch
        t = self.stage.new_ids(len(arr))
        t.copy_(torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int32)))
        return t
