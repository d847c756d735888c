"""Layer pipeline across GPUs for batched greedy decode (one process per GPU, torch.distributed).

The reference splits a model into stages by layer range (``xj_net.h:93-111``: a|r|b) and drives them
with ``xj_pipeline_eval`` over TCP. Here every rank holds one stage: a batch of ``n_seq`` sequences
over its layer range (``xj_cuda_batch_new_range``), the first stage also embeds and the last also
owns the LM head and the greedy pick. Per decode step and micro-batch of rows:

    rank 0:      ids -> embed -> layers [0, l1)   -> send x ------------\\
    rank i:      recv x -> layers [l0, l1) -> send x                    | activations: group gx
    rank N-1:    recv x -> layers [l0, L) -> head + argmax -> send ids -/  ids: group gt (to rank 0)

Micro-batches keep the stages busy at the same time: while the last stage works on micro-batch k of
step s, the first stage already runs micro-batch k+1. Activations ([rows][n_embd] fp32) and ids go
over NCCL (NVLink) on GPUs and over gloo in the CPU tests; they travel on two process groups, one per
direction, so a send in one direction never waits behind a receive in the other on one communicator.
On GPUs every stage call and every transfer is queued on the stage's own CUDA stream (the library's
stream, wrapped as a torch external stream), so they are ordered on the device and the host never waits
inside a step. The last rank sends each micro-batch's picks as soon as they are made, without waiting
for the send; rank 0 receives them only when the next step's micro-batch needs them. So the first
stage starts micro-batch k of the next step as soon as that micro-batch's picks exist, and no stream
ever holds a receive of activations behind a send of ids (which could deadlock the two communicators).
KV caches and recurrent state stay on the rank that owns the layer.

The per-stage compute is behind a small interface (``embed``, ``forward``, ``pick``) so that the
schedule itself is tested on CPU with a stand-in stage (tests/test_pipeline_cpu.py).
"""
from __future__ import annotations

import contextlib
import ctypes
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


class CudaStage:
    """One rank's stage on its GPU: xj_cuda_batch over layers [l0, l1) (head on the last rank)."""

    def __init__(self, model, l0: int, l1: int, has_head: bool, n_seq: int, n_ctx: int, device):
        import torch
        from . import xjcuda
        self.xc, self.torch, self.device = xjcuda, torch, device
        lib = xjcuda.lib()
        vp, ip, cp, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t
        for name, res, args in [
            ("xj_cuda_batch_new_range", vp, [vp, ip, ip, ctypes.c_bool, ip, ip, cp, sz]),
            ("xj_cuda_batch_embed_rows", ip, [vp, vp, vp, ip, cp, sz]),
            ("xj_cuda_batch_forward_rows", ip, [vp, vp, ip, ip, cp, sz]),
            ("xj_cuda_batch_pick_rows", ip, [vp, vp, ip, ip, vp, cp, sz]),
            ("xj_cuda_batch_stream", vp, [vp]),
            ("xj_cuda_batch_set_async", ip, [vp, ip]),
            ("xj_cuda_batch_sync", ip, [vp, cp, sz]),
        ]:
            getattr(lib, name).restype = res
            getattr(lib, name).argtypes = args
        self.lib = lib
        e = ctypes.create_string_buffer(512)
        self.p = lib.xj_cuda_batch_new_range(model.ptr, l0, l1, has_head, n_seq, n_ctx, e, 512)
        if not self.p:
            raise xjcuda.XjError(e.value.decode(errors="replace"))
        self.E = model.n_embd
        self.has_head = has_head
        self.first = l0 == 0
        # queue-only stage calls, ordered with the caller's transfers on the library's stream
        lib.xj_cuda_batch_set_async(self.p, 1)
        self.stream = torch.cuda.ExternalStream(lib.xj_cuda_batch_stream(self.p), device=device)

    def _check(self, rc, e):
        if rc:
            raise self.xc.XjError(e.value.decode(errors="replace"))

    def new_x(self, nrows):
        return self.torch.empty((nrows, self.E), dtype=self.torch.float32, device=self.device)

    def context(self):
        """Everything of a step runs on the stage's stream (transfers included)."""
        return self.torch.cuda.stream(self.stream)

    def sync(self):
        # transfers run on the stage's own stream (see context), so a received tensor is ordered before
        # the kernels that read it without waiting on the host
        pass

    def host_sync(self):
        e = ctypes.create_string_buffer(512)
        self._check(self.lib.xj_cuda_batch_sync(self.p, e, 512), e)

    def new_ids(self, nrows):
        return self.torch.empty(nrows, dtype=self.torch.int32, device=self.device)

    def embed(self, ids, x):
        e = ctypes.create_string_buffer(512)
        self._check(self.lib.xj_cuda_batch_embed_rows(self.p, ids.data_ptr(), x.data_ptr(), ids.numel(), e, 512), e)

    def forward(self, x, row0, nrows):
        e = ctypes.create_string_buffer(512)
        self._check(self.lib.xj_cuda_batch_forward_rows(self.p, x.data_ptr(), row0, nrows, e, 512), e)

    def pick(self, x, row0, nrows, ids):
        e = ctypes.create_string_buffer(512)
        self._check(self.lib.xj_cuda_batch_pick_rows(self.p, x.data_ptr(), row0, nrows, ids.data_ptr(), e, 512), e)

    def close(self):
        if self.p:
            self.xc.lib().xj_cuda_batch_free(self.p)
            self.p = None


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
