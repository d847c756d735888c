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
KV caches and recurrent state stay on the rank that owns the layer.

The per-stage compute is behind a small interface (``embed``, ``forward``, ``pick``) so that the
schedule itself is tested on CPU with a stand-in stage (tests/test_pipeline_cpu.py).
"""
from __future__ import annotations

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

    def _check(self, rc, e):
        if rc:
            raise self.xc.XjError(e.value.decode(errors="replace"))

    def new_x(self, nrows):
        return self.torch.empty((nrows, self.E), dtype=self.torch.float32, device=self.device)

    def sync(self):
        # received tensors are written on torch's streams; the library's kernels run on the stage's own
        # stream, so the data must have landed before a pointer is handed over
        self.torch.cuda.synchronize(self.device)

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

    def _send_x(self, x):
        self.dist.send(x, self.rank + 1, group=self.gx)
        self.stats.sent_x_bytes += x.numel() * x.element_size()

    def _recv_x(self, x):
        self.dist.recv(x, self.rank - 1, group=self.gx)
        self.stage.sync()

    def step(self, ids_by_mb, pick: bool):
        """One token of every sequence. Rank 0 passes ids_by_mb (one id tensor per micro-batch) and,
        when pick, receives the next ids from the last rank; returns them (rank 0 and last rank)."""
        out = []
        last = self.rank == self.world - 1
        for k, (r0, n) in enumerate(self.mbs):
            x = self.stage.new_x(n)
            if self.rank == 0:
                self.stage.embed(ids_by_mb[k], x)
            else:
                self._recv_x(x)
            self.stage.forward(x, r0, n)
            if not last:
                self._send_x(x)
            elif pick:
                ids = self.stage.new_ids(n)
                self.stage.pick(x, r0, n, ids)
                out.append(ids)
        # the ids go back to rank 0 after every micro-batch of the step has been sent forward, on their
        # own group: rank 0 receives them in micro-batch order
        if pick and self.world > 1:
            if last:
                for ids in out:
                    self.dist.send(ids, 0, group=self.gt)
                    self.stats.sent_id_bytes += ids.numel() * ids.element_size()
            elif self.rank == 0:
                out = []
                for (r0, n) in self.mbs:
                    ids = self.stage.new_ids(n)
                    self.dist.recv(ids, self.world - 1, group=self.gt)
                    out.append(ids)
                self.stage.sync()
        self.stats.steps += 1
        return out

    def decode(self, prompts, n_gen: int):
        """Greedy decode: prompts [n_seq][P] (numpy, used on rank 0). Returns ids [n_seq][n_gen] on rank 0
        (None elsewhere): the prompt goes through in P lockstep steps, the last of which picks out[:, 0];
        each generated id but the last is fed back."""
        P = int(prompts.shape[1]) if self.rank == 0 else None
        if self.world > 1:
            import torch
            t = torch.tensor([P if P is not None else 0], dtype=torch.int64, device=self.stage.device)
            self.dist.broadcast(t, 0, group=self.gx)
            P = int(t.item())
        gen = []
        ids = None
        for i in range(P + n_gen - 1):
            pick = i >= P - 1
            if self.rank == 0:
                if i < P:
                    ids = [self._ids_from(prompts[r0:r0 + n, i]) for (r0, n) in self.mbs]
                # else: ids are the previous step's picks
            got = self.step(ids, pick)
            if pick and self.rank == 0:
                ids = got
                gen.append(np.concatenate([g.cpu().numpy() for g in got]))
        if self.rank != 0:
            return None
        return np.stack(gen, axis=1).astype(np.int32)

    def _ids_from(self, arr):
        import torch
        t = self.stage.new_ids(len(arr))
        t.copy_(torch.from_numpy(np.ascontiguousarray(arr, dtype=np.int32)))
        return t
