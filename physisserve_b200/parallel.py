"""Multi-GPU placement of the attention-prep path: stream sharding and the 2-stage handoff.

The prep kernels have no collective: every stream (its chunk, its KV ring) is independent,
so streams are sharded over GPUs (``shard_streams``), the way PhysisServe's pool placement
puts whole streams on disjoint GPU sets (physisserve/engine/strategies/placement.py:186-263,
MappedLayout 237-263).  The pipelined configuration splits the DiT's blocks into stages
(StageEqual, engine/strategies/stage_equal.py:21-57): a stage runs its blocks for a chunk's
denoising step, then hands the hidden state [tokens, C] to the next stage with a
point-to-point send/recv, as the reference's transport does with batch_isend_irecv
(engine/transport.py:116-150).  Only the hidden state crosses GPUs; each stage keeps the KV
history of its own blocks, so no KV ever moves (model_runner.py:44-69).
"""
from __future__ import annotations

import datetime
import math
from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist


def shard_streams(n_streams: int, rank: int, world: int) -> list[int]:
    """Streams owned by ``rank``: stream i runs on GPU i mod world (disjoint and complete)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_streams, world))


def stage_blocks(stage: int, stages: int, num_blocks: int) -> range:
    """Contiguous equal split of the blocks over stages (StageEqual's layout)."""
    if not 0 <= stage < stages or stages > num_blocks:
        raise ValueError(f"stage {stage} of {stages} for {num_blocks} blocks")
    base, extra = divmod(num_blocks, stages)
    start = stage * base + min(stage, extra)
    return range(start, start + base + (1 if stage < extra else 0))


@dataclass(frozen=True)
class PipelineLayout:
    """Ranks grouped into pipelines of ``stages`` consecutive ranks; streams sharded over pipelines."""

    world: int
    stages: int

    def __post_init__(self):
        if self.stages < 1 or self.world % self.stages:
            raise ValueError(f"{self.world} ranks do not split into pipelines of {self.stages} stages")

    @property
    def pipelines(self) -> int:
        return self.world // self.stages

    def stage_of(self, rank: int) -> int:
        return rank % self.stages

    def pipeline_of(self, rank: int) -> int:
        return rank // self.stages

    def peer(self, rank: int, offset: int) -> int:
        """The rank ``offset`` stages after ``rank`` in its pipeline (wrapping around)."""
        p = self.pipeline_of(rank)
        return p * self.stages + (self.stage_of(rank) + offset) % self.stages

    def streams(self, n_streams: int, rank: int) -> list[int]:
        return shard_streams(n_streams, self.pipeline_of(rank), self.pipelines)


def pipeline_tick(layout: PipelineLayout, rank: int, hidden: torch.Tensor,
                  run_blocks: Callable[[torch.Tensor], torch.Tensor], group=None) -> torch.Tensor:
    """One tick of a ring pipeline with one micro-batch per stage.

    Every stage runs its blocks on the micro-batch it holds, then all stages exchange in one
    grouped send/recv: the result goes to the next stage and the previous stage's result
    arrives in ``hidden`` (the last stage feeds stage 0, which starts that micro-batch's next
    denoising step).  Grouping the send with the receive makes the exchange deadlock-free for
    any number of stages.  Returns ``hidden`` holding the received micro-batch.
    """
    out = run_blocks(hidden)
    if layout.stages == 1:
        hidden.copy_(out)
        return hidden
    _exchange(send=(out, layout.peer(rank, 1)), recv=(hidden, layout.peer(rank, -1)), group=group)
    return hidden


def _exchange(send=None, recv=None, group=None):
    ops = []
    if send is not None:
        ops.append(dist.P2POp(dist.isend, send[0].contiguous(), send[1], group=group))
    if recv is not None:
        ops.append(dist.P2POp(dist.irecv, recv[0], recv[1], group=group))
    for work in dist.batch_isend_irecv(ops):
        work.wait()


# --------------------------------------------------------------------------------------
# Asynchronous stage handoff
# --------------------------------------------------------------------------------------
class _Handle:
    """One backend work handle shared by every consumer of a posted batch: the backend is
    waited on at most once (gloo receive handles allow one wait), while completion for
    buffer retention is polled separately (a stream wait does not mean the copy is done)."""

    __slots__ = ("work", "waited")

    def __init__(self, work):
        self.work, self.waited = work, False

    def wait(self):
        if not self.waited:
            self.work.wait()
            self.waited = True

    def done(self) -> bool:
        return bool(self.work.is_completed())


class Pending:
    """The tensors of one received item.  ``wait()`` returns them once they hold the data:
    for NCCL it makes the current CUDA stream wait (the host goes on), for gloo it blocks.
    The consumer waits when it runs, not when the transfer is posted (transport.py:54-67,
    model_runner.py:184)."""

    __slots__ = ("tensors", "handles")

    def __init__(self, tensors, handles=()):
        self.tensors, self.handles = tensors, tuple(handles)

    def wait(self):
        for h in self.handles:
            h.wait()
        self.handles = ()
        return self.tensors


def _dtype_groups(spec):
    """Indices of ``spec`` entries grouped by dtype, in first-appearance order."""
    groups = {}
    for i, (_, dtype) in enumerate(spec):
        groups.setdefault(dtype, []).append(i)
    return list(groups.items())


class Transport:
    """Ordered point-to-point transfers between the ranks of a stage pipeline, posted
    asynchronously (the contract of the reference's ``Distributed`` transport,
    engine/transport.py:84-156).

    ``transfer(items)`` takes ``(tag, src, dst, spec, tensors)`` items in the same order on
    every rank; ``spec`` is ``[(shape, dtype), ...]`` and ``tensors`` is needed on the source
    only.  All of a call's sends and receives go out as one ``batch_isend_irecv``; the result
    maps the tags this rank receives (or keeps, when src == dst) to ``Pending``.

    Same-dtype tensors of an item travel as ONE message: the sender copies them into one
    contiguous packet, the receiver receives into one allocation and hands out views of it
    (a hidden state and a latent are one message, not two).  Receive allocations are fresh
    per transfer, never pooled, because callers keep received tensors.  Every posted packet
    and receive buffer stays referenced until the backend reports the operation complete,
    so callers may drop or overwrite their own tensors as soon as ``transfer`` returns.
    """

    def __init__(self, device, group=None):
        self.device, self.group = torch.device(device), group
        self.rank = dist.get_rank(group)
        self.inflight = []  # (handles, tensors) kept until every handle reports completion

    def _peer(self, rank: int) -> int:
        return dist.get_global_rank(self.group, rank) if self.group is not None else rank

    def _receive_packets(self, spec):
        """(views in spec order, packet buffers) for one received item."""
        views = [None] * len(spec)
        packets = []
        for dtype, idx in _dtype_groups(spec):
            sizes = [math.prod(spec[i][0]) for i in idx]
            packet = torch.empty(sum(sizes), dtype=dtype, device=self.device)
            offset = 0
            for i, n in zip(idx, sizes):
                views[i] = packet.narrow(0, offset, n).view(spec[i][0])
                offset += n
            packets.append(packet)
        return tuple(views), packets

    def _send_packets(self, spec, tensors):
        packets = []
        for dtype, idx in _dtype_groups(spec):
            parts = [tensors[i] for i in idx]
            for i in idx:
                if tuple(tensors[i].shape) != tuple(spec[i][0]) or tensors[i].dtype != dtype:
                    raise ValueError(f"tensor {i} is {tuple(tensors[i].shape)} {tensors[i].dtype}, spec says "
                                     f"{tuple(spec[i][0])} {dtype}")
            if len(parts) == 1:
                packets.append(parts[0].reshape(-1).contiguous())
            else:
                packets.append(torch.cat([t.reshape(-1) for t in parts]))
        return packets

    def transfer(self, items):
        self.inflight = [entry for entry in self.inflight if not all(h.done() for h in entry[0])]
        ops, kept, received, result = [], [], {}, {}
        for tag, src, dst, spec, tensors in items:
            if src == dst:
                if src == self.rank:
                    result[tag] = Pending(tensors)
                continue
            if dst == self.rank:
                views, packets = self._receive_packets(spec)
                received[tag] = (views, len(ops), len(ops) + len(packets))
                ops += [dist.P2POp(dist.irecv, b, self._peer(src), group=self.group) for b in packets]
                kept += packets
            elif src == self.rank:
                packets = self._send_packets(spec, tensors)
                ops += [dist.P2POp(dist.isend, b, self._peer(dst), group=self.group) for b in packets]
                kept += packets
        if not ops:
            return result
        handles = [_Handle(w) for w in dist.batch_isend_irecv(ops)]
        self.inflight.append((handles, tuple(kept)))
        # Gloo gives one handle per operation; coalesced NCCL may give one for the whole batch,
        # which every receiver then shares.
        per_op = len(handles) == len(ops)
        for tag, (views, first, last) in received.items():
            result[tag] = Pending(views, handles[first:last] if per_op else handles)
        return result

    def flush(self):
        """Wait for everything still in flight (the end of a request)."""
        for handles, _ in self.inflight:
            for h in handles:
                h.wait()
        self.inflight = []


def init_process_group(backend: str, timeout_s: float = 60.0, device_id=None):
    """Process group from the torchrun environment with a short timeout, so a rank that
    fails makes its peers' next collective end with an error instead of waiting."""
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kwargs["device_id"] = device_id
    dist.init_process_group(backend, **kwargs)
    return dist.get_rank(), dist.get_world_size()


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank value (device timings are reported as the max over ranks)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(values: Sequence[float], device=None) -> list[float]:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t.tolist()]
