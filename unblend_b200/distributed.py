"""One track's segments sharded across ranks, with the overlap-strip exchange.

The reference separates a track on one device (unblend/apply.py:1009-1333): the
segments at offsets ``range(0, L, stride)`` are independent forwards, coupled
only by the linear weighted overlap-add and the final ``out / sum_weight``.
Here the segment list is split into contiguous, count-balanced runs, one per
rank (one process per GPU). Each rank separates its run and overlap-adds it
into a local accumulator; the output positions are partitioned into disjoint
*owned* ranges, rank r owning from the first offset of its run to the first
offset of the next non-empty run. The only exchange is the strip of a rank's
accumulator (and weight sum) that falls into a neighbour's owned range: with
overlap 0.25 that is the last ``segment - stride`` samples, sent to the next
rank with point-to-point ``send``/``recv`` (NCCL over NVLink on GPUs, gloo on
CPU). Each rank then divides its owned range; ``gather`` optionally collects
the owned ranges into the full ``[S, C, L]`` result on every rank.

Because the overlap-add is a sum, the stitched result equals the one-device
result up to the order of fp32 additions in the strips.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from . import _lib
from .apply import ValidationError, _accumulate, _segment_plan, _to_host


@dataclass(frozen=True)
class Shard:
    """One rank's part of a track: its chunk offsets, the span they touch, the range it owns."""

    rank: int
    offsets: tuple[int, ...]
    lo: int        # first position touched by the rank's chunks (== own_lo when non-empty)
    hi: int        # one past the last position touched
    own_lo: int    # owned output positions [own_lo, own_hi)
    own_hi: int


def shard_plan(length: int, segment: int, stride: int, world: int) -> list[Shard]:
    """Split the segment offsets of a ``length``-sample track into ``world`` contiguous runs.

    Runs differ in size by at most one segment (the first ``n % world`` ranks
    take one more). Owned ranges partition ``[0, length)``; a rank with no
    segment owns an empty range.
    """
    if length <= 0 or segment <= 0 or stride <= 0 or world <= 0:
        raise ValidationError("length, segment, stride and world must be positive")
    offsets = list(range(0, length, stride))
    n = len(offsets)
    runs, start = [], 0
    for r in range(world):
        cnt = n // world + (1 if r < n % world else 0)
        runs.append(offsets[start:start + cnt])
        start += cnt
    firsts = [run[0] if run else None for run in runs]
    shards = []
    for r, run in enumerate(runs):
        if not run:
            shards.append(Shard(r, (), 0, 0, 0, 0))
            continue
        lo = run[0]
        hi = min(length, run[-1] + segment)
        nxt = next((f for f in firsts[r + 1:] if f is not None), length)
        shards.append(Shard(r, tuple(run), lo, hi, lo, nxt))
    return shards


def _intersect(a0: int, a1: int, b0: int, b1: int) -> tuple[int, int]:
    return max(a0, b0), min(a1, b1)


def stitch(acc: torch.Tensor, sum_w: torch.Tensor, plan: list[Shard], rank: int,
           group: Any = None) -> torch.Tensor:
    """Exchange overlap strips and return this rank's owned output ``acc / sum_w``.

    :param acc: ``[rows, L]`` weighted sums of this rank's chunks (full track length).
    :param sum_w: ``[L]`` weight sums of this rank's chunks.
    :param plan: :func:`shard_plan` for the track (same on every rank).
    :param rank: This rank's index in ``plan``.
    :param group: Process group (default group when None).
    :return: ``[rows, own_hi - own_lo]``.
    """
    me = plan[rank]
    rows = acc.shape[0]
    ops, recvs = [], []
    # Every rank walks the same (src, dst) list, so sends and receives pair up.
    for src in plan:
        for dst in plan:
            if src.rank == dst.rank or not src.offsets or not dst.offsets:
                continue
            p0, p1 = _intersect(src.lo, src.hi, dst.own_lo, dst.own_hi)
            if p1 <= p0:
                continue
            if src.rank == rank:
                strip = torch.cat([acc[:, p0:p1], sum_w[None, p0:p1]]).contiguous()
                ops.append(dist.P2POp(dist.isend, strip, dst.rank, group))
            elif dst.rank == rank:
                buf = torch.empty(rows + 1, p1 - p0, device=acc.device, dtype=acc.dtype)
                ops.append(dist.P2POp(dist.irecv, buf, src.rank, group))
                recvs.append((p0, p1, buf))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    own_acc = acc[:, me.own_lo:me.own_hi].clone()
    own_w = sum_w[me.own_lo:me.own_hi].clone()
    for p0, p1, buf in recvs:
        own_acc[:, p0 - me.own_lo:p1 - me.own_lo] += buf[:rows]
        own_w[p0 - me.own_lo:p1 - me.own_lo] += buf[rows]
    return own_acc / own_w


def gather_owned(own: torch.Tensor, plan: list[Shard], rank: int, length: int, group: Any = None) -> torch.Tensor:
    """All-gather every rank's owned range into the full ``[rows, L]`` output."""
    rows = own.shape[0]
    width = max(s.own_hi - s.own_lo for s in plan)
    padded = torch.zeros(rows, width, device=own.device, dtype=own.dtype)
    padded[:, :own.shape[1]] = own
    parts = [torch.empty_like(padded) for _ in plan]
    dist.all_gather(parts, padded, group=group)
    out = torch.empty(rows, length, device=own.device, dtype=own.dtype)
    for s, part in zip(plan, parts):
        out[:, s.own_lo:s.own_hi] = part[:, :s.own_hi - s.own_lo]
    return out


def apply_model_sharded(model: Any, mix: torch.Tensor, *, overlap: float = 0.25, chunk_batch_size: int = 1,
                        shifts: int = 0, shift_offsets: list[int] | None = None, group: Any = None,
                        gather: bool = True, device: Any = None,
                        timings: list | None = None) -> torch.Tensor | tuple[int, int, torch.Tensor]:
    """``apply_model`` for one ``[C, L]`` track with its segments sharded across the ranks of ``group``.

    Every rank calls this with the same track and arguments. The track is either
    on this rank's CUDA device, or on the host, in which case it is copied to
    ``device`` (default: the current CUDA device) and the result comes back in
    page-locked host memory, as ``apply_model`` does for a host input. With
    ``shifts`` the random offsets are drawn on rank 0 and broadcast, so every
    rank separates the same shifted rounds.

    :param timings: When a list, one dict of CUDA events per round is appended
        (``start``, ``separated``, ``exchanged``, ``gathered``), recorded on the
        current stream around this rank's separation, the strip exchange and the
        gather, for phase timing.
    :return: the full ``[S, C, L]`` result on every rank when ``gather`` (always
        with ``shifts``), else ``(own_lo, own_hi, out[S, C, own_hi - own_lo])`` for
        this rank. Ranks are those of the default process group when ``group`` is None.
    """
    if not 0.0 <= overlap < 1.0:
        raise ValidationError(f"overlap must be in [0, 1), got {overlap}")
    host_io = mix.device.type == "cpu"
    if host_io:
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise ValidationError("the B200 segment engine runs on CUDA devices only")
        mix = mix.to(dev, non_blocking=True)
    if mix.dim() != 2 or mix.device.type != "cuda":
        raise ValidationError("expected one [C, L] track on the host or on this rank's CUDA device")
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    # A collective first: NCCL's batched point-to-point calls need every rank to
    # have joined the communicator before the first one.
    dist.barrier(group=group)
    segment, stride = _segment_plan(model, overlap)
    S = len(model.sources)
    mix = mix.float().contiguous()
    C, L = mix.shape
    if not shifts:
        rounds = [(0, mix)]
        max_shift = 0
    else:
        max_shift = int(0.5 * model.samplerate)
        if shift_offsets is None:
            offs = torch.tensor([random.randint(0, max_shift) for _ in range(shifts)] if rank == 0 else [0] * shifts,
                                device=mix.device, dtype=torch.int64)
            dist.broadcast(offs, 0, group=group)
            shift_offsets = offs.tolist()
        padded = torch.nn.functional.pad(mix, (max_shift, max_shift))
        rounds = [(off, padded[:, off:L + max_shift].contiguous()) for off in shift_offsets]
    total = None

    def mark(ev: dict | None, name: str) -> None:
        if ev is not None:
            ev[name] = torch.cuda.Event(enable_timing=True)
            ev[name].record()

    for off, track in rounds:
        ev = {} if timings is not None else None
        mark(ev, "start")
        Lr = track.shape[-1]
        plan = shard_plan(Lr, segment, stride, world)
        me = plan[rank]
        acc = torch.empty(S * C, Lr, device=mix.device, dtype=torch.float32)
        sum_w = torch.empty(Lr, device=mix.device, dtype=torch.float32)
        _lib.call("unblend_zero_f32", acc.data_ptr(), acc.numel(), 1, 0)
        _lib.call("unblend_zero_f32", sum_w.data_ptr(), sum_w.numel(), 1, 0)
        if me.offsets:
            off_dev = torch.tensor(me.offsets, device=mix.device, dtype=torch.int64)
            _accumulate(model, track, S, segment, list(me.offsets), off_dev, chunk_batch_size, acc, sum_w)
        mark(ev, "separated")
        own = stitch(acc, sum_w, plan, rank, group)
        mark(ev, "exchanged")
        if ev is not None:
            timings.append(ev)
        if not gather and not shifts:
            own = own.view(S, C, me.own_hi - me.own_lo)
            return me.own_lo, me.own_hi, _to_host(own) if host_io else own
        full = gather_owned(own, plan, rank, Lr, group)
        mark(ev, "gathered")
        if shifts:
            full = full[:, max_shift - off:][:, :L]
        total = full if total is None else total.add_(full)
    out = (total / len(rounds)).view(S, C, L)
    return _to_host(out) if host_io else out


__all__ = ["Shard", "shard_plan", "stitch", "gather_owned", "apply_model_sharded"]
