"""Sharding one track's segments across ranks (no GPU): the shard plan, and the
overlap-strip exchange + owned-range gather on world_size 2 and 3 gloo ranks
against the single-process overlap-add of the oracle."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.apply_oracle import apply_unshifted, center_trim, padded_chunk, split_weight
from unblend_b200.apply import ValidationError
from unblend_b200.distributed import gather_owned, shard_plan, stitch


@pytest.mark.parametrize("length,segment,stride,world", [
    (700, 100, 75, 3), (1000, 100, 75, 8), (10, 100, 75, 4), (343980 * 3, 343980, 257985, 2),
    (7_938_000, 343980, 257985, 8), (151, 40, 10, 4)])
def test_shard_plan_partitions_the_track(length, segment, stride, world):
    plan = shard_plan(length, segment, stride, world)
    offsets = [o for s in plan for o in s.offsets]
    assert offsets == list(range(0, length, stride))
    counts = [len(s.offsets) for s in plan]
    assert max(counts) - min(counts) <= 1
    owned = [(s.own_lo, s.own_hi) for s in plan if s.offsets]
    assert owned[0][0] == 0 and owned[-1][1] == length
    assert all(a[1] == b[0] for a, b in zip(owned, owned[1:]))
    for s in plan:
        if s.offsets:
            assert s.lo == s.own_lo == s.offsets[0] and s.hi == min(length, s.offsets[-1] + segment)


def test_shard_plan_rejects_bad_arguments():
    with pytest.raises(ValidationError):
        shard_plan(100, 0, 10, 2)


def _model(batch: torch.Tensor) -> torch.Tensor:
    """A pointwise two-stem model: (x, x^2 - 0.1)."""
    return torch.stack([batch, batch * batch - 0.1], dim=1)


def _local_accumulate(mix: torch.Tensor, offsets, segment: int):
    """This rank's weighted chunk sums over the whole track, as the oracle computes them."""
    C, L = mix.shape
    w = split_weight(segment)
    acc = torch.zeros(2 * C, L)
    sum_w = torch.zeros(L)
    for o in offsets:
        chunk = padded_chunk(mix[None], o, segment, segment)
        y = center_trim(_model(chunk), min(segment, L - o))[0]  # [2, C, len]
        n = y.shape[-1]
        acc[:, o:o + n] += (y * w[:n]).reshape(2 * C, n)
        sum_w[o:o + n] += w[:n]
    return acc, sum_w


def _worker(rank: int, world: int, port: int, length: int, segment: int, stride: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        mix = torch.randn(2, length)
        plan = shard_plan(length, segment, stride, world)
        acc, sum_w = _local_accumulate(mix, plan[rank].offsets, segment)
        own = stitch(acc, sum_w, plan, rank)
        full = gather_owned(own, plan, rank, length)
        ref = apply_unshifted(_model, mix[None], 2, segment, overlap=1 - stride / segment)[0].reshape(4, length)
        me = plan[rank]
        q.put((rank, float((full - ref).abs().max()),
               float((own - ref[:, me.own_lo:me.own_hi]).abs().max()) if own.numel() else 0.0))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,length,segment,stride", [(2, 1000, 120, 90), (3, 2000, 160, 120), (3, 150, 100, 75)])
def test_stitched_shards_equal_single_process(world, length, segment, stride):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, length, segment, stride, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, full_err, own_err in results:
        assert full_err < 1e-5 and own_err < 1e-5, (rank, full_err, own_err)
