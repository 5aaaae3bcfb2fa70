"""Host logic of the segment engine (no GPU): the full / tail pools of several
mixes, batch runs, OOM halving and its propagation rules, the residency
budget and the planned chunk counts. Modelled on the reference's own backoff
tests (tests/test_apply.py:468-640), with a fake batch runner in place of the
device forward."""

from __future__ import annotations

import pytest
import torch

from unblend_b200 import _lib
from unblend_b200.apply import (_drain, _gpu_accum_bytes_needed, _looks_like_cuda_oom, _planned_counts, _pools,
                                _runs, _split_weight_host)


def test_pools_pool_tails_across_mixes():
    full, tail = _pools([5, 3, 8], 4)
    assert full == [(0, k) for k in range(4)] + [(2, k) for k in range(8)]
    assert tail == [(0, 4), (1, 0), (1, 1), (1, 2)]
    # Every chunk appears exactly once, and a mix's chunks ascend within each pool.
    assert sorted(full + tail) == sorted((m, k) for m, n in enumerate([5, 3, 8]) for k in range(n))
    f1, t1 = _pools([7], 32)
    assert f1 == [] and t1 == [(0, k) for k in range(7)]


def test_runs_group_consecutive_chunks_of_a_mix():
    items = [(0, 4), (1, 0), (1, 1), (1, 2), (3, 9)]
    assert _runs(items) == [(0, 4, 1, 0), (1, 0, 3, 1), (3, 9, 1, 4)]
    assert _runs([(2, 3), (2, 5)]) == [(2, 3, 1, 0), (2, 5, 1, 1)]


class _FakeRunner:
    """Runs batches of items; raises an OOM-shaped error above ``fits`` items."""

    def __init__(self, fits: int, message: str = "CUDA out of memory (fake, for backoff test)") -> None:
        self.fits = fits
        self.message = message
        self.ooms = 0
        self.seen: list = []
        self.emitted: list = []

    def run(self, batch: list) -> list:
        if len(batch) > self.fits:
            self.ooms += 1
            raise RuntimeError(self.message)
        self.seen += batch
        return [len(batch)]

    def drain(self, pool: list, state: dict | None, cbs: int, fixed: bool = False) -> None:
        size = (lambda: max(1, int(state["chunk_batch_size"]))) if state is not None else (lambda: cbs)
        _drain(pool, self.run, size, state, fixed, lambda: None, self.emitted.append)


def test_oom_backoff_halves_until_fit_and_runs_every_item_once():
    pool = list(range(23))
    r = _FakeRunner(fits=2)
    state = {"chunk_batch_size": 8}
    r.drain(pool, state, 8)
    assert state["chunk_batch_size"] == 2
    assert r.ooms == 2
    assert r.seen == pool
    assert sum(p[0] for p in r.emitted) == len(pool)


def test_oom_without_backoff_state_propagates():
    r = _FakeRunner(fits=1)
    with pytest.raises(RuntimeError, match="out of memory"):
        r.drain(list(range(9)), None, 4)


def test_oom_at_batch_one_raises_with_state_floored():
    r = _FakeRunner(fits=0)
    state = {"chunk_batch_size": 4}
    with pytest.raises(RuntimeError, match="out of memory"):
        r.drain(list(range(9)), state, 4)
    assert state["chunk_batch_size"] == 1


def test_non_oom_error_propagates_with_state_untouched():
    r = _FakeRunner(fits=0, message="illegal instruction (not memory)")
    state = {"chunk_batch_size": 4}
    with pytest.raises(RuntimeError, match="illegal"):
        r.drain(list(range(9)), state, 4)
    assert state["chunk_batch_size"] == 4


def test_fixed_batch_shape_blocks_backoff():
    r = _FakeRunner(fits=1)
    state = {"chunk_batch_size": 4}
    with pytest.raises(RuntimeError, match="out of memory"):
        r.drain(list(range(9)), state, 4, fixed=True)
    assert state["chunk_batch_size"] == 4


def test_library_oom_text_is_recognised():
    with pytest.raises(RuntimeError) as info:
        _lib.check("unblend_conv2d_tc", 2)  # cudaErrorMemoryAllocation
    assert _looks_like_cuda_oom(info.value)
    with pytest.raises(RuntimeError) as info:
        _lib.check("unblend_conv2d_tc", 700)
    assert not _looks_like_cuda_oom(info.value)
    assert _looks_like_cuda_oom(torch.cuda.OutOfMemoryError("x"))


def test_residency_budget_and_planned_counts():
    # Track, [S, C, L] accumulator and weight sum in fp32 (unblend/apply.py:387-400).
    assert _gpu_accum_bytes_needed(1, 4, 2, 1000) == (2 * 5 * 1000 + 1000) * 4

    class M:
        samplerate = 100
        max_allowed_segment = 1.0
        sources = ["a", "b"]

    rows = [torch.zeros(2, 250), torch.zeros(2, 75)]
    assert _planned_counts(M, rows, 0, 0.25, None) == [4, 1]
    # Shifted rounds separate L + max_shift - offset samples (unblend/apply.py:954-960).
    assert _planned_counts(M, rows, 2, 0.25, [[0, 50], [10, 0]]) == [
        -(-300 // 75) + -(-290 // 75), -(-75 // 75) + -(-125 // 75)]


@pytest.mark.parametrize("power", [1.0, 2.0, 3.5])
def test_host_split_weight_is_the_powered_triangle(power):
    w = _split_weight_host(7, power)
    tri = torch.tensor([1, 2, 3, 4, 3, 2, 1], dtype=torch.float32)
    assert torch.allclose(w, (tri / 4) ** power)


def test_free_memory_query_is_reused_and_corrected(monkeypatch):
    """The residency budget re-queries cudaMemGetInfo at most once a second per device and
    corrects a cached answer by what this process reserved since."""
    from unblend_b200 import apply as eng

    state = {"queries": 0, "reserved": 1000, "now": 50.0}

    def fake_info(idx):
        state["queries"] += 1
        return 10_000, 80_000

    monkeypatch.setattr(eng.torch.cuda, "mem_get_info", fake_info)
    monkeypatch.setattr(eng.torch.cuda, "memory_reserved", lambda idx=None: state["reserved"])
    monkeypatch.setattr(eng.time, "monotonic", lambda: state["now"])
    monkeypatch.setattr(eng, "_FREE_QUERY", {})
    dev = torch.device("cuda", 3)
    assert eng._free_device_bytes(dev) == 10_000 and state["queries"] == 1
    state["reserved"] = 4000  # this process reserved 3000 more bytes
    state["now"] += 0.5
    assert eng._free_device_bytes(dev) == 7_000 and state["queries"] == 1
    state["now"] += 0.6  # the cached answer is older than a second: query again
    assert eng._free_device_bytes(dev) == 10_000 and state["queries"] == 2


def test_tail_padding_rule_for_graph_replayed_models():
    """Fixed-shape models are zero-padded up to the batch, except that models whose graphs
    leave smaller batches to eager launches (``_eager_tails``) keep tails below 7/8 of it."""
    from types import SimpleNamespace

    from unblend_b200.apply import _PooledRun

    def rows(model, n, cbs=16):
        run = _PooledRun(model, [], torch.device("cpu"), 8, 4, cbs, 1.0, None, None, True)
        return run._rows(n)

    plain = SimpleNamespace(_fixed_batch_shape=False)
    fixed = SimpleNamespace(_fixed_batch_shape=True)
    eager = SimpleNamespace(_fixed_batch_shape=True, _eager_tails=True)
    assert [rows(plain, n) for n in (2, 14, 16)] == [2, 14, 16]
    assert [rows(fixed, n) for n in (2, 14, 16)] == [16, 16, 16]
    assert [rows(eager, n) for n in (2, 13, 14, 16)] == [2, 13, 16, 16]
    assert rows(eager, 31, 32) == 32 and rows(eager, 27, 32) == 27
