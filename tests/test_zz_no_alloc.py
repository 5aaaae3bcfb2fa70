"""The allocation-free statistics entry point, ``unblend_mean_std_noalloc``.

Callers that cannot allocate device memory while they run (a real-time audio
thread, where cudaMalloc may stall on a device-wide synchronisation, or a host
whose memory manager owns every device allocation) use this variant: it keeps
its accumulator in a fixed static device array instead of a caller buffer.
Its results must equal those of ``unblend_mean_std``, which takes the buffer
from the caller, call after call (the shared array keeps the previous call's
contents, so each call must clear what it uses).

This file is collected last on purpose, so that a run stopping at the first
failure has already run every other test.
"""

from __future__ import annotations

import pytest
import torch

from unblend_b200 import _lib

pytestmark = pytest.mark.gpu


def _with_buffer(x: torch.Tensor) -> torch.Tensor:
    batch, n = x.shape
    work = torch.empty(2 * batch, device=x.device, dtype=torch.float64)
    out = torch.empty(2 * batch, device=x.device)
    _lib.call("unblend_mean_std", x.data_ptr(), work.data_ptr(), out.data_ptr(), batch, n)
    return out


def _no_alloc(x: torch.Tensor) -> torch.Tensor:
    batch, n = x.shape
    out = torch.empty(2 * batch, device=x.device)
    _lib.call("unblend_mean_std_noalloc", x.data_ptr(), out.data_ptr(), batch, n)
    return out


def test_no_alloc_matches_buffered_entry_point_twice():
    g = torch.Generator(device="cuda").manual_seed(11)
    # Two calls in a row; the second uses fewer batch items, so stale sums from
    # the first call sit in the shared array and must not leak in.
    for batch, n, shift in ((7, 300_001, 3.0), (3, 12_345, -1.5)):
        x = torch.randn(batch, n, device="cuda", generator=g) * 2 + shift
        got = _no_alloc(x)
        want = _with_buffer(x)
        torch.cuda.synchronize()
        assert torch.allclose(got, want, rtol=1e-6, atol=1e-7), (got, want)
        var, mean = torch.var_mean(x.double(), dim=1)
        assert torch.allclose(got[0::2].double(), mean, rtol=1e-5, atol=1e-6)
        assert torch.allclose(got[1::2].double(), var.sqrt(), rtol=1e-5)


def test_no_alloc_rejects_batches_beyond_capacity():
    x = torch.zeros(_lib.NOALLOC_MAX_BATCH + 1, 2, device="cuda")
    out = torch.empty(2 * x.shape[0], device="cuda")
    with pytest.raises(RuntimeError, match="fixed built-in capacity"):
        _lib.call("unblend_mean_std_noalloc", x.data_ptr(), out.data_ptr(), x.shape[0], 2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_no_alloc_on_a_second_device():
    # The array's address is resolved per device: device 1 after device 0, one stream each.
    for dev in (0, 1):
        with torch.cuda.device(dev):
            g = torch.Generator(device=f"cuda:{dev}").manual_seed(5 + dev)
            x = torch.randn(5, 40_001, device=f"cuda:{dev}", generator=g) + dev
            got = _no_alloc(x)
            want = _with_buffer(x)
            torch.cuda.synchronize(dev)
            assert torch.allclose(got, want, rtol=1e-6, atol=1e-7), (dev, got, want)
