"""Segment engine control paths on the GPU against the oracle's overlap-add.

Cross-mix tail pooling (unblend/apply.py:1102-1155), the transition power of
the cross-fade (unblend/apply.py:426-430), host accumulation when the
accumulators do not fit the device (unblend/apply.py:1058-1085), OOM halving
(unblend/apply.py:1264-1306), zero-padded tails for fixed-shape models
(unblend/apply.py:1189-1196) and the progress payloads. The models are small
CUDA stand-ins (pointwise and position-dependent) so that a dropped, doubled
or misplaced chunk shows in the output.
"""

from __future__ import annotations

import pytest
import torch

import unblend_b200.apply as eng
from conftest import rel_err
from oracle.apply_oracle import apply_unshifted

pytestmark = pytest.mark.gpu


class _Positional(torch.nn.Module):
    """[B, C, T] -> [B, 3, C, T]: x, 2x and a running sum along T (position-dependent)."""

    sources = ["a", "b", "c"]
    samplerate = 1000
    audio_channels = 2
    max_allowed_segment = 0.9

    def __init__(self, fits: int | None = None) -> None:
        super().__init__()
        self.fits = fits
        self.batches: list[int] = []
        self.ooms = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fits is not None and x.shape[0] > self.fits:
            self.ooms += 1
            raise RuntimeError("CUDA out of memory (stand-in model, for the backoff test)")
        self.batches.append(x.shape[0])
        return torch.stack([x, 2 * x, 1e-2 * x.cumsum(-1)], 1)


class _Pointwise(_Positional):
    """x, 2x and x*x: per-sample, so any batch size gives bit-identical chunk outputs."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fits is not None and x.shape[0] > self.fits:
            self.ooms += 1
            raise RuntimeError("CUDA out of memory (stand-in model, for the backoff test)")
        self.batches.append(x.shape[0])
        return torch.stack([x, 2 * x, x * x], 1)


def _oracle(model, track: torch.Tensor, power: float = 1.0, overlap: float = 0.25) -> torch.Tensor:
    seg = int(round(model.samplerate * model.max_allowed_segment))
    fwd = lambda b: torch.stack([b, 2 * b, 1e-2 * b.cumsum(-1)], 1)  # noqa: E731
    return apply_unshifted(fwd, track.cpu()[None], 3, seg, overlap, 4, transition_power=power)[0]


def _tracks():
    g = torch.Generator().manual_seed(7)
    return [torch.randn(2, n, generator=g).cuda() for n in (4000, 2301, 901, 5555)]


def test_pooled_tails_match_per_track_overlap_add():
    m = _Positional()
    tracks = _tracks()
    outs = eng.apply_model_multi(m, tracks, chunk_batch_size=4)
    for t, o in zip(tracks, outs):
        assert o.shape == (3, 2, t.shape[-1])
        assert rel_err(o, _oracle(m, t)) < 1e-6
    # Chunks per track at stride 675: 6, 4, 2, 9 -> full batches 4, 4, 4, 8 then pooled tails 2+0+2+1 = 5.
    assert m.batches == [4, 4, 4, 4, 4, 1]


@pytest.mark.parametrize("power", [2.0, 3.0])
def test_transition_power(power):
    m = _Positional()
    t = _tracks()[0]
    out = eng.apply_model(m, t, chunk_batch_size=3, transition_power=power)
    assert rel_err(out, _oracle(m, t, power)) < 1e-6


def test_host_accumulation_matches_device_accumulation(monkeypatch):
    m = _Positional()
    tracks = [t.cpu() for t in _tracks()]
    resident = eng.apply_model_multi(m, tracks, chunk_batch_size=4, transition_power=2.0)
    monkeypatch.setattr(eng, "_gpu_accum_budget_bytes", lambda device, reserve=None: 0)
    host = eng.apply_model_multi(m, tracks, chunk_batch_size=4, transition_power=2.0)
    for a, b, t in zip(host, resident, tracks):
        assert a.device.type == "cpu" and b.device.type == "cpu"
        # Host accumulation adds chunk by chunk, the device kernel position by position: fp32 rounding only.
        assert rel_err(a, b) < 1e-5
        assert rel_err(a, _oracle(m, t, 2.0)) < 1e-5
    # A track on the device, shifted rounds, host accumulators.
    t = tracks[0].cuda()
    host_s = eng.apply_model(m, t, chunk_batch_size=4, shifts=2, shift_offsets=[13, 400])
    monkeypatch.undo()
    res_s = eng.apply_model(m, t, chunk_batch_size=4, shifts=2, shift_offsets=[13, 400])
    assert rel_err(host_s, res_s) < 1e-5


def test_oom_backoff_halves_and_output_is_exact():
    clean = eng.apply_model(_Pointwise(), _tracks()[3], chunk_batch_size=8)
    m = _Pointwise(fits=2)
    state = {"chunk_batch_size": 8}
    out = eng.apply_model(m, _tracks()[3], chunk_batch_size=8, oom_backoff_state=state)
    assert state["chunk_batch_size"] == 2 and m.ooms == 2
    assert torch.equal(out, clean)
    with pytest.raises(RuntimeError, match="out of memory"):
        eng.apply_model(_Positional(fits=1), _tracks()[3], chunk_batch_size=4)


def test_fixed_shape_models_get_zero_padded_pooled_tails():
    m = _Positional()
    m._fixed_batch_shape = True
    tracks = _tracks()
    outs = eng.apply_model_multi(m, tracks, chunk_batch_size=4)
    assert set(m.batches) == {4}
    for t, o in zip(tracks, outs):
        assert rel_err(o, _oracle(m, t)) < 1e-6


def test_progress_payloads_cover_every_chunk():
    events = []
    tracks = _tracks()
    eng.apply_model_multi(_Positional(), tracks, chunk_batch_size=4, shifts=1,
                          progress_callback=lambda e, d: events.append((e, dict(d))))
    assert events[0][0] == "processing_start" and events[-1][0] == "processing_complete"
    chunks = [d for e, d in events if e == "chunk_complete"]
    total = events[0][1]["total_chunks"]
    assert len(chunks) == total == sum(events[0][1]["input_total_chunks"])
    assert [d["completed_chunks"] for d in chunks] == list(range(1, total + 1))
    for i, n in enumerate(events[0][1]["input_total_chunks"]):
        mine = [d["input_completed_chunks"] for d in chunks if d["input_index"] == i]
        assert mine == list(range(1, n + 1))
