"""The audio I/O oracle against the reference's own outputs (no GPU), and the
host-side validation of the GPU audio API."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle.audio_oracle import convert_channels, pcm16_decode, prevent_clip, resample


def test_resample_matches_reference():
    g = golden("audio_io.pt")
    for case in g["resample"]:
        x = convert_channels(case["x"].numpy(), case["channels"])
        y = resample(x, case["from"], case["to"])
        assert y.shape == tuple(case["y"].shape)
        assert np.abs(y - case["y"].numpy()).max() < 2e-6


def test_pcm16_decode_and_channels_match_reference():
    w = golden("audio_io.pt")["wav"]
    import io
    import wave

    with wave.open(io.BytesIO(w["bytes"]), "rb") as f:
        raw = f.readframes(f.getnframes())
    assert np.array_equal(pcm16_decode(raw, 3, 3), w["decoded"].numpy())
    assert np.array_equal(pcm16_decode(raw, 3, 2), w["stereo"].numpy())
    assert np.allclose(pcm16_decode(raw, 3, 1), w["mono"].numpy(), rtol=0, atol=1e-7)


def test_prevent_clip_matches_reference():
    c = golden("audio_io.pt")["clip"]
    for mode in ("rescale", "clamp", "tanh"):
        assert np.abs(prevent_clip(c["x"].numpy(), mode) - c[mode].numpy()).max() < 1e-6


def test_audio_api_validation():
    from unblend_b200.apply import ValidationError
    from unblend_b200.audio import _check_channels, prevent_clip as gpu_clip, sinc_resample_kernel

    with pytest.raises(ValidationError):
        _check_channels(2, 3)
    with pytest.raises(ValidationError):
        gpu_clip(torch.zeros(4), "wrap")
    kern, lin, lout, width = sinc_resample_kernel(48000, 44100)
    assert (lin, lout) == (160, 147) and kern.shape == (147, 2 * width + 160)
    assert abs(float(kern.sum()) / lout - 1.0) < 1e-3  # each phase passes DC with unit gain
