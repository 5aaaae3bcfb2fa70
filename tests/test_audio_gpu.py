"""GPU audio I/O edges against the reference's own outputs: 16-bit WAV decode
with channel conversion, windowed-sinc resampling, clipping guards."""

from __future__ import annotations

import os
import tempfile

import pytest
import torch

from conftest import golden
from unblend_b200.audio import convert_audio, prevent_clip, read_pcm16_wav

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("channels,key", [(3, "decoded"), (2, "stereo"), (1, "mono")])
def test_read_pcm16_wav(channels, key):
    w = golden("audio_io.pt")["wav"]
    with tempfile.NamedTemporaryFile(suffix=".wav", delete=False) as f:
        f.write(w["bytes"])
        path = f.name
    try:
        out, rate = read_pcm16_wav(path, channels=channels, device="cuda")
    finally:
        os.unlink(path)
    assert rate == w["rate"]
    assert (out.cpu() - w[key]).abs().max() <= (1e-7 if key == "mono" else 0.0)
    assert read_pcm16_wav(__file__, device="cuda") is None  # not a WAV: caller falls back


def test_convert_audio_matches_reference():
    for case in golden("audio_io.pt")["resample"]:
        y = convert_audio(case["x"].cuda(), case["from"], case["to"], case["channels"]).cpu()
        assert y.shape == case["y"].shape
        assert (y - case["y"]).abs().max() < 2e-6, (case["from"], case["to"])


@pytest.mark.parametrize("mode", ["rescale", "clamp", "tanh"])
def test_prevent_clip_matches_reference(mode):
    c = golden("audio_io.pt")["clip"]
    y = prevent_clip(c["x"].cuda(), mode).cpu()
    assert (y - c[mode]).abs().max() < 1e-6
