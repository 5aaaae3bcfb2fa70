"""GPU audio I/O edges against the reference's own outputs: 16-bit WAV decode
with channel conversion, windowed-sinc resampling, clipping guards."""

from __future__ import annotations

import os
import tempfile

import pytest
import torch

from conftest import golden
from oracle.audio_oracle import encode_pcm16
from unblend_b200.audio import convert_audio, export_pcm16_wav, prevent_clip, read_pcm16_wav

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


@pytest.mark.parametrize("clip", [None, "rescale", "clamp", "tanh"])
def test_export_pcm16_wav_matches_oracle(clip):
    import io
    import wave

    import numpy as np

    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 100_003, generator=g) * 0.6
    x[0, :8] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, 40000.0, -40000.0, 3.0]) / 32768  # ties, saturation
    data = export_pcm16_wav(x.cuda(), 44100, clip=clip)
    with wave.open(io.BytesIO(data), "rb") as f:
        assert (f.getnchannels(), f.getsampwidth(), f.getframerate(), f.getnframes()) == (2, 2, 44100, 100_003)
        got = np.frombuffer(f.readframes(f.getnframes()), dtype="<i2").reshape(-1, 2)
    want = encode_pcm16(x.numpy(), clip)
    diff = np.abs(got.astype(np.int32) - want.astype(np.int32)).max()
    assert diff <= (1 if clip == "tanh" else 0), diff  # tanh: CUDA's tanhf may differ from numpy by an ulp


def test_export_pcm16_wav_file_round_trip(tmp_path):
    w = golden("audio_io.pt")["wav"]
    out = export_pcm16_wav(w["decoded"].cuda(), w["rate"], path=tmp_path / "sub" / "stem", clip=None)
    assert out == tmp_path / "sub" / "stem.wav"
    import io
    import wave

    frames = []
    for blob in (out.read_bytes(), w["bytes"]):
        with wave.open(io.BytesIO(blob), "rb") as f:
            frames.append(f.readframes(f.getnframes()))
    assert frames[0] == frames[1]  # the reference fixture's samples, byte for byte
    back, rate = read_pcm16_wav(out, channels=3, device="cuda")
    assert rate == w["rate"] and torch.equal(back.cpu(), w["decoded"])
