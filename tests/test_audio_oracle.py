"""The audio I/O oracle against the reference's own outputs (no GPU), and the
host-side validation of the GPU audio API."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle.audio_oracle import convert_channels, encode_pcm16, pcm16_decode, prevent_clip, resample


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


def test_encode_pcm16_round_trips_reference_decode():
    """Decoding the reference's fixture WAV then encoding it gives its sample bytes back."""
    import io
    import wave

    w = golden("audio_io.pt")["wav"]
    with wave.open(io.BytesIO(w["bytes"]), "rb") as f:
        raw = f.readframes(f.getnframes())
    assert encode_pcm16(w["decoded"].numpy(), None).tobytes() == raw


def test_encode_pcm16_rounding_and_saturation():
    lsb = 1.0 / 32768
    x = np.array([[0.5 * lsb, 1.5 * lsb, 2.5 * lsb, -0.5 * lsb, -1.5 * lsb, 1.0, -1.0, 1.5, -7.0, np.nan]],
                 dtype=np.float32)
    assert encode_pcm16(x, None)[:, 0].tolist() == [0, 2, 2, 0, -2, 32767, -32768, 32767, -32768, 0]
    # rescale divides by max(1.01 max|x|, 1) first: the peak lands at 32768 / 1.01
    assert encode_pcm16(np.array([[2.0, -1.0]], dtype=np.float32), "rescale")[:, 0].tolist() == [32444, -16222]


def test_export_header_and_validation():
    import io
    import wave

    from unblend_b200.apply import ValidationError
    from unblend_b200.audio import _pcm16_wav_header, export_pcm16_wav

    pcm = np.arange(-6, 6, dtype="<i2")
    with wave.open(io.BytesIO(_pcm16_wav_header(3, 22050, 4) + pcm.tobytes()), "rb") as f:
        assert (f.getnchannels(), f.getsampwidth(), f.getframerate(), f.getnframes()) == (3, 2, 22050, 4)
        assert f.readframes(4) == pcm.tobytes()
    with pytest.raises(ValidationError):
        export_pcm16_wav(torch.zeros(2, 4), 44100, format="mp3")
    with pytest.raises(ValidationError):
        export_pcm16_wav(torch.zeros(2, 4), 44100, clip="wrap")
    with pytest.raises(ValidationError):
        export_pcm16_wav(torch.zeros(2, 4), 44100, path="stem.flac")
