"""CPU restatement of the audio I/O edges (test infrastructure only).

* ``pcm16_decode``: unblend/api.py:1080-1112 (``int16 / 32768``, interleaved -> planar)
  followed by ``convert_audio_channels`` (unblend/audio.py:14-48).
* ``resample``: the reference calls ``torchaudio.functional.resample`` with its
  defaults (unblend/audio.py:67; torchaudio 2.11.0 in this image): band-limited
  interpolation with a Hann-windowed sinc of 6 zero crossings and roll-off 0.99
  on gcd-reduced rates. Restated here from that published method with numpy,
  the filter bank evaluated in float32 like the dependency does for float32
  audio and the polyphase sums in float64; pinned against torchaudio's own outputs
  (``tests/golden/audio_io.pt``, made by ``tests/golden/make_audio_golden.py``).
* ``prevent_clip``: unblend/audio.py:70-90.
* ``encode_pcm16``: unblend/api.py:94-148 (``export_stem``: ``prevent_clip``,
  then the encoder). The reference hands the clipped float stem to torchcodec's
  ``AudioEncoder`` (not installed in this image), whose 16-bit PCM WAV path
  converts samples with FFmpeg libswresample's float -> s16 rule: round
  ``x * 2**15`` to nearest, ties to even (``lrintf``), saturate to int16.
  Restated from that published rule; pinned by the round trip through the
  reference's own decoded fixture (decode -> encode gives the file's bytes back).
"""

from __future__ import annotations

import math

import numpy as np


def convert_channels(x: np.ndarray, cout: int) -> np.ndarray:
    cin = x.shape[0]
    if cin == cout:
        return x
    if cout == 1:
        return x.mean(axis=0, keepdims=True, dtype=np.float32).astype(np.float32)
    if cin == 1:
        return np.repeat(x, cout, axis=0)
    if cin > cout:
        return x[:cout]
    raise ValueError("fewer channels than requested and not mono")


def pcm16_decode(raw: bytes, cin: int, cout: int) -> np.ndarray:
    samples = np.frombuffer(raw, dtype="<i2").reshape(-1, cin)
    return convert_channels((samples.astype(np.float32) / np.float32(32768.0)).T.copy(), cout)


def filter_bank(orig: int, new: int, zeros: int = 6, rolloff: float = 0.99):
    g = math.gcd(orig, new)
    lin, lout = orig // g, new // g
    fc = min(lin, lout) * rolloff
    width = int(math.ceil(zeros * lin / fc))
    pos = np.arange(-width, width + lin).astype(np.float32) / np.float32(lin)
    shift = np.arange(0, -lout, -1).astype(np.float32) / np.float32(lout)
    t = np.clip((shift[:, None] + pos[None, :]) * np.float32(fc), -zeros, zeros).astype(np.float32)
    hann = np.cos(t * np.float32(math.pi) / np.float32(zeros) / np.float32(2)).astype(np.float32) ** 2
    arg = (t * np.float32(math.pi)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        s = np.where(arg == 0, np.float32(1), np.sin(arg) / arg).astype(np.float32)
    return (s * hann * np.float32(fc / lin)).astype(np.float32), lin, lout, width


def resample(x: np.ndarray, orig: int, new: int) -> np.ndarray:
    """``[C, L]`` -> ``[C, ceil(new L / orig)]``."""
    if orig == new:
        return x
    bank, lin, lout, width = filter_bank(orig, new)
    C, L = x.shape
    taps = bank.shape[1]
    xp = np.pad(x.astype(np.float64), ((0, 0), (width, width + lin)))
    frames = L // lin + 1
    idx = np.arange(frames)[:, None] * lin + np.arange(taps)[None, :]
    out = np.einsum("cft,pt->cfp", xp[:, idx], bank.astype(np.float64)).reshape(C, -1)
    return out[:, : int(math.ceil(lout * L / lin))].astype(np.float32)


def prevent_clip(x: np.ndarray, mode: str | None = "rescale") -> np.ndarray:
    if mode == "rescale":
        return (x / max(np.float32(1.01) * np.abs(x).max(), np.float32(1.0))).astype(np.float32)
    if mode == "clamp":
        return np.clip(x, -0.99, 0.99).astype(np.float32)
    if mode == "tanh":
        return np.tanh(x).astype(np.float32)
    return x


def encode_pcm16(x: np.ndarray, clip: str | None = "rescale") -> np.ndarray:
    """Planar float32 ``[C, L]`` -> interleaved int16 ``[L, C]``."""
    y = prevent_clip(np.asarray(x, dtype=np.float32), clip).astype(np.float32)
    q = np.rint(y * np.float32(32768.0))
    q = np.where(np.isnan(q), 0.0, np.clip(q, -32768, 32767))
    return q.astype(np.int16).T.copy()
