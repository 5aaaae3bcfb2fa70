"""Audio I/O edges on the GPU (mirrors of unblend/audio.py and the WAV fast path).

At 1000x realtime and more, decoding, resampling and clipping on the host take
longer than the separation itself. These keep them on the device:

* :func:`read_pcm16_wav` parses a plain 16-bit PCM WAV header on the host (the
  same acceptance rules as ``Separator._read_pcm16_wav``, unblend/api.py:1080-1112),
  ships the 2-byte samples once through pinned memory and converts them to
  planar float32 (``int16 / 32768``) with the channel conversion of
  :func:`convert_audio_channels` in one kernel; other formats return None.
* :func:`convert_audio` (unblend/audio.py:51-67): channel conversion, then
  ``torchaudio.functional.resample``'s default band-limited interpolation
  (Hann-windowed sinc, 6 zero crossings, roll-off 0.99, rates reduced by their
  gcd) as a polyphase CUDA kernel.
* :func:`prevent_clip` (unblend/audio.py:70-90): rescale / clamp / tanh.
* :func:`export_pcm16_wav` (unblend/api.py:94-148 ``export_stem`` for WAV):
  the clipping guard and the float -> 16-bit PCM conversion in one kernel,
  then a canonical 44-byte WAV header on the host.
"""

from __future__ import annotations

import math
import struct
import wave
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .apply import ValidationError

CLIP_MODES = {"rescale": 1, "clamp": 2, "tanh": 3}


def _check_channels(cin: int, cout: int) -> None:
    if not (cin == cout or cout == 1 or cin == 1 or cin > cout):
        raise ValidationError("The audio file has less channels than requested but is not mono.")
    if cin > 8 or cout > 8:
        raise ValidationError("at most 8 audio channels are supported")


def read_pcm16_wav(path: Path | str, channels: int = 2, device: torch.device | str = "cuda"
                   ) -> tuple[torch.Tensor, int] | None:
    """Decode a 16-bit PCM WAV file to ``[channels, samples]`` float32 on ``device``.

    :return: ``(waveform, sample_rate)``, or None when the file is not readable
        uncompressed 16-bit PCM (the caller then falls back to a general decoder).
    """
    try:
        with wave.open(str(path), "rb") as w:
            if w.getsampwidth() != 2 or w.getcomptype() != "NONE":
                return None
            frames, cin, rate = w.getnframes(), w.getnchannels(), w.getframerate()
            raw = w.readframes(frames)
    except (wave.Error, EOFError, OSError, ValueError):
        return None
    if cin <= 0 or rate <= 0 or not raw or len(raw) % (2 * cin) != 0:
        return None
    _check_channels(cin, channels)
    n = len(raw) // (2 * cin)
    host = torch.empty(len(raw) // 2, dtype=torch.int16, pin_memory=True)
    host.numpy()[:] = np.frombuffer(raw, dtype="<i2")
    dev = torch.device(device)
    src = host.to(dev, non_blocking=True)
    out = torch.empty(channels, n, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.call("unblend_pcm16_to_f32", src.data_ptr(), cin, n, out.data_ptr(), channels)
    return out, rate


def convert_audio_channels(wav: torch.Tensor, channels: int = 2) -> torch.Tensor:
    """``[..., C, L]`` CUDA audio to ``channels`` channels (unblend/audio.py:14-48)."""
    *shape, cin, length = wav.shape
    _check_channels(cin, channels)
    if cin == channels:
        return wav
    x = wav.float().contiguous().view(-1, cin, length)
    y = torch.empty(x.shape[0], channels, length, device=wav.device, dtype=torch.float32)
    for b in range(x.shape[0]):
        _lib.call("unblend_convert_channels", x[b].data_ptr(), cin, length, y[b].data_ptr(), channels)
    return y.view(*shape, channels, length)


def sinc_resample_kernel(orig: int, new: int, lowpass_filter_width: int = 6, rolloff: float = 0.99
                         ) -> tuple[torch.Tensor, int, int, int]:
    """Polyphase filter bank of band-limited interpolation from ``orig`` to ``new`` Hz.

    The rates are reduced by their gcd to ``lin -> lout``; the cut-off is
    ``rolloff * min(lin, lout)`` (in reduced-rate units); each of the ``lout``
    output phases p gets a Hann-windowed sinc (``lowpass_filter_width`` zero
    crossings each side) sampled at input offsets ``-width .. width + lin - 1``,
    shifted by ``-p / lout``. Evaluated in float32, as the reference's resampler
    does for float32 audio (a float64 evaluation differs from it by ~3e-5 of
    full scale): ``[lout, 2 width + lin]`` with ``(lin, lout, width)``.
    """
    g = math.gcd(orig, new)
    lin, lout = orig // g, new // g
    cutoff = min(lin, lout) * rolloff
    width = math.ceil(lowpass_filter_width * lin / cutoff)
    offs = torch.arange(-width, width + lin, dtype=torch.float32)[None, :] / lin
    t = torch.arange(0, -lout, -1, dtype=torch.float32)[:, None] / lout + offs
    t = (t * cutoff).clamp(-lowpass_filter_width, lowpass_filter_width)
    window = torch.cos(t * math.pi / lowpass_filter_width / 2) ** 2
    t = t * math.pi
    sinc = torch.where(t == 0, torch.ones_like(t), torch.sin(t) / t)
    return (sinc * window * (cutoff / lin)).contiguous(), lin, lout, width


_KERNELS: dict = {}


def resample(wav: torch.Tensor, orig: int, new: int) -> torch.Tensor:
    """``[..., L]`` CUDA audio resampled from ``orig`` to ``new`` Hz; output length ``ceil(new * L / orig)``."""
    if orig == new:
        return wav
    if orig <= 0 or new <= 0:
        raise ValidationError("sample rates must be positive")
    key = (orig, new, str(wav.device))
    if key not in _KERNELS:
        kern, lin, lout, width = sinc_resample_kernel(orig, new)
        _KERNELS[key] = (kern.to(wav.device), lin, lout, width)
    kern, lin, lout, width = _KERNELS[key]
    *shape, length = wav.shape
    x = wav.float().contiguous().view(-1, length)
    out_len = math.ceil(lout * length / lin)
    y = torch.empty(x.shape[0], out_len, device=wav.device, dtype=torch.float32)
    _lib.call("unblend_resample", x.data_ptr(), x.shape[0], length, kern.data_ptr(), kern.shape[1], lin, lout, width,
              y.data_ptr(), out_len)
    return y.view(*shape, out_len)


def convert_audio(wav: torch.Tensor, from_samplerate: int, to_samplerate: int, channels: int) -> torch.Tensor:
    """Channel conversion then resampling (unblend/audio.py:51-67), on the device."""
    return resample(convert_audio_channels(wav, channels), from_samplerate, to_samplerate)


def prevent_clip(audio: torch.Tensor, mode: str | None = "rescale") -> torch.Tensor:
    """Clipping guard before export (unblend/audio.py:70-90): "rescale", "clamp", "tanh" or None."""
    if not mode:
        return audio
    if mode not in CLIP_MODES:
        raise ValidationError(f"Invalid clip mode '{mode}'. Must be one of: 'rescale', 'clamp', 'tanh', or None")
    x = audio.float().contiguous()
    y = torch.empty_like(x)
    bits = None
    if mode == "rescale":
        bits = torch.zeros(1, device=x.device, dtype=torch.int32)
        _lib.call("unblend_max_abs", x.data_ptr(), x.numel(), bits.data_ptr())
    _lib.call("unblend_prevent_clip", x.data_ptr(), y.data_ptr(), x.numel(), CLIP_MODES[mode], _lib.ptr(bits))
    return y


def _pcm16_wav_header(channels: int, sample_rate: int, frames: int) -> bytes:
    """Canonical 44-byte RIFF/WAVE header of 16-bit PCM."""
    data = frames * channels * 2
    if data > 0xFFFFFFFF - 36:
        raise ValidationError("stem too long for a RIFF WAV file (4 GiB data limit)")
    return (b"RIFF" + struct.pack("<I", 36 + data) + b"WAVE"
            + b"fmt " + struct.pack("<IHHIIHH", 16, 1, channels, sample_rate, sample_rate * channels * 2,
                                    channels * 2, 16)
            + b"data" + struct.pack("<I", data))


def export_pcm16_wav(audio: torch.Tensor, sample_rate: int, path: Path | str | None = None,
                     format: str = "wav", clip: str | None = "rescale") -> Path | bytes:
    """One stem ``[channels, samples]`` to a 16-bit PCM WAV file or bytes (unblend/api.py:94-148 export_stem).

    The clipping guard (``prevent_clip``) and the float -> 16-bit conversion run
    in one kernel on the device, so only the 2-byte interleaved samples cross to
    the host. A ``path`` without a suffix gets ``.{format}``; only ``wav`` is
    encoded here (other containers go through a general-purpose encoder).

    :return: the written path when ``path`` is given, else the file's bytes.
    """
    if clip and clip not in CLIP_MODES:
        raise ValidationError(f"Invalid clip mode '{clip}'. Must be one of: 'rescale', 'clamp', 'tanh', or None")
    file_path = None
    if path is not None:
        file_path = Path(path)
        if not file_path.suffix:
            file_path = file_path.with_suffix(f".{format}")
        fmt = file_path.suffix[1:].lower()
    else:
        fmt = format.lower()
    if fmt != "wav":
        raise ValidationError(f"only 16-bit PCM WAV is encoded on the device, got '{fmt}'")
    if audio.dim() != 2:
        raise ValidationError("expected one stem as [channels, samples]")
    if sample_rate <= 0:
        raise ValidationError("sample rate must be positive")
    channels, frames = audio.shape
    header = _pcm16_wav_header(channels, sample_rate, frames)
    dev = audio.device if audio.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    x = audio.to(dev, dtype=torch.float32, non_blocking=True).contiguous()
    host = torch.empty(frames * channels, dtype=torch.int16, pin_memory=True)
    if frames:
        with torch.cuda.device(dev):
            bits = None
            if clip == "rescale":
                bits = torch.zeros(1, device=dev, dtype=torch.int32)
                _lib.call("unblend_max_abs", x.data_ptr(), x.numel(), bits.data_ptr())
            pcm = torch.empty(frames * channels, device=dev, dtype=torch.int16)
            _lib.call("unblend_encode_pcm16", x.data_ptr(), channels, frames, CLIP_MODES.get(clip, 0) if clip else 0,
                      _lib.ptr(bits), pcm.data_ptr())
            host.copy_(pcm, non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
    body = host.numpy().tobytes()
    if file_path is None:
        return header + body
    file_path.parent.mkdir(exist_ok=True, parents=True)
    with open(file_path, "wb") as f:
        f.write(header)
        f.write(body)
    return file_path


__all__ = ["read_pcm16_wav", "convert_audio_channels", "convert_audio", "resample", "sinc_resample_kernel",
           "prevent_clip", "export_pcm16_wav"]
