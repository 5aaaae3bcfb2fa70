"""Golden fixture of the audio I/O edges, made with the reference itself.

Run from the repository root where the reference is mounted at /root/reference::

    python tests/golden/make_audio_golden.py [/root/reference]

Imports the reference (``torchcodec`` stubbed, as in make_golden.py) and
records, on short synthetic clips: ``unblend.audio.convert_audio`` (its
``torchaudio.functional.resample`` call, torchaudio 2.11.0 here) for several
rate pairs and channel counts, ``Separator._read_pcm16_wav`` on a 3-channel
16-bit WAV written here, and ``prevent_clip`` in its three modes. Saves
``tests/golden/audio_io.pt``.
"""

from __future__ import annotations

import io
import os
import sys
import tempfile
import wave

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from make_golden import import_reference, reference_path  # noqa: E402
from unblend_b200.synth import synth_track  # noqa: E402


def main(ref_path: str) -> None:
    unblend = import_reference(ref_path)
    import unblend.api
    import unblend.audio

    res = {"resample": [], "clip": {}}
    for sr_in, sr_out, ch, seed in ((48000, 44100, 2, 40), (44100, 32000, 2, 41), (22050, 44100, 2, 42),
                                    (96000, 44100, 1, 43)):
        x = synth_track(0.25, seed, samplerate=sr_in)
        y = unblend.audio.convert_audio(x, sr_in, sr_out, ch)
        res["resample"].append({"from": sr_in, "to": sr_out, "channels": ch, "x": x, "y": y.clone()})
    rng = np.random.default_rng(7)
    pcm = rng.integers(-32768, 32767, size=(5000, 3), dtype=np.int16)
    buf = io.BytesIO()
    with wave.open(buf, "wb") as w:
        w.setnchannels(3)
        w.setsampwidth(2)
        w.setframerate(44100)
        w.writeframes(pcm.tobytes())
    wav_bytes = buf.getvalue()
    with tempfile.NamedTemporaryFile(suffix=".wav", delete=False) as f:
        f.write(wav_bytes)
        path = f.name
    try:
        decoded, rate = unblend.api.Separator._read_pcm16_wav(path)
    finally:
        os.unlink(path)
    res["wav"] = {"bytes": wav_bytes, "rate": rate, "decoded": decoded.clone(),
                  "stereo": unblend.audio.convert_audio_channels(decoded, 2).clone(),
                  "mono": unblend.audio.convert_audio_channels(decoded, 1).clone()}
    x = synth_track(0.25, 44) * 3.0
    res["clip"]["x"] = x
    for mode in ("rescale", "clamp", "tanh"):
        res["clip"][mode] = unblend.audio.prevent_clip(x, mode).clone()
    torch.save(res, os.path.join(HERE, "audio_io.pt"))
    print("wrote", os.path.join(HERE, "audio_io.pt"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else reference_path())
