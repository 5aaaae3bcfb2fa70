"""Time the oracle port against the reference's own CPU path on the same sample.

Test infrastructure, not product code. ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` time the oracle (``kind: "port"``), because the reference
is a Python package that is not installed beside the repository on the GPU
host. This script, run where a reference checkout exists
(``$UNBLEND_REFERENCE``, else ``reference`` beside this repository), times both
on the same bounded sample with the same thread count: the registry
``htdemucs`` (seed-0 random init, identical weights in both) through
``apply_model`` over a synthetic stereo track, fp32, overlap 0.25, batch 32.
It prints one JSON line with both throughputs and the largest difference
between the two outputs relative to the reference output's RMS.

    python oracle/time_against_reference.py [seconds]
"""

from __future__ import annotations

import json
import os
import sys
import time
import types

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle.apply_oracle import apply_model as oracle_apply  # noqa: E402
from oracle.htdemucs_oracle import htdemucs_forward, segment_length  # noqa: E402
from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track  # noqa: E402


def reference_path() -> str:
    path = os.environ.get("UNBLEND_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
    if not os.path.isdir(os.path.join(path, "unblend")):
        raise SystemExit(f"reference checkout not found at {path}; set UNBLEND_REFERENCE")
    return path


def import_reference(path: str):
    """The reference ``unblend`` package with its audio-file codec (``torchcodec``, absent here) stubbed."""
    for name in ("torchcodec", "torchcodec.decoders", "torchcodec.encoders"):
        mod = types.ModuleType(name)
        mod.AudioDecoder = object
        mod.AudioEncoder = object
        sys.modules.setdefault(name, mod)
    sys.path.insert(0, path)
    import unblend.apply
    import unblend.htdemucs

    return unblend


def main(seconds: float) -> None:
    unblend = import_reference(reference_path())
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = htdemucs_config("htdemucs")
    torch.manual_seed(0)
    ref_model = unblend.htdemucs.HTDemucs(**cfg).eval()
    sd = htdemucs_state_dict(cfg, 0)
    for k, v in ref_model.state_dict().items():
        assert torch.equal(v, sd[k]), f"weight {k} differs"
    mix = synth_track(seconds, 1)[None]
    seg = segment_length(cfg)
    with torch.inference_mode():
        fwd = lambda b: htdemucs_forward(sd, b, cfg)  # noqa: E731
        fwd(mix[..., :seg])  # warm-up segment, as bench.py's cpu_baseline
        t0 = time.perf_counter()
        port = oracle_apply(fwd, mix, 4, seg, cfg["samplerate"], overlap=0.25, chunk_batch_size=32)
        t_port = time.perf_counter() - t0
        ref_model(mix[..., :seg])
        t0 = time.perf_counter()
        ref = unblend.apply.apply_model(ref_model, mix, device="cpu", shifts=0, overlap=0.25, chunk_batch_size=32)
        t_ref = time.perf_counter() - t0
    diff = float((port.double() - ref.double()).abs().max() / ref.double().pow(2).mean().sqrt())
    print(json.dumps({"sample": f"registry htdemucs (seed 0), {seconds:g} s synthetic track (seed 1), fp32, "
                                f"overlap 0.25, batch 32", "threads": threads,
                      "port_audio_s_per_s": round(seconds / t_port, 3),
                      "reference_audio_s_per_s": round(seconds / t_ref, 3),
                      "port_over_reference": round(t_ref / t_port, 3), "max_abs_diff_over_rms": diff}))


if __name__ == "__main__":
    main(float(sys.argv[1]) if len(sys.argv) > 1 else 30.0)
