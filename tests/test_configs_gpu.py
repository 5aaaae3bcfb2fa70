"""Parity at the configurations that are measured.

* The 10 s registry clip through ``apply_model`` at batch 1 (fp32), against the
  reference's own output (``htdemucs_cfg0.pt``) and, sample for sample over the
  whole output, the oracle run on the host.
* HTDemucs-6s with one shift round, vocals only, bf16, against the reference
  fixture (``htdemucs_6s_cfg2.pt``) and the oracle.
* The exact launch the headline bench times: the registry ``htdemucs`` on the
  chunks of the 180 s seed-1 track at 32 rows per forward, fp32 and bf16. Every
  row is compared over its full output with a batch-1 forward of the same row,
  and three rows with the oracle.
* BS-RoFormer (dim 512, depth 12) at 16 rows per forward in bf16, every row
  against batch 1, one row against the oracle.

Tolerances: fp32 max-abs error <= 1e-4 x output RMS; bf16 >= 40 dB SNR per stem.
"""

from __future__ import annotations

import hashlib
import math

import pytest
import torch

from conftest import golden, rel_err
from oracle.apply_oracle import apply_model as oracle_apply
from oracle.apply_oracle import padded_chunk
from oracle.htdemucs_oracle import htdemucs_forward, segment_length
from unblend_b200 import _lib
from unblend_b200.apply import apply_model
from unblend_b200.htdemucs import HTDemucsCuda
from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-4
BF16_MIN_SNR_DB = 40.0


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> list[float]:
    """Per-stem SNR in dB of ``out`` against ``ref`` ([B, S, C, L])."""
    o, r = out.double().cpu(), ref.double().cpu()
    res = []
    for s in range(r.shape[1]):
        den = (o[:, s] - r[:, s]).pow(2).sum()
        res.append(float(10 * math.log10(r[:, s].pow(2).sum() / den)) if den > 0 else float("inf"))
    return res


def _fixture(fname: str):
    g = golden(fname)
    mix = synth_track(g["mix_seconds"], g["mix_seed"])[None]
    assert hashlib.sha256(mix.contiguous().numpy().tobytes()).hexdigest() == g["mix_digest"]
    return g, mix, htdemucs_state_dict(g["config"], g["seed"])


def _windows(out: torch.Tensor, g: dict) -> torch.Tensor:
    return torch.stack([out[..., s:s + g["window"]] for s in g["windows"]])


def test_config0_ten_second_clip_fp32():
    g, mix, sd = _fixture("htdemucs_cfg0.pt")
    cfg = g["config"]
    m = HTDemucsCuda(cfg, sd, precision="fp32").cuda()
    out = apply_model(m, mix.cuda(), shifts=0, overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"]).cpu()
    assert out.shape == (1, 4, 2, mix.shape[-1])
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < FP32_TOL
    assert rel_err(_windows(out, g), g["win_out"]) < FP32_TOL
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["sumsq"], rtol=1e-4)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = oracle_apply(lambda b: htdemucs_forward(sd, b, cfg), mix, 4, segment_length(cfg), cfg["samplerate"],
                       overlap=g["overlap"], chunk_batch_size=1)
    assert rel_err(out, ref) < FP32_TOL
    assert _lib.error_flag() == 0


def test_config2_six_source_vocals_bf16_one_shift():
    g, mix, sd = _fixture("htdemucs_6s_cfg2.pt")
    cfg = g["config"]
    m = HTDemucsCuda(cfg, sd, precision="bf16").cuda().select_sources([g["stem"]])
    out = apply_model(m, mix.cuda(), shifts=1, overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"],
                      shift_offsets=g["offsets"]).cpu()
    assert out.shape == (1, 1, 2, mix.shape[-1])
    assert min(snr_db(out[..., :: g["decimate"]], g["out"])) >= BF16_MIN_SNR_DB
    assert min(snr_db(_windows(out, g).flatten(0, 1), g["win_out"].flatten(0, 1))) >= BF16_MIN_SNR_DB
    ref = oracle_apply(lambda b: htdemucs_forward(sd, b, cfg), mix, 6, segment_length(cfg), cfg["samplerate"],
                       shifts=1, overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"], offsets=g["offsets"])
    v = cfg["sources"].index(g["stem"])
    assert min(snr_db(out, ref[:, v:v + 1])) >= BF16_MIN_SNR_DB
    assert _lib.error_flag() == 0


def _headline_batch(seconds: float = 180.0, seed: int = 1) -> tuple[dict, torch.Tensor]:
    """The 31 centred chunks of the bench track plus chunk 0 again: 32 rows."""
    cfg = htdemucs_config("htdemucs")
    seg = segment_length(cfg)
    track = synth_track(seconds, seed)[None]
    offs = list(range(0, track.shape[-1], int(0.75 * seg)))
    assert len(offs) == 31
    rows = [padded_chunk(track, o, seg, seg) for o in offs + [0]]
    return cfg, torch.cat(rows)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_headline_launch_batch32_every_row(precision):
    cfg, batch = _headline_batch()
    sd = htdemucs_state_dict(cfg, 0)
    m = HTDemucsCuda(cfg, sd, precision=precision).cuda()
    xb = batch.cuda()
    full = m(xb)
    assert full.shape == (32, 4, 2, batch.shape[-1])
    # Batch independence over the full output of every row (the same kernels at batch 1).
    row_tol = 1e-5 if precision == "fp32" else 1e-3
    for i in range(32):
        one = m(xb[i:i + 1])
        assert rel_err(full[i:i + 1], one) < row_tol, i
    assert rel_err(full[31:32], full[0:1]) < row_tol
    # Three rows (first, middle, last chunk) against the oracle over their full outputs.
    for i in (0, 15, 30):
        ref = htdemucs_forward(sd, batch[i:i + 1], cfg)
        if precision == "fp32":
            assert rel_err(full[i:i + 1], ref) < FP32_TOL, i
        else:
            assert min(snr_db(full[i:i + 1], ref)) >= BF16_MIN_SNR_DB, i
    assert _lib.error_flag() == 0


def test_bsroformer_batch16_bf16():
    from oracle.roformer_oracle import bsroformer_forward
    from unblend_b200.roformer import BSRoformerCuda
    from unblend_b200.synth import bsroformer_config, bsroformer_state_dict

    cfg = bsroformer_config()
    sd = bsroformer_state_dict(cfg, 3)
    seg = 352800
    track = synth_track(120.0, 1)[None]  # the first 16 chunks of the measured 300 s track layout
    offs = list(range(0, track.shape[-1], int(0.75 * seg)))[:16]
    batch = torch.cat([padded_chunk(track, o, seg, seg) for o in offs])
    m = BSRoformerCuda(cfg, sd, precision="bf16").cuda()
    xb = batch.cuda()
    full = m(xb)
    assert full.shape[0] == 16
    for i in range(16):
        assert rel_err(full[i:i + 1], m(xb[i:i + 1])) < 1e-3, i
    ref = bsroformer_forward(sd, batch[7:8], cfg)
    assert min(snr_db(full[7:8], ref)) >= BF16_MIN_SNR_DB
    assert _lib.error_flag() == 0
