"""The BS-RoFormer CPU oracle against the reference's own outputs (golden fixtures)."""

from __future__ import annotations

import hashlib

import pytest
import torch

from conftest import golden, rel_err
from oracle.apply_oracle import apply_unshifted
from oracle.roformer_oracle import bsroformer_forward
from unblend_b200.synth import bsroformer_state_dict

TOL = 1e-5


def _digest(sd: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("fname", ["bsroformer_small.pt", "bsroformer_full.pt"])
def test_roformer_weights_match_reference_init(fname):
    g = golden(fname)
    assert _digest(bsroformer_state_dict(g["config"], g["seed"])) == g["weights_digest"]


def test_roformer_oracle_small_forward():
    g = golden("bsroformer_small.pt")
    out = bsroformer_forward(bsroformer_state_dict(g["config"], g["seed"]), g["mix"], g["config"])
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < TOL


def test_roformer_oracle_full_forward():
    g = golden("bsroformer_full.pt")
    out = bsroformer_forward(bsroformer_state_dict(g["config"], g["seed"]), g["mix"], g["config"])
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < TOL
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["sumsq"], rtol=1e-5)


def test_roformer_oracle_apply_with_complement():
    g = golden("bsroformer_apply.pt")
    sd = bsroformer_state_dict(g["config"], g["seed"])
    fwd = lambda b: bsroformer_forward(sd, b, g["config"], complement=True)  # noqa: E731
    out = apply_unshifted(fwd, g["mix"], 2, g["segment_samples"], g["overlap"], g["chunk_batch_size"])
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < TOL
    # complement: the two stems sum back to the mixture
    assert torch.allclose(out.sum(dim=1), g["mix"], atol=1e-5)


def test_melband_oracle_matches_reference_fixture():
    """The Mel-Band restatement (band layout, gather, per-transformer norms, scatter-average) equals the
    reference's own outputs on the reduced model and the kim registry configuration."""
    from oracle.roformer_oracle import melband_forward, mel_supports
    from unblend_b200.synth import mel_band_layout, melband_state_dict

    g = golden("melband_small.pt")
    cfg = g["config"]
    idx, _, per_bin = mel_band_layout(44100, cfg["stft_n_fft"], cfg["num_bands"], True)
    assert torch.equal(idx, g["freq_indices"]) and torch.equal(per_bin, g["num_bands_per_freq"])
    sup = mel_supports(44100, cfg["stft_n_fft"], cfg["num_bands"])
    assert torch.equal(sup.sum(dim=0), g["num_bands_per_freq"])
    out = melband_forward(melband_state_dict(cfg, g["seed"]), g["mix"], cfg)
    assert rel_err(out, g["out"]) < 1e-5
    k = golden("melband_kim.pt")
    out = melband_forward(melband_state_dict(k["config"], k["seed"]), k["mix"], k["config"], complement=True,
                          match_length=True)
    assert rel_err(out[..., :: k["decimate"]], k["out"]) < 1e-5
