"""The SCNet oracle and weight generator against the reference's own outputs.

Fixtures come from ``tests/golden/make_golden.py <reference> scnet`` (the
reference ``SCNet`` / ``SCNetMasked`` built by ``build_scnet`` under
``torch.manual_seed``, fp32 CPU forward, unblend/scnet.py:746-895).
"""

from __future__ import annotations

import hashlib

import pytest
import torch

from conftest import golden, rel_err
from oracle.apply_oracle import apply_model
from oracle.scnet_oracle import band_splits, scnet_forward, stft_padding
from unblend_b200.synth import scnet_state_dict, synth_track

TOL = 1e-5


def _digest(sd: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("fname", ["scnet_small_reduced.pt", "scnet_plain_reduced.pt", "scnet_small_full.pt",
                                   "scnet_xl_full.pt"])
def test_weights_match_reference_init(fname):
    g = golden(fname)
    assert _digest(scnet_state_dict(g["config"], g["seed"])) == g["weights_digest"]


@pytest.mark.parametrize("fname", ["scnet_small_reduced.pt", "scnet_plain_reduced.pt"])
def test_oracle_reduced_forward(fname):
    g = golden(fname)
    out = scnet_forward(scnet_state_dict(g["config"], g["seed"]), g["mix"], g["config"])
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < TOL


@pytest.mark.parametrize("fname", ["scnet_small_full.pt", "scnet_xl_full.pt"])
def test_oracle_registry_forward(fname):
    g = golden(fname)
    out = scnet_forward(scnet_state_dict(g["config"], g["seed"]), g["mix"], g["config"])
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < TOL
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["sumsq"], rtol=1e-5)


def test_oracle_apply_model_two_segments():
    g = golden("scnet_apply.pt")
    cfg = g["config"]
    mix = synth_track(g["mix_seconds"], g["mix_seed"])[None]
    assert hashlib.sha256(mix.contiguous().numpy().tobytes()).hexdigest() == g["mix_digest"]
    sd = scnet_state_dict(cfg, g["seed"])
    out = apply_model(lambda b: scnet_forward(sd, b, cfg), mix, 4, cfg["segment_samples"], cfg["samplerate"],
                      overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"])
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < TOL
    wins = torch.stack([out[..., s:s + g["window"]] for s in g["windows"]])
    assert rel_err(wins, g["win_out"]) < TOL


def test_padding_and_band_split_rules():
    # An even frame count after the pad (unblend/scnet.py:543-572): 485100 samples -> 486400.
    assert stft_padding(485100, 1024) == 1300
    assert (485100 + stft_padding(485100, 1024)) // 1024 % 2 == 1
    assert stft_padding(2048, 1024) == 1024  # a whole extra hop even when already aligned
    cfg = {"band_SR": [0.175, 0.392, 0.433]}
    assert band_splits(2049, cfg) == [(0, 359), (359, 1162), (1162, 2049)]
