"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference implementation (``HTDemucs.forward`` and ``apply_model`` on seeded
random-init weights and synthetic audio). These tests pin the oracle that the
GPU parity tests then compare against.
"""

from __future__ import annotations

import hashlib

import pytest
import torch

from conftest import golden, rel_err
from oracle.apply_oracle import apply_model, padded_chunk, split_weight
from oracle.htdemucs_oracle import htdemucs_forward, segment_length
from unblend_b200.synth import htdemucs_config, htdemucs_state_dict, synth_track

TOL = 1e-5  # max-abs error relative to output RMS (fp32, different op order)


def _digest(sd: dict) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def test_weights_match_reference_init_small():
    g = golden("htdemucs_small.pt")
    assert _digest(htdemucs_state_dict(g["config"], g["seed"])) == g["weights_digest"]


@pytest.mark.parametrize("fname", ["htdemucs_full.pt", "htdemucs_6s_full.pt"])
def test_weights_match_reference_init_registry(fname):
    g = golden(fname)
    assert _digest(htdemucs_state_dict(g["config"], g["seed"])) == g["weights_digest"]


def test_synth_track_is_deterministic():
    g = golden("htdemucs_full.pt")
    assert torch.equal(synth_track(1.0, 0)[None], g["mix"])
    x = synth_track(2.0, 7)
    assert x.shape == (2, 88200) and abs(float(x.abs().max()) - 0.9) < 1e-6


def test_oracle_small_forward():
    g = golden("htdemucs_small.pt")
    sd = htdemucs_state_dict(g["config"], g["seed"])
    out = htdemucs_forward(sd, g["mix"], g["config"])
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < TOL


@pytest.mark.parametrize("fname", ["htdemucs_full.pt", "htdemucs_6s_full.pt"])
def test_oracle_registry_forward(fname):
    g = golden(fname)
    sd = htdemucs_state_dict(g["config"], g["seed"])
    out = htdemucs_forward(sd, g["mix"], g["config"])
    d = g["decimate"]
    assert rel_err(out[..., ::d], g["out"]) < TOL
    sums = out.double().sum(dim=(0, 2, 3))
    sumsq = out.double().pow(2).sum(dim=(0, 2, 3))
    assert torch.allclose(sums, g["sum"], rtol=1e-4, atol=1e-3)
    assert torch.allclose(sumsq, g["sumsq"], rtol=1e-5)


@pytest.mark.parametrize("key,shifts", [("shifts0", 0), ("shifts1", 1)])
def test_oracle_apply_model(key, shifts):
    g = golden("apply_small.pt")
    cfg = g["config"]
    sd = htdemucs_state_dict(cfg, g["seed"])
    out = apply_model(lambda b: htdemucs_forward(sd, b, cfg), g["mix"], len(cfg["sources"]),
                      segment_length(cfg), cfg["samplerate"], shifts=shifts, overlap=g["overlap"],
                      chunk_batch_size=g["chunk_batch_size"], offsets=g[key].get("offsets"))
    assert rel_err(out[..., :: g["decimate"]], g[key]["out"]) < TOL
    assert torch.allclose(out.double().sum(dim=(0, 2, 3)), g[key]["sum"], rtol=1e-4, atol=1e-3)


def test_apply_pointwise_model_reconstructs_input():
    """A model returning [x, 2x] must come back exactly (reference test_apply.py:269-313)."""
    mix = torch.randn(1, 2, 10000)
    out = apply_model(lambda b: torch.stack([b, 2 * b], dim=1), mix, 2, 3000, 44100, overlap=0.25,
                      chunk_batch_size=2)
    assert torch.allclose(out[:, 0], mix, atol=1e-5)
    assert torch.allclose(out[:, 1], 2 * mix, atol=1e-5)


def test_split_weight_and_padding_edges():
    w = split_weight(7)
    assert torch.allclose(w, torch.tensor([1, 2, 3, 4, 3, 2, 1], dtype=torch.float32) / 4)
    mix = torch.arange(10, dtype=torch.float32)[None, None]
    # last chunk of length 4 padded to 6 is centred: one sample before, one zero after
    assert padded_chunk(mix, 6, 6, 6).flatten().tolist() == [5, 6, 7, 8, 9, 0]


def test_oracle_rejects_too_long():
    cfg = htdemucs_config("htdemucs", channels=8, bottom_channels=32, t_heads=4, t_layers=1, segment=0.5)
    with pytest.raises(ValueError):
        htdemucs_forward(htdemucs_state_dict(cfg, 0), torch.zeros(1, 2, 22051), cfg)


def _config_fixture(fname: str):
    """A measured-configuration fixture, its regenerated input (digest-checked) and weights."""
    g = golden(fname)
    mix = synth_track(g["mix_seconds"], g["mix_seed"])[None]
    assert hashlib.sha256(mix.contiguous().numpy().tobytes()).hexdigest() == g["mix_digest"]
    sd = htdemucs_state_dict(g["config"], g["seed"])
    assert _digest(sd) == g["weights_digest"]
    return g, mix, sd


def check_config_record(out: torch.Tensor, g: dict, tol: float) -> None:
    """``out`` [1, S, C, L] against a fixture's decimated samples, full windows and per-stem sums."""
    w = g["window"]
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < tol
    wins = torch.stack([out[..., s:s + w] for s in g["windows"]])
    assert rel_err(wins, g["win_out"]) < tol
    assert torch.allclose(out.double().sum(dim=(0, 2, 3)), g["sum"], rtol=1e-4, atol=1e-2)
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["sumsq"], rtol=1e-4)


def test_oracle_config0_ten_second_clip():
    """The registry htdemucs on the 10 s seed-0 clip through apply_model, batch 1 (configs 0)."""
    g, mix, sd = _config_fixture("htdemucs_cfg0.pt")
    cfg = g["config"]
    out = apply_model(lambda b: htdemucs_forward(sd, b, cfg), mix, 4, segment_length(cfg), cfg["samplerate"],
                      overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"])
    check_config_record(out, g, TOL)


def test_oracle_config2_six_source_vocals_one_shift():
    """htdemucs_6s (seed 2) with one shift round drawn after random.seed(2); the vocals stem."""
    g, mix, sd = _config_fixture("htdemucs_6s_cfg2.pt")
    cfg = g["config"]
    out = apply_model(lambda b: htdemucs_forward(sd, b, cfg), mix, 6, segment_length(cfg), cfg["samplerate"],
                      shifts=1, overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"], offsets=g["offsets"])
    v = cfg["sources"].index(g["stem"])
    check_config_record(out[:, v:v + 1], g, TOL)
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["stem_sumsq"], rtol=1e-4)
