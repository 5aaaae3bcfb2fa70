"""Host-side logic of the CUDA BS-RoFormer (no GPU): weight packing into grouped
GEMM layouts, the band tables, the inference contract and its validation."""

from __future__ import annotations

import pytest
import torch

from conftest import golden
from unblend_b200.apply import ValidationError
from unblend_b200.roformer import BSRoformerCuda, build_roformer
from unblend_b200.synth import DEFAULT_FREQS_PER_BANDS, bsroformer_config, bsroformer_state_dict


@pytest.fixture(scope="module")
def small():
    g = golden("bsroformer_small.pt")
    return g["config"], bsroformer_state_dict(g["config"], g["seed"])


def test_band_tables_cover_the_features(small):
    cfg, sd = small
    m = BSRoformerCuda(cfg, sd, precision="fp32")
    assert m.bands == len(DEFAULT_FREQS_PER_BANDS) == 62
    assert m.features == 4 * (cfg["stft_n_fft"] // 2 + 1)
    assert m.starts[0] == 0 and m.starts[-1] == m.features
    assert all(s % 8 == 0 for s in m.starts[:-1])  # 16-byte aligned bf16 band slices


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_band_split_packing_reproduces_the_per_band_linears(small, precision):
    cfg, sd = small
    m = BSRoformerCuda(cfg, sd, precision=precision)
    lin = m._lin["band_split"]
    w = lin.hi.float() + (lin.lo if lin.lo is not None else 0)
    dim = cfg["dim"]
    for b, (a0, r0, n, k, o0) in enumerate(lin.groups):
        ref = sd[f"band_split.to_features.{b}.1.weight"]
        assert (a0, r0, n, k, o0) == (m.starts[b], b * dim, dim, m.widths[b], b * dim)
        tol = 0 if precision == "fp32" else 1e-2
        assert torch.allclose(w[r0:r0 + n, :k], ref, atol=tol)
        assert torch.count_nonzero(w[r0:r0 + n, k:]) == 0  # zero padding beyond the band


def test_mask_output_layer_is_glu_interleaved(small):
    cfg, sd = small
    m = BSRoformerCuda(cfg, sd, precision="fp32")
    lin = m._lin[m.mask_layers[0][-1]]
    w = lin.hi + lin.lo
    a0, r0, n, k, o0 = lin.groups[5]
    ref = sd["mask_estimators.0.to_freqs.5.0.2.weight"]
    half = n // 2
    assert torch.equal(w[r0:r0 + n:2], ref[:half]) and torch.equal(w[r0 + 1:r0 + n:2], ref[half:])
    assert o0 == m.starts[5] and n == 2 * m.widths[5]


def test_inference_contract_and_validation(small):
    cfg, sd = small
    m = build_roformer("bs_roformer", cfg, sources=["vocals", "other"], samplerate=44100, segment_samples=22050,
                       state=sd, precision="fp32")
    assert m.output_complement and m.sources == ["vocals", "other"]
    assert m.max_allowed_segment == 0.5
    m.configure_inference(sources=["vocals"], samplerate=44100, segment_samples=44100)
    assert not m.output_complement
    with pytest.raises(ValidationError):
        m.configure_inference(sources=["a", "b", "c"], samplerate=44100, segment_samples=100)
    with pytest.raises(ValidationError):
        m.configure_inference(sources=["a"], samplerate=True, segment_samples=100)
    with pytest.raises(ValidationError):
        build_roformer("scnet", cfg, sources=["a"], samplerate=44100, segment_samples=100, state=sd)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        m(torch.zeros(1, 2, 4096))
    with pytest.raises(ValidationError):
        BSRoformerCuda(bsroformer_config(dim=64, depth=1, heads=4, dim_head=16, linear_transformer_depth=1), sd)
