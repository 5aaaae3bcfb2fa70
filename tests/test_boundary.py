"""Host-side boundary checks that need no GPU: construction from a reference
module, rejected configurations and argument validation of the segment engine."""

from __future__ import annotations

import sys

import pytest
import torch

from conftest import GOLDEN, reference_path
from unblend_b200.apply import ValidationError, apply_model
from unblend_b200.htdemucs import HTDemucsCuda, split_tf32
from unblend_b200.synth import htdemucs_config, htdemucs_state_dict

SMALL = dict(channels=8, bottom_channels=32, t_heads=4, t_layers=3, segment=0.5)
REF = reference_path()


def test_packed_weights_cover_contract_and_split_is_exact():
    cfg = htdemucs_config("htdemucs", **SMALL)
    m = HTDemucsCuda(cfg, htdemucs_state_dict(cfg, 0))
    assert m.sources == cfg["sources"] and m.samplerate == 44100 and m.max_allowed_segment == 0.5
    assert m._fixed_batch_shape is False
    assert all(not p.requires_grad for p in m.parameters())
    w = torch.randn(1000)
    hi, lo = split_tf32(w)
    assert torch.equal(hi + lo, w)
    assert torch.all((hi.view(torch.int32) & 0x1FFF) == 0)


def test_rejects_unsupported_variants_and_precisions():
    cfg = htdemucs_config("htdemucs", **SMALL)
    sd = htdemucs_state_dict(cfg, 0)
    with pytest.raises(ValueError):
        HTDemucsCuda(dict(cfg, nfft=2048), sd)
    with pytest.raises(ValueError):
        HTDemucsCuda(cfg, sd, precision="fp8")


def test_segment_engine_validates_arguments():
    cfg = htdemucs_config("htdemucs", **SMALL)
    m = HTDemucsCuda(cfg, htdemucs_state_dict(cfg, 0))
    with pytest.raises(ValidationError):
        apply_model(m, torch.zeros(2, 100), overlap=1.0)
    with pytest.raises(ValidationError):
        apply_model(m, torch.zeros(2, 100), transition_power=0.5)
    with pytest.raises(ValidationError):
        apply_model(m, torch.zeros(2, 100), chunk_batch_size=0)


@pytest.mark.skipif(REF is None, reason="reference checkout not found (set UNBLEND_REFERENCE)")
def test_from_reference_module_matches_direct_construction():
    sys.path.insert(0, GOLDEN)
    from make_golden import import_reference

    unblend = import_reference(REF)
    cfg = htdemucs_config("htdemucs", **SMALL)
    torch.manual_seed(0)
    ref = unblend.htdemucs.HTDemucs(**cfg)
    a = HTDemucsCuda.from_reference(ref)
    b = HTDemucsCuda(cfg, htdemucs_state_dict(cfg, 0))
    sa, sb = a.state_dict(), b.state_dict()
    assert sa.keys() == sb.keys()
    assert all(torch.equal(sa[k], sb[k]) for k in sa)


@pytest.mark.parametrize("freq", [True, False])
def test_transposed_conv_as_three_tap_phases(freq):
    """The packed transposed-conv weight, run as a 3-tap conv whose channel group s is
    output row 4p + s, reproduces ConvTranspose (stride 4, kernel 8, crop 2)."""
    import torch.nn.functional as F

    from unblend_b200.htdemucs import _convtr_taps3

    g = torch.Generator().manual_seed(3)
    B, P, Cin, Cout = 2, 9, 5, 3
    wt, x = torch.randn(Cin, Cout, 8, generator=g, dtype=torch.float64), torch.randn(B, Cin, P, generator=g,
                                                                                       dtype=torch.float64)
    w3 = _convtr_taps3(wt if not freq else wt[..., None])  # [4 Cout, 3, Cin]
    y = F.conv1d(x, w3.permute(0, 2, 1), padding=1)  # [B, 4 Cout, P]
    got = y.view(B, 4, Cout, P).permute(0, 2, 3, 1).reshape(B, Cout, 4 * P)
    ref = F.conv_transpose1d(x, wt, stride=4)[:, :, 2:2 + 4 * P]
    assert torch.allclose(got, ref, atol=1e-12)
