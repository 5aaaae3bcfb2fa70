"""End-to-end parity of the CUDA HTDemucs forward and segment engine against
the reference outputs (golden fixtures) and the CPU oracle.

Tolerances (north star): fp32 max-abs error <= 1e-4 x output RMS; bf16 at
>= 40 dB SNR per stem.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import golden, rel_err
from unblend_b200 import _lib
from unblend_b200.htdemucs import HTDemucsCuda
from unblend_b200.synth import htdemucs_state_dict

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-4
BF16_MIN_SNR_DB = 40.0


def _model(g, precision="fp32") -> HTDemucsCuda:
    return HTDemucsCuda(g["config"], htdemucs_state_dict(g["config"], g["seed"]), precision=precision).cuda()


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> list[float]:
    """Per-stem SNR in dB of ``out`` against ``ref`` ([B, S, C, L])."""
    o, r = out.double().cpu(), ref.double().cpu()
    res = []
    for s in range(r.shape[1]):
        num = r[:, s].pow(2).sum()
        den = (o[:, s] - r[:, s]).pow(2).sum()
        res.append(float(10 * math.log10(num / den)) if den > 0 else float("inf"))
    return res


@pytest.mark.parametrize("precision", ["fp32", "fp32-simt"])
def test_small_config_matches_reference(precision):
    g = golden("htdemucs_small.pt")
    out = _model(g, precision)(g["mix"].cuda())
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < FP32_TOL
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("precision", ["fp32", "fp32-simt"])
@pytest.mark.parametrize("fname", ["htdemucs_full.pt", "htdemucs_6s_full.pt"])
def test_registry_config_matches_reference(fname, precision):
    g = golden(fname)
    out = _model(g, precision)(g["mix"].cuda()).cpu()
    d = g["decimate"]
    assert rel_err(out[..., ::d], g["out"]) < FP32_TOL
    sums = out.double().pow(2).sum(dim=(0, 2, 3))
    assert torch.allclose(sums, g["sumsq"], rtol=1e-4)
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("split", ["bf16x3", "tf32x3"])
@pytest.mark.parametrize("fname", ["htdemucs_small.pt", "htdemucs_full.pt", "htdemucs_6s_full.pt"])
def test_fp32_operand_splits_match_reference(fname, split):
    """Both operand splits of the fp32 tensor-core convolutions and attention hold the fp32 bound."""
    g = golden(fname)
    m = _model(g)
    m.fp32_split = m.attention_split = split
    out = m(g["mix"].cuda()).cpu()
    d = g.get("decimate", 1)
    assert rel_err(out[..., ::d], g["out"]) < FP32_TOL
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("fname", ["htdemucs_full.pt", "htdemucs_6s_full.pt"])
def test_registry_config_bf16_snr(fname):
    g = golden(fname)
    out = _model(g, "bf16")(g["mix"].cuda()).cpu()
    d = g["decimate"]
    snrs = snr_db(out[..., ::d], g["out"])
    assert min(snrs) >= BF16_MIN_SNR_DB, snrs


def test_batch_rows_are_independent():
    g = golden("htdemucs_small.pt")
    m = _model(g)
    mix = g["mix"].cuda()
    both = m(mix)
    one = m(mix[1:2])
    assert rel_err(both[1:2], one) < 1e-5


def test_contract_and_validation():
    g = golden("htdemucs_small.pt")
    m = _model(g)
    assert m.sources == ["drums", "bass", "other", "vocals"]
    assert m.samplerate == 44100 and m.audio_channels == 2 and m.max_allowed_segment == 0.5
    with pytest.raises(ValueError):
        m(torch.zeros(1, 2, 22051, device="cuda"))
    with pytest.raises(RuntimeError):
        m.cpu()(torch.zeros(1, 2, 100))


@pytest.mark.parametrize("key,shifts", [("shifts0", 0), ("shifts1", 1)])
def test_apply_model_matches_reference(key, shifts):
    from unblend_b200.apply import apply_model

    g = golden("apply_small.pt")
    m = _model(g)
    out = apply_model(m, g["mix"].cuda(), shifts=shifts, overlap=g["overlap"],
                      chunk_batch_size=g["chunk_batch_size"], shift_offsets=g[key].get("offsets"))
    assert rel_err(out.cpu()[..., :: g["decimate"]], g[key]["out"]) < FP32_TOL


def test_compiled_core_replays_cuda_graphs():
    """enable_compiled_core: the captured launch sequence reproduces the eager forward; tails are zero-padded."""
    from unblend_b200.apply import apply_model

    g = golden("htdemucs_small.pt")
    m = _model(g)
    mix = g["mix"].cuda()
    eager = m(mix)
    eager_half = m(mix * 0.5)
    m.enable_compiled_core()
    assert m._fixed_batch_shape
    first = m(mix)
    second = m(mix * 0.5)
    assert torch.equal(first, eager)
    assert torch.equal(second, eager_half)
    m.disable_compiled_core()
    assert not m._fixed_batch_shape and "_graphed" not in m.__dict__
    ga = golden("apply_small.pt")
    ma = _model(ga)
    ma.enable_compiled_core()
    out = apply_model(ma, ga["mix"].cuda(), overlap=ga["overlap"], chunk_batch_size=ga["chunk_batch_size"])
    assert rel_err(out.cpu()[..., :: ga["decimate"]], ga["shifts0"]["out"]) < FP32_TOL
    # 4 chunks at 3 per batch: the full batch is replayed from a graph, the 1-chunk tail
    # (below 7/8 of a batch) runs eagerly at its own size instead of being padded.
    assert [k[0][0] for k in ma.__dict__["_graphed"].graphs] == [ga["chunk_batch_size"]]
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("fname,stems", [("htdemucs_6s_full.pt", ["vocals"]), ("htdemucs_small.pt", ["bass", "drums"])])
def test_selected_stems_match_reference_slices(fname, stems):
    """select_sources: only the chosen stems are materialised (last ConvTranspose rows and iSTFT), each equal
    to its slice of the reference output; the selection can be widened again and is validated."""
    from unblend_b200.apply import ValidationError

    g = golden(fname)
    m = _model(g)
    full_sources = list(m.sources)
    ref = g["out"]
    d = g.get("decimate", 1)
    m.select_sources(stems)
    assert m.sources == stems
    out = m(g["mix"].cuda()).cpu()
    assert out.shape[1] == len(stems)
    idx = [full_sources.index(s) for s in stems]
    assert rel_err(out[..., ::d], ref[:, idx]) < FP32_TOL
    m.select_sources(None)
    assert m.sources == full_sources
    assert rel_err(m(g["mix"].cuda()).cpu()[..., ::d], ref) < FP32_TOL
    with pytest.raises(ValidationError):
        m.select_sources(["kazoo"])
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("case", ["weighted", "only_drums", "only_bass"])
def test_model_ensemble_matches_reference(case):
    """ModelEnsemble under apply_model: per-source weights over shared shift offsets, and the one-hot
    specialist shortcut of use_only_stem, against the reference's own ensemble outputs."""
    from unblend_b200.apply import ModelEnsemble, apply_model

    g = golden("ensemble_small.pt")
    members = [HTDemucsCuda(g["config"], htdemucs_state_dict(g["config"], s), precision="fp32").cuda()
               for s in g["seeds"]]
    c = g[case]
    ens = ModelEnsemble(members, weights=c["weights"])
    kw = dict(overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"])
    if case == "weighted":
        out = apply_model(ens, g["mix"].cuda(), shifts=1, shift_offsets=c["offsets"], **kw)
    else:
        out = apply_model(ens, g["mix"].cuda(), use_only_stem=case[5:], **kw)
    assert rel_err(out.cpu()[..., :: g["decimate"]], c["out"]) < FP32_TOL
    assert _lib.error_flag() == 0
