"""Mel-Band RoFormer on the GPU: the band gather / scatter-average kernels
against PyTorch index_select / index_add, then the whole forward against the
reference's own outputs (golden fixtures: a reduced model and the
``melband_roformer_kim`` registry configuration).

Tolerances (north star): fp32 max-abs error <= 1e-4 x output RMS; bf16 at
>= 40 dB SNR per stem.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import golden, rel_err
from unblend_b200 import _lib
from unblend_b200.apply import apply_model
from unblend_b200.roformer import MelBandRoformerCuda, build_roformer
from unblend_b200.synth import melband_state_dict

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-4
BF16_MIN_SNR_DB = 40.0


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> list[float]:
    o, r = out.double().cpu(), ref.double().cpu()
    res = []
    for s in range(r.shape[1]):
        num = r[:, s].pow(2).sum()
        den = (o[:, s] - r[:, s]).pow(2).sum()
        res.append(float(10 * math.log10(num / den)) if den > 0 else float("inf"))
    return res


@pytest.mark.parametrize("rows,pairs,n", [(7, 50, 130), (300, 2050, 4100)])
def test_gather_and_scatter_mean_pairs(rows, pairs, n):
    g = torch.Generator().manual_seed(rows + n)
    src = torch.randn(rows, 2 * pairs + 6, generator=g).cuda()  # leading dim wider than the pairs
    idx = torch.cat([torch.arange(pairs), torch.randint(0, pairs, (n - pairs,), generator=g)])
    idx = idx[torch.randperm(n, generator=g)]
    dst = torch.full((rows, 2 * n + 4), float("nan"), device="cuda")
    _lib.call("unblend_gather_pairs", src.data_ptr(), src.shape[1], rows, idx.int().cuda().data_ptr(), n,
              dst.data_ptr(), dst.shape[1])
    ref = src[:, : 2 * pairs].view(rows, pairs, 2)[:, idx.cuda()].reshape(rows, 2 * n)
    assert torch.equal(dst[:, : 2 * n], ref)
    assert torch.isnan(dst[:, 2 * n:]).all()
    # Scatter back: every pair is covered at least once.
    order = torch.argsort(idx, stable=True)
    counts = torch.bincount(idx, minlength=pairs)
    off = torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]).int().cuda()
    back = torch.empty(rows, 2 * pairs, device="cuda")
    _lib.call("unblend_scatter_mean_pairs", dst.data_ptr(), dst.shape[1], rows, off.data_ptr(),
              order.int().cuda().data_ptr(), pairs, back.data_ptr(), 2 * pairs)
    summed = torch.zeros(rows, pairs, 2, device="cuda").index_add_(1, idx.cuda(), ref.view(rows, n, 2))
    expect = (summed / counts.cuda().view(1, -1, 1).float()).reshape(rows, 2 * pairs)
    assert rel_err(back, expect) < 1e-6
    assert rel_err(back, src[:, : 2 * pairs]) < 1e-6  # the mean of copies is the original


def _model(g, precision):
    return MelBandRoformerCuda(g["config"], melband_state_dict(g["config"], g["seed"]), precision=precision).cuda()


def test_small_forward_fp32_matches_reference():
    g = golden("melband_small.pt")
    out = _model(g, "fp32")(g["mix"].cuda())
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < FP32_TOL
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_kim_config_with_complement_matches_reference(precision):
    g = golden("melband_kim.pt")
    m = build_roformer("mel_band_roformer", g["config"], sources=g["sources"], samplerate=44100,
                       segment_samples=352800, state=melband_state_dict(g["config"], g["seed"]),
                       precision=precision).cuda()
    out = m(g["mix"].cuda()).cpu()[..., :: g["decimate"]]
    if precision == "fp32":
        assert rel_err(out, g["out"]) < FP32_TOL
    else:
        assert min(snr_db(out, g["out"])) >= BF16_MIN_SNR_DB
    assert _lib.error_flag() == 0


def test_apply_model_and_graphs_match_eager():
    """The segment engine drives the Mel-Band model like any other; CUDA-graph replay equals eager."""
    g = golden("melband_small.pt")
    m = _model(g, "fp32")
    m.configure_inference(sources=["vocals", "other"], samplerate=44100, segment_samples=22050)
    track = g["mix"][0].cuda()
    eager = apply_model(m, track, overlap=0.25, chunk_batch_size=2)
    m.enable_compiled_core()
    graphed = apply_model(m, track, overlap=0.25, chunk_batch_size=2)
    m.disable_compiled_core()
    assert eager.shape == (2, 2, track.shape[-1])
    assert rel_err(graphed, eager) < 1e-6

