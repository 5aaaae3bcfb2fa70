"""SCNet on the GPU: each new kernel against a PyTorch reference of the same op,
then the whole model and the segment engine against the reference's own
outputs (fixtures from ``tests/golden/make_golden.py <reference> scnet``).

Tolerances: fp32 max-abs error <= 1e-4 x output RMS; bf16 >= 40 dB SNR per stem.
"""

from __future__ import annotations

import hashlib
import math

import pytest
import torch
import torch.nn.functional as F

from conftest import golden, rel_err
from oracle.scnet_oracle import lstm_bidirectional
from unblend_b200 import _lib
from unblend_b200.apply import apply_model
from unblend_b200.scnet import SCNetCuda
from unblend_b200.synth import scnet_state_dict, synth_track

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-4
BF16_MIN_SNR_DB = 40.0


def snr_db(out: torch.Tensor, ref: torch.Tensor) -> list[float]:
    o, r = out.double().cpu(), ref.double().cpu()
    res = []
    for s in range(r.shape[1]):
        den = (o[:, s] - r[:, s]).pow(2).sum()
        res.append(float(10 * math.log10(r[:, s].pow(2).sum() / den)) if den > 0 else float("inf"))
    return res


# ---------------------------------------------------------------- kernels

def test_swap_axes_with_embedding_and_stem_split():
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2, 37, 45, 4, device="cuda", generator=g)
    pos = torch.randn(4, 45, device="cuda", generator=g)
    y = torch.empty(2, 45, 37, 4, device="cuda")
    _lib.call("unblend_swap_axes", x.data_ptr(), y.data_ptr(), pos.data_ptr(), 2, 37, 45, 1)
    assert torch.equal(y, x.permute(0, 2, 1, 3) + pos.t()[None, :, None, :])
    z = torch.randn(3, 33, 70, 12, device="cuda", generator=g)  # [B, F, T, 3 stems x 4]
    w = torch.empty(3, 3, 70, 33, 4, device="cuda")
    _lib.call("unblend_swap_axes", z.data_ptr(), w.data_ptr(), None, 3, 33, 70, 3)
    assert torch.equal(w, z.view(3, 33, 70, 3, 4).permute(3, 0, 2, 1, 4))


def test_depthwise3_and_row_sums():
    g = torch.Generator(device="cuda").manual_seed(2)
    rows, T, c = 11, 476, 8
    z = torch.randn(rows, T, c, device="cuda", generator=g)
    w = torch.randn(c, 3, device="cuda", generator=g)
    b = torch.randn(c, device="cuda", generator=g)
    u = torch.empty_like(z)
    st = torch.empty(2 * rows, device="cuda", dtype=torch.float64)
    _lib.call("unblend_depthwise3", z.data_ptr(), w.data_ptr(), b.data_ptr(), u.data_ptr(), st.data_ptr(), rows, T, c)
    ref = F.conv1d(z.permute(0, 2, 1), w[:, None, :], b, padding=1, groups=c).permute(0, 2, 1)
    assert rel_err(u, ref) < 1e-6
    assert torch.allclose(st[0::2], ref.double().sum((1, 2)), rtol=1e-6, atol=1e-6)
    assert torch.allclose(st[1::2], ref.double().pow(2).sum((1, 2)), rtol=1e-6)


@pytest.mark.parametrize("act,fn", [(_lib.ACT_NONE, lambda v: v), (_lib.ACT_GELU, F.gelu), (_lib.ACT_TANH, torch.tanh),
                                    (_lib.ACT_SWISH, lambda v: v * torch.sigmoid(v))])
def test_act_copy_strided(act, fn):
    x = torch.randn(3, 1000, device="cuda") * 3
    y = torch.zeros(3, 1200, device="cuda")
    _lib.call("unblend_act_copy", x.data_ptr(), 1000, y.data_ptr(), 1200, 3, 1000, act)
    assert rel_err(y[:, :1000], fn(x)) < 2e-6
    assert torch.equal(y[:, 1000:], torch.zeros(3, 200, device="cuda"))


@pytest.mark.parametrize("T,c", [(476, 128), (32, 40)])
def test_real_dft_along_frames(T, c):
    g = torch.Generator(device="cuda").manual_seed(T)
    x = torch.randn(5, T, c, device="cuda", generator=g)
    K = T // 2 + 1
    y = torch.empty(5, K, 2 * c, device="cuda")
    _lib.call("unblend_rfft_time", x.data_ptr(), y.data_ptr(), 5, T, c)
    spec = torch.fft.rfft(x.double(), dim=1, norm="ortho")
    # Direct fp32 summation over T terms: a few 1e-6 of the RMS.
    assert rel_err(y, torch.cat([spec.real, spec.imag], dim=2)) < 1e-5
    z = torch.empty(5, T, c, device="cuda")
    _lib.call("unblend_irfft_time", y.data_ptr(), z.data_ptr(), 5, K, c)
    ref = torch.fft.irfft(torch.complex(y[..., :c].double(), y[..., c:].double()), dim=1, norm="ortho")
    assert rel_err(z, ref) < 1e-5
    assert rel_err(z, x) < 1e-5


# Hidden sizes up to 256 run the cluster kernel: one cluster (17, 21, 40 sequences), several
# with a ragged last one (300, 2400, 4700; the last two take eight sequences per thread).
@pytest.mark.parametrize("hid,d,steps,n_seq,freq_axis", [(32, 32, 9, 21, True), (128, 128, 57, 40, False),
                                                         (256, 256, 30, 17, True), (512, 256, 12, 9, False),
                                                         (256, 128, 5, 300, False), (128, 64, 4, 2400, True),
                                                         (64, 32, 3, 4700, False)])
def test_lstm_recurrence_both_directions(hid, d, steps, n_seq, freq_axis):
    torch.manual_seed(hid)
    lstm = torch.nn.LSTM(d, hid, bidirectional=True)
    sd = {f"l.{k}": v.detach() for k, v in lstm.state_dict().items()}
    x = torch.randn(steps, n_seq, d)
    ref = lstm_bidirectional(sd, "l", x)  # [steps, n_seq, 2H]
    with torch.no_grad():
        ref2, _ = lstm(x)
    assert rel_err(ref, ref2) < 1e-5
    # Device layout [B, F, T, 8H] with sequences along F (freq) or T (time), B = 1.
    xp = torch.cat([x @ sd["l.weight_ih_l0"].t() + sd["l.bias_ih_l0"] + sd["l.bias_hh_l0"],
                    x @ sd["l.weight_ih_l0_reverse"].t() + sd["l.bias_ih_l0_reverse"] + sd["l.bias_hh_l0_reverse"]],
                   dim=2)
    if freq_axis:  # sequences (b, t) = n_seq frames, steps along F
        xp_d, Fq, T = xp.contiguous(), steps, n_seq
        args = (n_seq, steps, hid, T, Fq * T, 1, T)
    else:          # sequences (b, f), steps along T
        xp_d, Fq, T = xp.permute(1, 0, 2).contiguous(), n_seq, steps
        args = (n_seq, steps, hid, Fq, Fq * T, T, 1)
    whh = torch.stack([sd["l.weight_hh_l0"].t(), sd["l.weight_hh_l0_reverse"].t()]).contiguous().cuda()
    xp_d = xp_d.cuda()
    h = torch.empty(xp_d.shape[0], xp_d.shape[1], 2 * hid, device="cuda")
    _lib.call("unblend_lstm_recurrence", xp_d.data_ptr(), whh.data_ptr(), h.data_ptr(), *args)
    got = h.cpu() if freq_axis else h.cpu().permute(1, 0, 2)
    assert rel_err(got, ref) < 2e-5


def _lstm_bf16_emulated(xp_seq: torch.Tensor, whh: torch.Tensor, hid: int) -> torch.Tensor:
    """The recurrence with W_hh and h rounded to bf16 for W_hh h (float64 otherwise):
    xp_seq [steps, n_seq, 8 hid] (both directions), whh [2][hid][4 hid] -> [steps, n_seq, 2 hid]."""
    steps, n_seq = xp_seq.shape[:2]
    out = torch.zeros(steps, n_seq, 2 * hid, dtype=torch.float64)
    for d in range(2):
        w = whh[d].to(torch.bfloat16).double()  # [hid, 4 hid] = W_hh^T
        h = torch.zeros(n_seq, hid, dtype=torch.float64)
        c = torch.zeros(n_seq, hid, dtype=torch.float64)
        order = range(steps) if d == 0 else range(steps - 1, -1, -1)
        for t in order:
            g = xp_seq[t, :, 4 * hid * d:4 * hid * (d + 1)].double() + h.to(torch.bfloat16).double() @ w
            i, f, gg, o = g.split(hid, dim=1)
            c = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(gg)
            h = torch.sigmoid(o) * torch.tanh(c)
            out[t, :, hid * d:hid * (d + 1)] = h
    return out


@pytest.mark.parametrize("hid,steps,n_seq,freq_axis", [(128, 13, 100, True), (256, 21, 70, False),
                                                       (256, 7, 130, True), (128, 40, 9, False)])
def test_lstm_recurrence_bf16_tensor_cores(hid, steps, n_seq, freq_axis):
    """The bf16 recurrence against the same arithmetic emulated in float64 (W_hh and h
    rounded to bf16 for the product), and against the fp32 LSTM within bf16 accuracy."""
    torch.manual_seed(hid + steps)
    d = 64
    lstm = torch.nn.LSTM(d, hid, bidirectional=True)
    sd = {f"l.{k}": v.detach() for k, v in lstm.state_dict().items()}
    x = torch.randn(steps, n_seq, d)
    ref32 = lstm_bidirectional(sd, "l", x)
    xp = torch.cat([x @ sd["l.weight_ih_l0"].t() + sd["l.bias_ih_l0"] + sd["l.bias_hh_l0"],
                    x @ sd["l.weight_ih_l0_reverse"].t() + sd["l.bias_ih_l0_reverse"] + sd["l.bias_hh_l0_reverse"]],
                   dim=2)
    whh = torch.stack([sd["l.weight_hh_l0"].t(), sd["l.weight_hh_l0_reverse"].t()]).contiguous()
    emu = _lstm_bf16_emulated(xp, whh, hid)
    if freq_axis:
        xp_d, T, Fq = xp.contiguous(), n_seq, steps
        args = (n_seq, steps, hid, T, Fq * T, 1, T)
    else:
        xp_d, Fq, T = xp.permute(1, 0, 2).contiguous(), n_seq, steps
        args = (n_seq, steps, hid, Fq, Fq * T, T, 1)
    xp_d = xp_d.cuda()
    h = torch.full((xp_d.shape[0], xp_d.shape[1], 2 * hid), float("nan"), device="cuda")
    _lib.call("unblend_lstm_recurrence_bf16", xp_d.data_ptr(), whh.cuda().data_ptr(), h.data_ptr(), *args)
    got = h.cpu() if freq_axis else h.cpu().permute(1, 0, 2)
    assert torch.isfinite(got).all()
    assert rel_err(got, emu) < 5e-3
    assert rel_err(got, ref32) < 5e-2
    assert _lib.error_flag() == 0


# ---------------------------------------------------------------- model

def _model(g, precision="fp32") -> SCNetCuda:
    return SCNetCuda(g["config"], scnet_state_dict(g["config"], g["seed"]), precision=precision).cuda()


@pytest.mark.parametrize("fname", ["scnet_small_reduced.pt", "scnet_plain_reduced.pt"])
@pytest.mark.parametrize("precision", ["fp32", "fp32-simt"])
def test_reduced_models_match_reference(fname, precision):
    g = golden(fname)
    out = _model(g, precision)(g["mix"].cuda())
    assert out.shape == g["out"].shape
    assert rel_err(out, g["out"]) < FP32_TOL
    assert _lib.error_flag() == 0


@pytest.mark.parametrize("fname", ["scnet_small_full.pt", "scnet_xl_full.pt"])
def test_registry_models_match_reference(fname):
    g = golden(fname)
    m = _model(g)
    out = m(g["mix"].cuda()).cpu()
    d = g["decimate"]
    assert rel_err(out[..., ::d], g["out"]) < FP32_TOL
    assert torch.allclose(out.double().pow(2).sum(dim=(0, 2, 3)), g["sumsq"], rtol=1e-4)
    bf = _model(g, "bf16")(g["mix"].cuda()).cpu()
    assert min(snr_db(bf[..., ::d], g["out"])) >= BF16_MIN_SNR_DB
    assert _lib.error_flag() == 0


def test_batch_rows_are_independent():
    g = golden("scnet_small_reduced.pt")
    m = _model(g)
    mix = g["mix"].cuda()
    assert rel_err(m(mix)[1:2], m(mix[1:2])) < 1e-5


def test_apply_model_two_segments_matches_reference():
    g = golden("scnet_apply.pt")
    mix = synth_track(g["mix_seconds"], g["mix_seed"])[None]
    assert hashlib.sha256(mix.contiguous().numpy().tobytes()).hexdigest() == g["mix_digest"]
    m = _model(g)
    out = apply_model(m, mix.cuda(), overlap=g["overlap"], chunk_batch_size=g["chunk_batch_size"]).cpu()
    assert rel_err(out[..., :: g["decimate"]], g["out"]) < FP32_TOL
    wins = torch.stack([out[..., s:s + g["window"]] for s in g["windows"]])
    assert rel_err(wins, g["win_out"]) < FP32_TOL


def test_contract_and_graph_replay():
    g = golden("scnet_small_reduced.pt")
    m = _model(g)
    assert m.sources == ["drums", "bass", "other", "vocals"] and m.samplerate == 44100
    assert abs(m.max_allowed_segment - 11.0) < 1e-9
    from unblend_b200.apply import ValidationError

    with pytest.raises(ValidationError, match="emits 4 stems"):
        m.configure_inference(sources=["vocals"], samplerate=44100, segment_samples=4096)
    mix = g["mix"].cuda()
    eager = m(mix)
    m.enable_compiled_core()
    assert m._fixed_batch_shape
    graphed = m(mix)
    graphed2 = m(mix)
    m.disable_compiled_core()
    assert rel_err(graphed, eager) < 1e-6 and rel_err(graphed2, eager) < 1e-6
    with pytest.raises(RuntimeError):
        m.cpu()(torch.zeros(1, 2, 8192))
