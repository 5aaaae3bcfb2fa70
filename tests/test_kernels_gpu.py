"""Per-kernel parity on the GPU: each C-ABI entry point against a plain PyTorch
fp32 reference of the same operation (small, odd shapes and edge cases, in the
manner of the reference's tests/test_metal_kernels.py)."""

from __future__ import annotations

import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err
from unblend_b200 import _lib
from unblend_b200._lib import ACT_GELU, ACT_GLU, ACT_NONE, PRO_ADD, PRO_GN_GELU, PRO_NONE, ConvParams

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _ref_conv(x, w, b, kh, kw, sh, sw, dh, dw, ph, pw):
    """x [B,H,W,C], w [N,KH,KW,C] -> [B,Ho,Wo,N] via F.conv2d."""
    y = F.conv2d(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2), b, (sh, sw), (ph, pw), (dh, dw))
    return y.permute(0, 2, 3, 1)


def _conv(x, w, b, y, *, B, H, W, C, in_s, Ho, Wo, N, out_s, kh=1, kw=1, sh=1, sw=1, dh=1, dw=1, ph=0, pw=0,
          act=ACT_NONE, prologue=PRO_NONE, pro_stats=None, pro_gamma=None, pro_beta=None, pro_per_h=0,
          pro_x2=None, res=None, res_scale=None, stats=None, stats_per_h=0, n_group=None, out_sg=0):
    p = ConvParams()
    p.batch, p.h_in, p.w_in, p.c_in = B, H, W, C
    p.in_sb, p.in_sh, p.in_sw = in_s
    p.h_out, p.w_out, p.n_out = Ho, Wo, N
    p.kh, p.kw, p.sh, p.sw, p.dh, p.dw, p.ph, p.pw = kh, kw, sh, sw, dh, dw, ph, pw
    p.out_sb, p.out_sh, p.out_sw = out_s
    p.out_sg = out_sg
    p.n_group = n_group or (N // 2 if act == ACT_GLU else N)
    p.act, p.prologue = act, prologue
    p.pro_stats, p.pro_gamma, p.pro_beta = _lib.ptr(pro_stats), _lib.ptr(pro_gamma), _lib.ptr(pro_beta)
    p.pro_group_per_h = pro_per_h
    p.pro_x2 = _lib.ptr(pro_x2)
    p.res, p.res_scale = _lib.ptr(res), _lib.ptr(res_scale)
    p.stats, p.stats_per_h = _lib.ptr(stats), stats_per_h
    _lib.call("unblend_conv2d_f32", x.data_ptr(), w.data_ptr(), _lib.ptr(b), y.data_ptr(), ctypes.byref(p))


def _cl(shape):
    return torch.randn(*shape, device="cuda")


# The first two cases (c_in <= 4, eight taps, n_out a multiple of 16) take the
# register-gather first-layer kernel; the others the tiled one.
@pytest.mark.parametrize("B,H,W,C,N,kh,sh,ph", [(2, 36, 13, 4, 48, 8, 4, 2), (1, 20, 7, 1, 16, 8, 4, 2),
                                                (2, 32, 13, 4, 12, 8, 4, 2), (1, 16, 70, 9, 130, 8, 4, 2)])
def test_conv_freq_encoder_gelu(B, H, W, C, N, kh, sh, ph):
    x, w, b = _cl((B, H, W, C)), _cl((N, kh, 1, C)) * 0.2, _cl((N,))
    Ho = (H + 2 * ph - kh) // sh + 1
    y = torch.empty(B, Ho, W, N, device="cuda")
    _conv(x, w, b, y, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=Ho, Wo=W, N=N,
          out_s=(Ho * W * N, W * N, N), kh=kh, sh=sh, ph=ph, act=ACT_GELU)
    ref = F.gelu(_ref_conv(x, w, b, kh, 1, sh, 1, 1, 1, ph, 0))
    assert rel_err(y, ref) < TOL


def test_conv_time_strided_rows_with_capacity():
    B, L, cap, C, N = 2, 37, 40, 3, 10
    xs = _cl((B, cap, C))
    w, b = _cl((N, 1, 8, C)) * 0.3, _cl((N,))
    Wo = -(-L // 4)
    y = torch.full((B, 12, N), float("nan"), device="cuda")
    _conv(xs, w, b, y, B=B, H=1, W=L, C=C, in_s=(cap * C, cap * C, C), Ho=1, Wo=Wo, N=N,
          out_s=(12 * N, 12 * N, N), kw=8, sw=4, pw=2)
    xp = F.pad(xs[:, :L].permute(0, 2, 1), (0, 4 - L % 4))
    ref = F.conv1d(xp, w[:, 0].permute(0, 2, 1), b, 4, 2).permute(0, 2, 1)
    assert rel_err(y[:, :Wo], ref) < TOL
    assert torch.isnan(y[:, Wo:]).all()  # rows past the output length are untouched


@pytest.mark.parametrize("C,N", [(2, 48), (4, 64)])
def test_conv_time_first_layer_thin_path(C, N):
    """Stereo (or CaC) input, 8 taps stride 4: the register-gather kernel, rows past Wo untouched."""
    B, L, cap = 3, 1001, 1004
    xs = _cl((B, cap, C))
    w, b = _cl((N, 1, 8, C)) * 0.3, _cl((N,))
    Wo = -(-L // 4)
    y = torch.full((B, Wo + 3, N), float("nan"), device="cuda")
    _conv(xs, w, b, y, B=B, H=1, W=L, C=C, in_s=(cap * C, cap * C, C), Ho=1, Wo=Wo, N=N,
          out_s=((Wo + 3) * N, (Wo + 3) * N, N), kw=8, sw=4, pw=2, act=ACT_GELU)
    xp = F.pad(xs[:, :L].permute(0, 2, 1), (0, 4 - L % 4))
    ref = F.gelu(F.conv1d(xp, w[:, 0].permute(0, 2, 1), b, 4, 2)).permute(0, 2, 1)
    assert rel_err(y[:, :Wo], ref) < TOL
    assert torch.isnan(y[:, Wo:]).all()


def test_conv_dilated_with_group_stats():
    B, H, W, C, N = 2, 5, 41, 16, 2
    x, w, b = _cl((B, H, W, C)), _cl((N, 1, 3, C)) * 0.2, _cl((N,))
    y = torch.empty(B, H, W, N, device="cuda")
    st = torch.zeros(2 * B * H, device="cuda", dtype=torch.float64)
    _conv(x, w, b, y, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
          out_s=(H * W * N, W * N, N), kw=3, dw=2, pw=2, stats=st, stats_per_h=1)
    ref = _ref_conv(x, w, b, 1, 3, 1, 1, 1, 2, 0, 2)
    assert rel_err(y, ref) < TOL
    # statistics are those of the values written (fp32 partials summed in double)
    r = y.double().reshape(B * H, -1)
    assert torch.allclose(st[0::2], r.sum(1), rtol=1e-6, atol=1e-5)
    assert torch.allclose(st[1::2], r.pow(2).sum(1), rtol=1e-6, atol=1e-5)


def test_conv_gn_gelu_prologue_and_glu_epilogue():
    B, H, W, C, N = 2, 3, 50, 6, 20
    x = _cl((B, H, W, C)) * 3 + 1
    w, b = _cl((N, 1, 1, C)) * 0.3, _cl((N,))
    g, be = _cl((C,)), _cl((C,))
    xg = x.reshape(B * H, -1).double()
    mean, var = xg.mean(1), xg.var(1, unbiased=False)
    st = torch.stack([mean, 1.0 / torch.sqrt(var + 1e-5)], 1).float().reshape(-1).contiguous()
    y = torch.empty(B, H, W, N // 2, device="cuda")
    _conv(x, w, b, y, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
          out_s=(H * W * N // 2, W * N // 2, N // 2), act=ACT_GLU, prologue=PRO_GN_GELU, pro_stats=st,
          pro_gamma=g, pro_beta=be, pro_per_h=1)
    xn = F.group_norm(x.permute(0, 1, 3, 2).reshape(B * H, C, W), 1, g, be, 1e-5)
    xn = F.gelu(xn).reshape(B, H, C, W).permute(0, 1, 3, 2)
    z = _ref_conv(xn, w, b, 1, 1, 1, 1, 1, 1, 0, 0)
    ref = z[..., 0::2] * torch.sigmoid(z[..., 1::2])
    assert rel_err(y, ref) < TOL


def test_conv_skip_add_3x3_glu():
    B, H, W, C, N = 1, 9, 17, 12, 24
    x, s = _cl((B, H, W, C)), _cl((B, H, W, C))
    w, b = _cl((N, 3, 3, C)) * 0.1, _cl((N,))
    y = torch.empty(B, H, W, N // 2, device="cuda")
    _conv(x, w, b, y, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
          out_s=(H * W * N // 2, W * N // 2, N // 2), kh=3, kw=3, ph=1, pw=1, act=ACT_GLU,
          prologue=PRO_ADD, pro_x2=s)
    z = _ref_conv(x + s, w, b, 3, 3, 1, 1, 1, 1, 1, 1)
    assert rel_err(y, z[..., 0::2] * torch.sigmoid(z[..., 1::2])) < TOL


def test_linear_residual_layerscale_with_stats_inplace():
    B, L, K, N = 3, 77, 64, 48
    x, w, b = _cl((B, L, K)), _cl((N, 1, 1, K)) * 0.1, _cl((N,))
    res, sc = _cl((B, L, N)), _cl((N,))
    out = res.clone()
    st = torch.zeros(2 * B, device="cuda", dtype=torch.float64)
    _conv(x, w, b, out, B=B, H=1, W=L, C=K, in_s=(L * K, L * K, K), Ho=1, Wo=L, N=N,
          out_s=(L * N, L * N, N), res=out, res_scale=sc, stats=st)
    ref = res + sc * (x @ w[:, 0, 0].t() + b)
    assert rel_err(out, ref) < TOL
    assert torch.allclose(st[0::2], ref.double().reshape(B, -1).sum(1), rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("freq", [True, False])
def test_transposed_conv_phase_split(freq):
    from unblend_b200.htdemucs import _convtr_taps3

    B, P, T, Cin, Cout = 2, 7, 5, 12, 6
    wt, bias = torch.randn(Cin, Cout, 8) * 0.2, torch.randn(Cout)
    w3, b4 = _convtr_taps3(wt).cuda(), bias.repeat(4).cuda()
    if freq:
        x = _cl((B, P, T, Cin))
        out = torch.empty(B, 4 * P, T, Cout, device="cuda")
        row = T * Cout
        _conv(x, w3, b4, out.view(-1), B=B, H=P, W=T, C=Cin, in_s=(P * T * Cin, T * Cin, Cin), Ho=P, Wo=T,
              N=4 * Cout, out_s=(4 * P * T * Cout, 4 * row, Cout), kh=3, ph=1, n_group=Cout, out_sg=row)
        ref = F.conv_transpose2d(x.permute(0, 3, 1, 2), wt[..., None].cuda(), bias.cuda(), (4, 1))
        ref = ref[:, :, 2:-2, :].permute(0, 2, 3, 1)
    else:
        x = _cl((B, P, Cin))
        out = torch.empty(B, 4 * P, Cout, device="cuda")
        _conv(x, w3, b4, out.view(-1), B=B, H=1, W=P, C=Cin, in_s=(P * Cin, P * Cin, Cin), Ho=1, Wo=P,
              N=4 * Cout, out_s=(4 * P * Cout, 4 * P * Cout, 4 * Cout), kw=3, pw=1, n_group=Cout, out_sg=Cout)
        ref = F.conv_transpose1d(x.permute(0, 2, 1), wt.cuda(), bias.cuda(), 4)[:, :, 2:2 + 4 * P]
        ref = ref.permute(0, 2, 1)
    assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("lq,lk,heads,hd", [(100, 70, 3, 64), (130, 64, 2, 48), (9, 200, 4, 8)])
def test_attention(lq, lk, heads, hd):
    B, D = 2, heads * hd
    q, k, v = _cl((B, lq, D)), _cl((B, lk, D)), _cl((B, lk, D))
    o = torch.empty(B, lq, D, device="cuda")
    _lib.call("unblend_attention_f32", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, heads, lq, lk,
              hd, lq * D, D, lk * D, D, lq * D, D, 1.0 / math.sqrt(hd))
    qh = q.view(B, lq, heads, hd).transpose(1, 2)
    kh = k.view(B, lk, heads, hd).transpose(1, 2)
    vh = v.view(B, lk, heads, hd).transpose(1, 2)
    ref = (torch.softmax(qh @ kh.transpose(-1, -2) / math.sqrt(hd), -1) @ vh).transpose(1, 2).reshape(B, lq, D)
    assert rel_err(o, ref) < TOL


def test_layer_norm_with_positional_table():
    rows, c, prow = 50, 512, 25
    x, g, b, pos = _cl((rows, c)) * 2 + 3, _cl((c,)), _cl((c,)), _cl((prow, c))
    y = torch.empty_like(x)
    _lib.call("unblend_layer_norm", x.data_ptr(), y.data_ptr(), g.data_ptr(), b.data_ptr(), pos.data_ptr(), 1.0,
              prow, rows, c)
    ref = F.layer_norm(x, (c,), g, b, 1e-5) + pos.repeat(2, 1)
    assert rel_err(y, ref) < TOL


def test_group_norm_apply_and_mean_std():
    B, n = 3, 10007
    x = _cl((B, n)) * 5 + 2
    work = torch.empty(2 * B, device="cuda", dtype=torch.float64)
    st = torch.empty(2 * B, device="cuda")
    _lib.call("unblend_mean_std", x.data_ptr(), work.data_ptr(), st.data_ptr(), B, n)
    var, mean = torch.var_mean(x.double(), dim=1)
    assert torch.allclose(st[0::2].double(), mean, rtol=1e-6, atol=1e-6)
    assert torch.allclose(st[1::2].double(), var.sqrt(), rtol=1e-6)
    y = torch.empty_like(x)
    _lib.call("unblend_standardize", x.data_ptr(), y.data_ptr(), st.data_ptr(), n, B)
    assert rel_err(y, (x - mean[:, None].float()) / (1e-5 + var.sqrt()[:, None].float())) < TOL


def test_stft_front_end():
    from oracle.htdemucs_oracle import _spec

    mix = _cl((2, 2, 30000)) * 0.3
    frames = -(-30000 // 1024)
    spec = torch.empty(2, 2048, frames, 4, device="cuda")
    win = torch.hann_window(4096, device="cuda")
    _lib.call("unblend_stft_cac", mix.data_ptr(), spec.data_ptr(), win.data_ptr(), 2, 30000, 4096)
    z = _spec(mix.cpu(), 4096)  # [B, 2, 2048, frames] complex
    ref = torch.view_as_real(z).permute(0, 2, 3, 1, 4).reshape(2, 2048, frames, 4)
    assert rel_err(spec, ref) < 1e-5


def test_istft_output_stage():
    from oracle.htdemucs_oracle import _ispec

    B, S, L = 2, 3, 30000
    frames = -(-L // 1024)
    spec = _cl((B, 2048, frames, S * 4)) * 0.1
    xt = _cl((B, L + 3, S * 2)) * 0.1
    fst = torch.tensor([0.01, 1.5, -0.02, 0.7], device="cuda")
    tst = torch.tensor([0.03, 0.4, 0.0, 2.0], device="cuda")
    win = torch.hann_window(4096, device="cuda")
    fb = torch.empty(B * S * 2 * frames * 4096, device="cuda")
    out = torch.empty(B, S, 2, L, device="cuda")
    _lib.call("unblend_istft_output", spec.data_ptr(), xt.data_ptr(), (L + 3) * S * 2, fst.data_ptr(),
              tst.data_ptr(), win.data_ptr(), fb.data_ptr(), out.data_ptr(), B, S, L, 4096)
    sc = spec.cpu().view(B, 2048, frames, S, 2, 2)  # (s, c, ri)
    den = sc * fst.cpu()[1::2].view(B, 1, 1, 1, 1, 1) + fst.cpu()[0::2].view(B, 1, 1, 1, 1, 1)
    zc = torch.view_as_complex(den.permute(0, 3, 4, 1, 2, 5).contiguous())  # [B, S, 2, F, T]
    xs = _ispec(zc, L, 4096)
    xtt = xt.cpu()[:, :L].view(B, L, S, 2).permute(0, 2, 3, 1)
    ref = xs + xtt * tst.cpu()[1::2].view(B, 1, 1, 1) + tst.cpu()[0::2].view(B, 1, 1, 1)
    assert rel_err(out, ref) < 1e-5


def test_segment_engine_pointwise_model():
    from oracle.apply_oracle import apply_unshifted

    C, L, seg, stride = 2, 10000, 3000, 2250
    track = _cl((C, L))
    offsets = list(range(0, L, stride))
    acc = torch.zeros(2 * C, L, device="cuda")
    sw = torch.zeros(L, device="cuda")
    for i in range(0, len(offsets), 3):
        grp = offsets[i : i + 3]
        off_t = torch.tensor(grp, device="cuda", dtype=torch.int64)
        batch = torch.empty(len(grp), C, seg, device="cuda")
        _lib.call("unblend_gather_chunks", track.data_ptr(), C, L, off_t.data_ptr(), len(grp), seg, batch.data_ptr())
        y = torch.stack([batch, 2 * batch], 1).contiguous()  # [n, S=2, C, seg]
        hi = min(L, grp[-1] + seg)
        _lib.call("unblend_overlap_add", y.data_ptr(), len(grp), 2 * C, seg, off_t.data_ptr(), L, grp[0], hi,
                  1.0, acc.data_ptr(), sw.data_ptr())
    out = torch.empty_like(acc)
    _lib.call("unblend_divide", acc.data_ptr(), sw.data_ptr(), out.data_ptr(), 2 * C, L)
    ref = apply_unshifted(lambda b: torch.stack([b, 2 * b], 1), track.cpu()[None], 2, seg, 0.25, 3)
    assert rel_err(out.view(1, 2, C, L), ref) < 1e-6
    assert torch.allclose(out.view(2, C, L)[0], track, atol=1e-5)


# ---------------------------------------------------------------- tensor-core (tcgen05) convolution

def _split_tf32(w: torch.Tensor):
    from unblend_b200.htdemucs import split_tf32

    return split_tf32(w)


def _conv_tc(x, w, b, y, mode, block_n, **kw):
    """Same parameter block as _conv, launched on the tcgen05 kernel."""
    wf = w.reshape(w.shape[0], -1).contiguous()
    if mode == _lib.TC_TF32X3:
        whi, wlo = _split_tf32(wf)
    elif mode in (_lib.TC_BF16X3, _lib.TC_BF16X3_TAPS):
        from unblend_b200.convnet import split_bf16

        whi, wlo = split_bf16(wf)
    else:
        whi, wlo = wf.to(torch.bfloat16).contiguous(), None
    p = ConvParams()
    B, H, W, C = kw["B"], kw["H"], kw["W"], kw["C"]
    p.batch, p.h_in, p.w_in, p.c_in = B, H, W, C
    p.in_sb, p.in_sh, p.in_sw = kw["in_s"]
    p.h_out, p.w_out, p.n_out = kw["Ho"], kw["Wo"], kw["N"]
    p.kh, p.kw, p.sh, p.sw = kw.get("kh", 1), kw.get("kw", 1), kw.get("sh", 1), kw.get("sw", 1)
    p.dh, p.dw, p.ph, p.pw = kw.get("dh", 1), kw.get("dw", 1), kw.get("ph", 0), kw.get("pw", 0)
    p.out_sb, p.out_sh, p.out_sw = kw["out_s"]
    p.out_sg = kw.get("out_sg", 0)
    act = kw.get("act", ACT_NONE)
    p.n_group = kw.get("n_group") or (kw["N"] // 2 if act == ACT_GLU else kw["N"])
    p.act = act
    p.res, p.res_scale = _lib.ptr(kw.get("res")), _lib.ptr(kw.get("res_scale"))
    p.stats, p.stats_per_h = _lib.ptr(kw.get("stats")), kw.get("stats_per_h", 0)
    if kw.get("post") is not None:
        p.post, p.post_sh = kw["post"].data_ptr(), kw["post"].shape[1]
    p.y_bf16 = 1 if y.dtype == torch.bfloat16 else 0
    p.x_bf16 = 1 if x.dtype == torch.bfloat16 else 0
    _lib.call("unblend_conv2d_tc", x.data_ptr(), whi.data_ptr(), _lib.ptr(wlo), _lib.ptr(b), y.data_ptr(),
              ctypes.byref(p), mode, block_n)
    torch.cuda.synchronize()
    assert _lib.error_flag() == 0


# 3-pass TF32 (hi*hi + hi*lo + lo*hi) leaves ~2^-20 relative error per product;
# over K = 512..864 that is a few 1e-5 of the output RMS. 3-pass bf16 keeps 16
# significant bits per operand (~2^-16 per product, random in sign), which with
# the accumulator's own rounding stays within 1e-4 of the RMS.
TC_TOL = {_lib.TC_TF32X3: 6e-5, _lib.TC_BF16: 3e-2, _lib.TC_BF16X3: 1e-4}
MODES = [_lib.TC_TF32X3, _lib.TC_BF16, _lib.TC_BF16X3]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("block_n", [64, 128, 256])
def test_tc_linear_residual_stats(mode, block_n):
    B, L, K, N = 2, 300, 512, 200
    x, w, b = _cl((B, L, K)), _cl((N, 1, 1, K)) * 0.05, _cl((N,))
    res, sc = _cl((B, L, N)), _cl((N,))
    out = res.clone()
    st = torch.zeros(2 * B, device="cuda", dtype=torch.float64)
    _conv_tc(x, w, b, out, mode, block_n, B=B, H=1, W=L, C=K, in_s=(L * K, L * K, K), Ho=1, Wo=L, N=N,
             out_s=(L * N, L * N, N), res=out, res_scale=sc, stats=st)
    ref = res + sc * (x @ w[:, 0, 0].t() + b)
    assert rel_err(out, ref) < TC_TOL[mode]
    # statistics are those of the values written
    o = out.double().reshape(B, -1)
    assert torch.allclose(st[0::2], o.sum(1), rtol=1e-6, atol=1e-4)
    assert torch.allclose(st[1::2], o.pow(2).sum(1), rtol=1e-6)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("block_n", [128, 256])
def test_tc_freq_encoder_conv_112_row_tiles(mode, block_n):
    B, H, W, C, N = 2, 16, 336, 48, 96
    x, w, b = _cl((B, H, W, C)), _cl((N, 8, 1, C)) * 0.05, _cl((N,))
    Ho = H // 4
    y = torch.empty(B, Ho, W, N, device="cuda")
    _conv_tc(x, w, b, y, mode, block_n, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=Ho, Wo=W, N=N,
             out_s=(Ho * W * N, W * N, N), kh=8, sh=4, ph=2, act=ACT_GELU)
    ref = F.gelu(_ref_conv(x, w, b, 8, 1, 4, 1, 1, 1, 2, 0))
    assert rel_err(y, ref) < TC_TOL[mode]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("block_n", [128, 192, 256])
def test_tc_3x3_glu_and_dilated(mode, block_n):
    B, H, W, C, N = 1, 8, 336, 96, 192
    x, w, b = _cl((B, H, W, C)), _cl((N, 3, 3, C)) * 0.03, _cl((N,))
    y = torch.empty(B, H, W, N // 2, device="cuda")
    _conv_tc(x, w, b, y, mode, block_n, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
             out_s=(H * W * N // 2, W * N // 2, N // 2), kh=3, kw=3, ph=1, pw=1, act=ACT_GLU)
    z = _ref_conv(x, w, b, 3, 3, 1, 1, 1, 1, 1, 1)
    assert rel_err(y, z[..., 0::2] * torch.sigmoid(z[..., 1::2])) < TC_TOL[mode]
    # dilated k=3 along w with per-(b, h) statistics
    w2, b2 = _cl((64, 1, 3, C)) * 0.05, _cl((64,))
    y2 = torch.empty(B, H, W, 64, device="cuda")
    st = torch.zeros(2 * B * H, device="cuda", dtype=torch.float64)
    _conv_tc(x, w2, b2, y2, mode, 64, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=64,
             out_s=(H * W * 64, W * 64, 64), kw=3, dw=2, pw=2, stats=st, stats_per_h=1)
    ref2 = _ref_conv(x, w2, b2, 1, 3, 1, 1, 1, 2, 0, 2)
    assert rel_err(y2, ref2) < TC_TOL[mode]
    o2 = y2.double().reshape(B * H, -1)
    assert torch.allclose(st[0::2], o2.sum(1), rtol=1e-6, atol=1e-4)


@pytest.mark.parametrize("block_n", [64, 96, 128])
def test_tc_3pass_shared_tap_loads(block_n):
    """Mode 4: the three taps of each 3-wide kernel row share one input load and hi / lo split; the
    fp32 bound holds on 3x3 GLU, dilated k=3 (shifts 2 and 4) and the time branch's 1x3 rewrite, and the
    result stays within fp32 summation-order noise of mode 2."""
    B, H, W, C, N = 1, 8, 336, 96, 192
    x, w, b = _cl((B, H, W, C)), _cl((N, 3, 3, C)) * 0.03, _cl((N,))
    kw = dict(B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
              out_s=(H * W * N // 2, W * N // 2, N // 2), kh=3, kw=3, ph=1, pw=1, act=ACT_GLU)
    y = torch.empty(B, H, W, N // 2, device="cuda")
    _conv_tc(x, w, b, y, _lib.TC_BF16X3_TAPS, block_n, **kw)
    z = _ref_conv(x, w, b, 3, 3, 1, 1, 1, 1, 1, 1)
    assert rel_err(y, z[..., 0::2] * torch.sigmoid(z[..., 1::2])) < TC_TOL[_lib.TC_BF16X3]
    y2 = torch.empty_like(y)
    _conv_tc(x, w, b, y2, _lib.TC_BF16X3, block_n, **kw)
    assert rel_err(y, y2) < 1e-5
    for dw in (1, 2, 4):
        w2, b2 = _cl((64, 1, 3, C)) * 0.05, _cl((64,))
        y3 = torch.empty(B, H, W, 64, device="cuda")
        st = torch.zeros(2 * B * H, device="cuda", dtype=torch.float64)
        _conv_tc(x, w2, b2, y3, _lib.TC_BF16X3_TAPS, min(block_n, 64), B=B, H=H, W=W, C=C,
                 in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=64, out_s=(H * W * 64, W * 64, 64), kw=3, dw=dw,
                 pw=dw, stats=st, stats_per_h=1)
        assert rel_err(y3, _ref_conv(x, w2, b2, 1, 3, 1, 1, 1, dw, 0, dw)) < TC_TOL[_lib.TC_BF16X3], dw
        o3 = y3.double().reshape(B * H, -1)
        assert torch.allclose(st[0::2], o3.sum(1), rtol=1e-6, atol=1e-4)
    # time branch: 1 x 3 over 2 x 1000 positions (tiles past the end of the rows are masked)
    L, Ct = 1000, 48
    xt, wt, bt = _cl((2, 1, L, Ct)), _cl((96, 1, 3, Ct)) * 0.05, _cl((96,))
    yt = torch.empty(2, 1, L, 48, device="cuda")
    _conv_tc(xt, wt, bt, yt, _lib.TC_BF16X3_TAPS, block_n, B=2, H=1, W=L, C=Ct, in_s=(L * Ct, L * Ct, Ct), Ho=1,
             Wo=L, N=96, out_s=(L * 48, L * 48, 48), kw=3, pw=1, act=ACT_GLU)
    zt = _ref_conv(xt, wt, bt, 1, 3, 1, 1, 1, 1, 0, 1)
    assert rel_err(yt, zt[..., 0::2] * torch.sigmoid(zt[..., 1::2])) < TC_TOL[_lib.TC_BF16X3]


def test_tc_3pass_shared_tap_loads_rejects_wide_tiles():
    x, w, b = _cl((1, 4, 64, 32)), _cl((64, 3, 3, 32)), _cl((64,))
    y = torch.empty(1, 4, 64, 64, device="cuda")
    with pytest.raises(RuntimeError):
        _conv_tc(x, w, b, y, _lib.TC_BF16X3_TAPS, 192, B=1, H=4, W=64, C=32, in_s=(4 * 64 * 32, 64 * 32, 32), Ho=4,
                 Wo=64, N=64, out_s=(4 * 64 * 64, 64 * 64, 64), kh=3, kw=3, ph=1, pw=1)


@pytest.mark.parametrize("mode", MODES + [_lib.TC_BF16X3_TAPS], ids=["tf32x3", "bf16", "bf16x3", "bf16x3-taps"])
@pytest.mark.parametrize("B", [8, 32])
def test_tc_decoder3_rewrite_headline_shape(mode, B):
    """The largest 3x3 rewrite of the headline forward: HTDemucs decoder.3 (512 frequency rows x 336
    frames per segment, 48 -> 96 channels, GLU) at the bench's 32 segments per launch and at 8, with
    the tile width the model picks (96), checked over every output against torch's fp32 convolution."""
    H, W, C, N = 512, 336, 48, 96
    g = torch.Generator(device="cuda").manual_seed(B)
    x = torch.randn(B, H, W, C, device="cuda", generator=g)
    w = torch.randn(N, 3, 3, C, device="cuda", generator=g) * 0.05
    b = torch.randn(N, device="cuda", generator=g)
    y = torch.empty(B, H, W, N // 2, device="cuda")
    _conv_tc(x, w, b, y, mode, 96, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
             out_s=(H * W * N // 2, W * N // 2, N // 2), kh=3, kw=3, ph=1, pw=1, act=ACT_GLU)
    err = 0.0
    for i in range(0, B, 4):  # the fp32 reference in slices of 4 segments (bounded memory)
        z = _ref_conv(x[i:i + 4], w, b, 3, 3, 1, 1, 1, 1, 1, 1)
        err = max(err, rel_err(y[i:i + 4], z[..., 0::2] * torch.sigmoid(z[..., 1::2])))
    assert err < TC_TOL[_lib.TC_BF16X3 if mode == _lib.TC_BF16X3_TAPS else mode]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("block_n", [128, 256])
def test_tc_time_stride4_super_rows(mode, block_n):
    B, L, C, N = 2, 1001, 48, 96
    cap = 4 * -(-L // 4)
    xs = torch.zeros(B, cap, C, device="cuda")
    xs[:, :L] = _cl((B, L, C))
    w, b = _cl((N, 1, 8, C)) * 0.05, _cl((N,))
    Wo = -(-L // 4)
    y = torch.empty(B, Wo, N, device="cuda")
    _conv_tc(xs, w, b, y, mode, block_n, B=B, H=1, W=L, C=C, in_s=(cap * C, cap * C, C), Ho=1, Wo=Wo, N=N,
             out_s=(Wo * N, Wo * N, N), kw=8, sw=4, pw=2)
    xp = F.pad(xs[:, :L].permute(0, 2, 1), (0, cap - L))
    ref = F.conv1d(xp, w[:, 0].permute(0, 2, 1), b, 4, 2).permute(0, 2, 1)
    assert rel_err(y, ref) < TC_TOL[mode]


@pytest.mark.parametrize("mode", MODES)
def test_tc_transposed_conv_phase_split(mode):
    from unblend_b200.htdemucs import _convtr_taps3

    B, P, T, Cin, Cout = 2, 8, 336, 96, 48
    wt, bias = torch.randn(Cin, Cout, 8) * 0.05, torch.randn(Cout)
    w3, b4 = _convtr_taps3(wt).cuda(), bias.repeat(4).cuda()
    x = _cl((B, P, T, Cin))
    out = torch.empty(B, 4 * P, T, Cout, device="cuda")
    row = T * Cout
    _conv_tc(x, w3[:, :, None, :], b4, out.view(-1), mode, 192, B=B, H=P, W=T, C=Cin,
             in_s=(P * T * Cin, T * Cin, Cin), Ho=P, Wo=T, N=4 * Cout, out_s=(4 * P * T * Cout, 4 * row, Cout),
             kh=3, ph=1, n_group=Cout, out_sg=row, act=ACT_GELU)
    ref = F.conv_transpose2d(x.permute(0, 3, 1, 2), wt[..., None].cuda(), bias.cuda(), (4, 1))
    ref = F.gelu(ref[:, :, 2:-2, :].permute(0, 2, 3, 1))
    assert rel_err(out, ref) < TC_TOL[mode]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("with_res", [False, True])
def test_tc_post_activation_add(mode, with_res):
    """GLU(conv) + post[h, c] per output row (the frequency-embedding fold), through the
    bulk-store epilogue (no residual) and the per-lane residual epilogue."""
    B, H, W, C, N = 2, 6, 336, 48, 96
    x, w, b = _cl((B, H, W, C)), _cl((N, 1, 1, C)) * 0.1, _cl((N,))
    post = _cl((H, N // 2))
    res = _cl((B, H, W, N // 2)) if with_res else None
    y = res.clone() if with_res else torch.empty(B, H, W, N // 2, device="cuda")
    _conv_tc(x, w, b, y, mode, 128, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
             out_s=(H * W * N // 2, W * N // 2, N // 2), act=ACT_GLU, post=post, res=y if with_res else None)
    z = _ref_conv(x, w, b, 1, 1, 1, 1, 1, 1, 0, 0)
    ref = z[..., 0::2] * torch.sigmoid(z[..., 1::2]) + post[None, :, None, :]
    if with_res:
        ref = ref + res
    assert rel_err(y, ref) < TC_TOL[mode]


@pytest.mark.parametrize("block_n", [128, 256])
def test_tc_bf16_output(block_n):
    """Linear layer whose output leaves the bulk-store epilogue as bf16 (round to nearest
    even of the fp32 result), rows not a multiple of 128."""
    B, L, K, N = 2, 300, 512, 1536
    x, w, b = _cl((B, L, K)), _cl((N, 1, 1, K)) * 0.05, _cl((N,))
    y = torch.empty(B, L, N, device="cuda", dtype=torch.bfloat16)
    _conv_tc(x, w, b, y, _lib.TC_BF16, block_n, B=B, H=1, W=L, C=K, in_s=(L * K, L * K, K), Ho=1, Wo=L, N=N,
             out_s=(L * N, L * N, N))
    ref = x @ w[:, 0, 0].t() + b
    assert rel_err(y.float(), ref) < TC_TOL[_lib.TC_BF16]


@pytest.mark.parametrize("kh,kw,C,N,block_n,act", [(3, 3, 48, 96, 96, ACT_GLU), (1, 1, 512, 512, 256, ACT_GELU),
                                                   (1, 3, 64, 192, 192, ACT_NONE)])
def test_tc_bf16_activations_match_the_converted_path(kh, kw, C, N, block_n, act):
    """Mode 3 (bf16 activations loaded as they are) against mode 1 on the same values in fp32:
    mode 1 rounds its fp32 A tiles to bf16 (nearest even) before the same MMAs, so the two
    outputs are identical, sub-tap groups of 3-wide kernel rows included."""
    B, H, W = 2, 5, 300
    x = _cl((B, H, W, C)).to(torch.bfloat16)
    w, b = _cl((N, kh, kw, C)) * 0.05, _cl((N,))
    n_final = N // 2 if act == ACT_GLU else N
    outs = []
    for mode, xin in ((_lib.TC_BF16, x.float()), (_lib.TC_BF16_ACT, x)):
        y = torch.empty(B, H, W, n_final, device="cuda")
        _conv_tc(xin, w, b, y, mode, block_n, B=B, H=H, W=W, C=C, in_s=(H * W * C, W * C, C), Ho=H, Wo=W, N=N,
                 out_s=(H * W * n_final, W * n_final, n_final), kh=kh, kw=kw, ph=kh // 2, pw=kw // 2, act=act)
        outs.append(y)
    assert torch.equal(outs[0], outs[1])
    ref = _ref_conv(x.float(), w, b, kh, kw, 1, 1, 1, 1, kh // 2, kw // 2)
    if act == ACT_GLU:
        ref = ref[..., 0::2] * torch.sigmoid(ref[..., 1::2])
    elif act == ACT_GELU:
        ref = torch.nn.functional.gelu(ref)
    assert rel_err(outs[1], ref) < TC_TOL[_lib.TC_BF16]


def test_layer_norm_bf16_output():
    rows, c = 3000, 512
    x = torch.randn(rows, c, device="cuda") * 3 + 1
    g, bt = torch.randn(c, device="cuda"), torch.randn(c, device="cuda")
    y = torch.empty(rows, c, device="cuda", dtype=torch.bfloat16)
    _lib.call("unblend_layer_norm_bf16", x.data_ptr(), y.data_ptr(), g.data_ptr(), bt.data_ptr(), None, 1.0, 1,
              rows, c)
    ref = torch.nn.functional.layer_norm(x, (c,), g, bt, 1e-5)
    # One bf16 rounding of an fp32-accurate value: within half an ulp of bf16 (2^-9 relative).
    assert ((y.float() - ref).abs() <= ref.abs() * 2.0 ** -8 + 1e-6).all()


@pytest.mark.parametrize("C,N,kh,kw,dw,act,res", [(48, 96, 3, 3, 1, ACT_GLU, False), (64, 130, 1, 1, 1, ACT_NONE, True),
                                                  (32, 64, 1, 3, 2, ACT_GELU, False)])
def test_conv_simt_wide_tiles_match_the_generic_kernel(C, N, kh, kw, dw, act, res):
    """Channels a multiple of 16 and >= 64 outputs take the 128 x 128 tile kernel; the same
    problem with a padded channel stride takes the generic one. Both sum every output over K
    in the same order (bit-identical), and match torch's fp32 convolution."""
    B, H, W = 2, 5, 301
    x = _cl((B, H, W, C))
    w, b = _cl((N, kh, kw, C)) * 0.1, _cl((N,))
    xp = torch.zeros(B, H, W, C + 4, device="cuda")
    xp[..., :C] = x
    n_final = N // 2 if act == ACT_GLU else N
    r = _cl((B, H, W, n_final)) if res else None
    sc = _cl((n_final,)) if res else None
    outs = []
    for xin, cs in ((x, C), (xp, C + 4)):
        y = torch.empty(B, H, W, n_final, device="cuda")
        st = torch.zeros(2 * B * H, device="cuda", dtype=torch.float64)
        _conv(xin, w, b, y, B=B, H=H, W=W, C=C, in_s=(H * W * cs, W * cs, cs), Ho=H, Wo=W, N=N,
              out_s=(H * W * n_final, W * n_final, n_final), kh=kh, kw=kw, dw=dw, ph=kh // 2, pw=dw * (kw // 2),
              act=act, res=r, res_scale=sc, stats=st, stats_per_h=1)
        outs.append((y, st))
    assert torch.equal(outs[0][0], outs[1][0])
    # Statistics: fp32 partial sums of 8 (wide) or 4 (generic) values per thread, then double.
    assert torch.allclose(outs[0][1], outs[1][1], rtol=1e-6, atol=1e-4)
    z = _ref_conv(x, w, b, kh, kw, 1, 1, 1, dw, kh // 2, dw * (kw // 2))
    if act == ACT_GLU:
        z = z[..., 0::2] * torch.sigmoid(z[..., 1::2])
    elif act == ACT_GELU:
        z = F.gelu(z)
    if res:
        z = r + sc * z
    assert rel_err(outs[0][0], z) < TOL
