"""Restatement of the SCNet forward (CPU oracle, test use only).

Restates ``SCNet.forward`` / ``SCNetMasked.forward`` (unblend/scnet.py:746-800,
837-895) as plain fp32 torch CPU operations on a reference-layout
``state_dict``: the normalised STFT without a window (Hann for the masked
variant), the ``SDblock`` encoder (band split, per-band strided convolutions,
``ConvolutionModule`` stacks, GELU, global 3x3 convolution;
unblend/scnet.py:50-330), the dual-path trunk (GroupNorm, bidirectional LSTM
along frequency then time, linear projection, residual; real FFT along time
between layers; unblend/scnet.py:333-540), the decoder (``FusionLayer`` and
``SUlayer``; unblend/scnet.py:100-235) and the inverse STFT. The LSTM is the
explicit recurrence of ``torch.nn.LSTM`` (gates i, f, g, o; c = f c + i g;
h = o tanh c), written out so the oracle does not depend on a fused kernel.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def stft_padding(samples: int, hop: int) -> int:
    """Trailing zeros before the STFT: to a hop boundary, plus one hop for an odd frame count
    (unblend/scnet.py:543-572)."""
    padding = hop - samples % hop
    if (samples + padding) // hop % 2 == 0:
        padding += hop
    return padding


def band_splits(freq: int, cfg: dict) -> list[tuple[int, int]]:
    """The three frequency bands of an SD layer (unblend/scnet.py:186-194)."""
    sr = cfg["band_SR"]
    a = math.ceil(freq * sr[0])
    b = math.ceil(freq * (sr[0] + sr[1]))
    return [(0, a), (a, b), (b, freq)]


def _conv_module(sd: dict, p: str, x: torch.Tensor, depth: int, kernel: int) -> torch.Tensor:
    """``ConvolutionModule`` on [N, C, T] (unblend/scnet.py:50-97)."""
    pad = kernel // 2
    for d in range(abs(depth)):
        q = f"{p}.layers.{d}"
        y = F.group_norm(x, 1, sd[f"{q}.0.weight"], sd[f"{q}.0.bias"], 1e-5)
        y = F.conv1d(y, sd[f"{q}.1.weight"], sd[f"{q}.1.bias"], padding=pad)
        y = F.glu(y, 1)
        h = y.shape[1]
        y = F.conv1d(y, sd[f"{q}.3.weight"], sd[f"{q}.3.bias"], padding=pad, groups=h)
        y = F.group_norm(y, 1, sd[f"{q}.4.weight"], sd[f"{q}.4.bias"], 1e-5)
        y = y * y.sigmoid()
        y = F.conv1d(y, sd[f"{q}.6.weight"], sd[f"{q}.6.bias"])
        x = x + y
    return x


def _sd_block(sd: dict, p: str, x: torch.Tensor, cfg: dict):
    """``SDblock`` (unblend/scnet.py:238-330) on [B, C, F, T]."""
    freq = x.shape[2]
    bands, orig = [], []
    for j, (start, end) in enumerate(band_splits(freq, cfg)):
        stride, kernel = cfg["band_stride"][j], cfg["band_kernel"][j]
        e = x[:, :, start:end, :]
        orig.append(end - start)
        total = kernel - stride if stride == 1 else (stride - e.shape[2] % stride) % stride
        e = F.pad(e, (0, 0, total // 2, total - total // 2))
        y = F.conv2d(e, sd[f"{p}.SDlayer.convs.{j}.weight"], sd[f"{p}.SDlayer.convs.{j}.bias"], (stride, 1))
        b, c, f, t = y.shape
        z = _conv_module(sd, f"{p}.conv_modules.{j}", y.permute(0, 2, 1, 3).reshape(b * f, c, t),
                         cfg["conv_depths"][j], cfg["conv_kernel"])
        bands.append(F.gelu(z.view(b, f, c, t).permute(0, 2, 1, 3)))
    lengths = [band.shape[2] for band in bands]
    full = torch.cat(bands, dim=2)
    out = F.conv2d(full, sd[f"{p}.globalconv.weight"], sd[f"{p}.globalconv.bias"], padding=1)
    return out, full, lengths, orig


def _fusion(sd: dict, p: str, x: torch.Tensor, skip: torch.Tensor) -> torch.Tensor:
    """``FusionLayer``: (x + skip) repeated on channels, 3x3 conv, GLU (unblend/scnet.py:100-145)."""
    x = (x + skip).repeat(1, 2, 1, 1)
    return F.glu(F.conv2d(x, sd[f"{p}.conv.weight"], sd[f"{p}.conv.bias"], padding=1), dim=1)


def _su_layer(sd: dict, p: str, x: torch.Tensor, lengths: list[int], orig: list[int], cfg: dict) -> torch.Tensor:
    """``SUlayer``: per-band transposed convolutions, symmetric trim, concatenation (unblend/scnet.py:196-235)."""
    outs, start = [], 0
    for j in range(3):
        end = start + lengths[j] if j < 2 else x.shape[2]
        y = F.conv_transpose2d(x[:, :, start:end, :], sd[f"{p}.convtrs.{j}.weight"], sd[f"{p}.convtrs.{j}.bias"],
                               (cfg["band_stride"][j], 1))
        dist = abs(orig[j] - y.shape[2]) // 2
        outs.append(y[:, :, dist:dist + orig[j], :])
        start = end
    return torch.cat(outs, dim=2)


def lstm_bidirectional(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    """One bidirectional ``nn.LSTM`` layer on [L, N, d] -> [L, N, 2H] (forward | reverse)."""
    outs = []
    for suffix in ("", "_reverse"):
        wih, whh = sd[f"{p}.weight_ih_l0{suffix}"], sd[f"{p}.weight_hh_l0{suffix}"]
        hid = whh.shape[1]
        xp = x @ wih.t() + sd[f"{p}.bias_ih_l0{suffix}"] + sd[f"{p}.bias_hh_l0{suffix}"]
        h = x.new_zeros(x.shape[1], hid)
        c = x.new_zeros(x.shape[1], hid)
        out = x.new_empty(x.shape[0], x.shape[1], hid)
        steps = range(x.shape[0]) if not suffix else range(x.shape[0] - 1, -1, -1)
        for t in steps:
            g = xp[t] + h @ whh.t()
            i, f, gg, o = g.chunk(4, dim=1)
            c = f.sigmoid() * c + i.sigmoid() * gg.tanh()
            h = o.sigmoid() * c.tanh()
            out[t] = h
        outs.append(out)
    return torch.cat(outs, dim=2)


def _dual_path(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    """``DualPathRNN`` (unblend/scnet.py:440-500): frequency path, then time path, each residual."""
    b, c, f, t = x.shape
    y = F.group_norm(x, 1, sd[f"{p}.norm_layers.0.weight"], sd[f"{p}.norm_layers.0.bias"], 1e-5)
    y = y.permute(2, 0, 3, 1).reshape(f, b * t, c)
    y = lstm_bidirectional(sd, f"{p}.lstm_layers.0", y)
    y = F.linear(y, sd[f"{p}.linear_layers.0.weight"], sd[f"{p}.linear_layers.0.bias"])
    x = y.view(f, b, t, c).permute(1, 3, 0, 2) + x
    y = F.group_norm(x, 1, sd[f"{p}.norm_layers.1.weight"], sd[f"{p}.norm_layers.1.bias"], 1e-5)
    y = y.permute(3, 0, 2, 1).reshape(t, b * f, c)
    y = lstm_bidirectional(sd, f"{p}.lstm_layers.1", y)
    y = F.linear(y, sd[f"{p}.linear_layers.1.weight"], sd[f"{p}.linear_layers.1.bias"])
    return y.view(t, b, f, c).permute(1, 3, 2, 0) + x


def _feature_conversion(x: torch.Tensor, inverse: bool) -> torch.Tensor:
    """Orthonormal real FFT along time, real and imaginary parts on channels (unblend/scnet.py:333-437)."""
    if inverse:
        half = x.shape[1] // 2
        return torch.fft.irfft(torch.complex(x[:, :half], x[:, half:]), dim=3, norm="ortho")
    spec = torch.fft.rfft(x, dim=3, norm="ortho")
    return torch.cat([spec.real, spec.imag], dim=1)


def forward_core(sd: dict, x: torch.Tensor, cfg: dict) -> torch.Tensor:
    """Encoder, trunk and decoder on the packed spectrogram [B, 2C, F, T] (unblend/scnet.py:713-744)."""
    skips, lens, origs = [], [], []
    for i in range(len(cfg["dims"]) - 1):
        x, skip, lengths, orig = _sd_block(sd, f"encoder.{i}", x, cfg)
        skips.append(skip)
        lens.append(lengths)
        origs.append(orig)
    for i in range(cfg["num_dplayer"]):
        x = _dual_path(sd, f"separation_net.dp_modules.{i}", x)
        x = _feature_conversion(x, inverse=bool(i % 2))
    for j in range(len(cfg["dims"]) - 1):
        x = _fusion(sd, f"decoder.{j}.0", x, skips.pop())
        x = _su_layer(sd, f"decoder.{j}.1", x, lens.pop(), origs.pop(), cfg)
    return x


def _stft_kwargs(cfg: dict, masked: bool) -> dict:
    kw = dict(n_fft=cfg["nfft"], hop_length=cfg["hop_size"], win_length=cfg["win_size"], center=True,
              normalized=cfg["normalized"])
    if masked:
        kw["window"] = torch.hann_window(cfg["nfft"], periodic=True)
    return kw


def scnet_forward(sd: dict, mix: torch.Tensor, cfg: dict) -> torch.Tensor:
    """``SCNet.forward`` / ``SCNetMasked.forward``: [B, C, L] -> [B, S, C, L]."""
    masked = cfg.get("architecture") == "scnet_masked"
    batch, chans = mix.shape[0], mix.shape[1]
    S = len(cfg["sources"])
    padding = stft_padding(mix.shape[-1], cfg["hop_size"])
    mix = F.pad(mix, (0, padding))
    kw = _stft_kwargs(cfg, masked)
    x = torch.stft(mix.float().reshape(-1, mix.shape[-1]), return_complex=True, **kw)
    x = torch.view_as_real(x)
    x = x.permute(0, 3, 1, 2).reshape(batch, 2 * chans, x.shape[1], x.shape[2])
    _, _, freq, frames = x.shape
    n = cfg["dims"][0]
    if masked:
        mixture = x.repeat(1, S, 1, 1)
        x = x + sd["pos_embed_f"][:, :, :freq, :]
        y = forward_core(sd, x, cfg)
        y = F.gelu(F.conv2d(y, sd["mask_layer.0.weight"], sd["mask_layer.0.bias"], padding=1))
        mask = torch.tanh(F.conv2d(y, sd["mask_layer.2.weight"], sd["mask_layer.2.bias"]))
        mixture = torch.view_as_complex(mixture.view(batch, n, -1, freq, frames).reshape(-1, 2, freq, frames)
                                        .permute(0, 2, 3, 1).contiguous())
        mask = torch.view_as_complex(mask.view(batch, n, -1, freq, frames).reshape(-1, 2, freq, frames)
                                     .permute(0, 2, 3, 1).contiguous())
        y = torch.istft(mixture * mask, **kw)
    else:
        y = forward_core(sd, x, cfg)
        y = torch.view_as_complex(y.view(batch, n, -1, freq, frames).reshape(-1, 2, freq, frames)
                                  .permute(0, 2, 3, 1).contiguous())
        y = torch.istft(y, **kw)
    y = y.reshape(batch, S, chans, -1)
    return y[:, :, :, :-padding]
