"""Functional fp32 restatement of ``BSRoformer.forward`` (CPU oracle, test use only).

Restates unblend/roformer.py with plain torch CPU ops over a reference-layout
``state_dict``: STFT (1312-1330), per-band RMSNorm + Linear (``BandSplit``,
673-705), the axial time/frequency transformers (``_run_transformers``,
1135-1159) of gated rotary ``Attention`` (478-511) and ``FeedForward``
(274-308), ``final_norm``, the per-band ``MaskEstimator`` MLPs (742-800),
complex masking, zero DC and iSTFT (1331-1379), and the optional
mixture-complement stem (1176-1189); and ``MelBandRoformer.forward``
(1382-1603): mel-band gather, per-transformer output norms, mask
scatter-average.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """``RMSNorm.forward`` off MPS: ``F.rms_norm(x, (dim,), gamma, eps=1e-12)`` (roformer.py:60-91)."""
    return F.rms_norm(x, (x.shape[-1],), gamma, eps=1e-12)


def rotary_tables(seq: int, freqs: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of ``position * freq`` in fp32 (``RotaryEmbedding._cos_sin``, roformer.py:176-198)."""
    angles = torch.arange(seq, dtype=torch.float32)[:, None] * freqs.float()
    return angles.cos(), angles.sin()


def rotate(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Interleaved pair rotation over the sequence axis (``rotate_queries_or_keys``, roformer.py:251-271)."""
    x1, x2 = t.unflatten(-1, (-1, 2)).unbind(dim=-1)
    return torch.stack((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1).flatten(-2)


def attention(sd: dict, p: str, x: torch.Tensor, heads: int) -> torch.Tensor:
    """Gated rotary self-attention ``Attention._forward_chunk`` (roformer.py:478-511)."""
    batch, seq, _ = x.shape
    xn = rms_norm(x, sd[f"{p}.norm.gamma"])
    q, k, v = F.linear(xn, sd[f"{p}.to_qkv.weight"]).chunk(3, dim=-1)
    q, k, v = (t.view(batch, seq, heads, -1).transpose(1, 2) for t in (q, k, v))
    cos, sin = rotary_tables(seq, sd[f"{p}.rotary_embed.freqs"])
    q, k = rotate(q, cos, sin), rotate(k, cos, sin)
    out = F.scaled_dot_product_attention(q, k, v)
    gates = F.linear(xn, sd[f"{p}.to_gates.weight"], sd[f"{p}.to_gates.bias"])
    out = out * gates.transpose(1, 2).unsqueeze(-1).sigmoid()
    out = out.transpose(1, 2).reshape(batch, seq, -1)
    return F.linear(out, sd[f"{p}.to_out.0.weight"])


def feed_forward(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    """``FeedForward``: RMSNorm -> Linear -> GELU -> Linear (roformer.py:274-308)."""
    h = F.gelu(F.linear(rms_norm(x, sd[f"{p}.net.0.gamma"]), sd[f"{p}.net.1.weight"], sd[f"{p}.net.1.bias"]))
    return F.linear(h, sd[f"{p}.net.4.weight"], sd[f"{p}.net.4.bias"])


def transformer(sd: dict, p: str, x: torch.Tensor, depth: int, heads: int) -> torch.Tensor:
    """``Transformer.forward`` with ``norm_output=False`` (roformer.py:612-670)."""
    for j in range(depth):
        x = attention(sd, f"{p}.layers.{j}.0", x, heads) + x
        x = feed_forward(sd, f"{p}.layers.{j}.1", x) + x
    return x


def stft_features(audio: torch.Tensor, cfg: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """STFT of ``[B, C, L]`` audio -> (real view ``[B, F*C, T, 2]``, features ``[B, T, F*C*2]``)."""
    batch, channels, length = audio.shape
    window = torch.hann_window(cfg["stft_win_length"])
    z = torch.stft(audio.reshape(batch * channels, length), n_fft=cfg["stft_n_fft"],
                   hop_length=cfg["stft_hop_length"], win_length=cfg["stft_win_length"],
                   normalized=cfg["stft_normalized"], window=window, return_complex=True)
    zr = torch.view_as_real(z)
    n_freqs, n_frames = zr.shape[-3], zr.shape[-2]
    zr = zr.view(batch, channels, n_freqs, n_frames, 2).permute(0, 2, 1, 3, 4)
    zr = zr.reshape(batch, n_freqs * channels, n_frames, 2)
    x = zr.permute(0, 2, 1, 3).reshape(batch, n_frames, -1)
    return zr, x


@torch.no_grad()
def bsroformer_forward(sd: dict, mix: torch.Tensor, cfg: dict, complement: bool = False) -> torch.Tensor:
    """``BSRoformer.forward`` (unblend/roformer.py:1312-1379) in fp32 on the CPU.

    :param sd: Reference-layout state dict.
    :param mix: ``[B, C, L]`` audio.
    :param cfg: BS-RoFormer constructor config.
    :param complement: Append the mixture-minus-prediction stem (single-stem models).
    :return: ``[B, S, C, L]``.
    """
    sd = {k: v.float().cpu() for k, v in sd.items()}
    mix = mix.float().cpu()
    batch, channels, length = mix.shape
    heads, dim = cfg["heads"], cfg["dim"]
    zr, x = stft_features(mix, cfg)
    n_frames = zr.shape[2]
    widths = [2 * f * channels for f in cfg["freqs_per_bands"]]
    outs, start = [], 0
    for b, w in enumerate(widths):
        xb = rms_norm(x[..., start : start + w], sd[f"band_split.to_features.{b}.0.gamma"])
        outs.append(F.linear(xb, sd[f"band_split.to_features.{b}.1.weight"],
                             sd[f"band_split.to_features.{b}.1.bias"]).unsqueeze(-2))
        start += w
    x = torch.cat(outs, dim=-2)  # [B, T, bands, dim]
    bands = len(widths)
    for i in range(cfg["depth"]):
        x = x.transpose(1, 2).reshape(batch * bands, n_frames, dim)
        x = transformer(sd, f"layers.{i}.0", x, cfg["time_transformer_depth"], heads)
        x = x.view(batch, bands, n_frames, dim).transpose(1, 2).reshape(batch * n_frames, bands, dim)
        x = transformer(sd, f"layers.{i}.1", x, cfg["freq_transformer_depth"], heads)
        x = x.view(batch, n_frames, bands, dim)
    x = rms_norm(x, sd["final_norm.gamma"])
    masks = []
    depth = cfg["mask_estimator_depth"]
    for s in range(cfg["num_stems"]):
        parts = []
        for b in range(bands):
            h = x[..., b, :]
            for k in range(depth):
                p = f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}"
                h = F.linear(h, sd[f"{p}.weight"], sd[f"{p}.bias"])
                if k < depth - 1:
                    h = torch.tanh(h)
            parts.append(F.glu(h, dim=-1))
        masks.append(torch.cat(parts, dim=-1))
    stems = cfg["num_stems"]
    m = torch.stack(masks, dim=1).view(batch, stems, n_frames, -1, 2).permute(0, 1, 3, 2, 4)
    out = torch.view_as_complex(zr.contiguous()).unsqueeze(1) * torch.view_as_complex(m.contiguous())
    n_freqs = out.shape[2] // channels
    out = out.view(batch, stems, n_freqs, channels, n_frames).permute(0, 1, 3, 2, 4)
    out = out.reshape(batch * stems * channels, n_freqs, n_frames)
    if cfg.get("zero_dc", True):
        out = out.clone()
        out[:, 0] = 0
    window = torch.hann_window(cfg["stft_win_length"])
    recon = torch.istft(out, n_fft=cfg["stft_n_fft"], hop_length=cfg["stft_hop_length"],
                        win_length=cfg["stft_win_length"], normalized=cfg["stft_normalized"], window=window,
                        return_complex=False, length=length)
    recon = recon.view(batch, stems, channels, -1)
    if complement:
        recon = torch.cat([recon, mix.unsqueeze(1) - recon], dim=1)
    return recon


def mel_supports(sample_rate: int, n_fft: int, num_bands: int) -> torch.Tensor:
    """``[num_bands, n_fft//2+1]`` bool support of the Slaney mel filter bank (roformer.py:803-878, 1459-1463).

    Written from the filter definition: ``num_bands + 2`` edges equally spaced
    on the Slaney mel scale (linear 200/3 Hz per mel to 1 kHz, then
    logarithmic with 27 steps per factor 6.4) from 0 Hz to Nyquist; filter m
    rises from edge m to m+1 and falls to m+2; a bin is in the band where the
    triangle is positive. DC goes to the first band, Nyquist to the last.
    """
    def to_mel(hz):
        return torch.where(hz < 1000.0, hz * 3.0 / 200.0,
                           15.0 + torch.log(hz.clamp(min=1000.0) / 1000.0) * 27.0 / math.log(6.4))

    def to_hz(mel):
        return torch.where(mel < 15.0, mel * 200.0 / 3.0, 1000.0 * torch.exp((mel - 15.0) * math.log(6.4) / 27.0))

    nyq = torch.tensor(sample_rate / 2, dtype=torch.float64)
    edges = to_hz(torch.linspace(0.0, float(to_mel(nyq)), num_bands + 2, dtype=torch.float64))
    bins = torch.linspace(0.0, sample_rate / 2, n_fft // 2 + 1, dtype=torch.float64)
    lo, mid, hi = edges[:-2, None], edges[1:-1, None], edges[2:, None]
    tri = torch.minimum((bins - lo) / (mid - lo), (hi - bins) / (hi - mid))
    sup = tri > 0
    sup[0, 0] = True
    sup[-1, -1] = True
    return sup


@torch.no_grad()
def melband_forward(sd: dict, mix: torch.Tensor, cfg: dict, complement: bool = False,
                    match_length: bool = False) -> torch.Tensor:
    """``MelBandRoformer.forward`` (unblend/roformer.py:1513-1603) in fp32 on the CPU.

    Overlapping mel bands gather their bins (index_select), every axial
    transformer ends with an RMSNorm, the mask MLPs have
    ``mask_estimator_depth`` hidden layers, and the band masks are scatter-summed
    onto the bins and divided by each bin's band count.
    """
    cfg = {"stft_normalized": False, "stft_win_length": cfg["stft_n_fft"], **cfg}
    sd = {k: v.float().cpu() for k, v in sd.items()}
    mix = mix.float().cpu()
    batch, channels, length = mix.shape
    heads, dim = cfg["heads"], cfg["dim"]
    zr, _ = stft_features(mix, cfg)
    n_bins, n_frames = zr.shape[1], zr.shape[2]
    sup = mel_supports(cfg.get("sample_rate", 44100), cfg["stft_n_fft"], cfg["num_bands"])
    idx = torch.cat([torch.nonzero(row)[:, 0] for row in sup])
    if channels == 2:
        idx = (idx[:, None] * 2 + torch.arange(2)).reshape(-1)
    per_band = sup.sum(dim=1).tolist()
    x = zr.index_select(1, idx).permute(0, 2, 1, 3).reshape(batch, n_frames, -1)
    widths = [2 * f * channels for f in per_band]
    outs, start = [], 0
    for b, w in enumerate(widths):
        xb = rms_norm(x[..., start : start + w], sd[f"band_split.to_features.{b}.0.gamma"])
        outs.append(F.linear(xb, sd[f"band_split.to_features.{b}.1.weight"],
                             sd[f"band_split.to_features.{b}.1.bias"]).unsqueeze(-2))
        start += w
    x = torch.cat(outs, dim=-2)
    bands = len(widths)
    for i in range(cfg["depth"]):
        x = x.transpose(1, 2).reshape(batch * bands, n_frames, dim)
        x = rms_norm(transformer(sd, f"layers.{i}.0", x, cfg["time_transformer_depth"], heads),
                     sd[f"layers.{i}.0.norm.gamma"])
        x = x.view(batch, bands, n_frames, dim).transpose(1, 2).reshape(batch * n_frames, bands, dim)
        x = rms_norm(transformer(sd, f"layers.{i}.1", x, cfg["freq_transformer_depth"], heads),
                     sd[f"layers.{i}.1.norm.gamma"])
        x = x.view(batch, n_frames, bands, dim)
    n_linear = cfg.get("mask_estimator_depth", 1) + 1
    stems = cfg.get("num_stems", 1)
    masks = []
    for s in range(stems):
        parts = []
        for b in range(bands):
            h = x[..., b, :]
            for k in range(n_linear):
                p = f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}"
                h = F.linear(h, sd[f"{p}.weight"], sd[f"{p}.bias"])
                if k < n_linear - 1:
                    h = torch.tanh(h)
            parts.append(F.glu(h, dim=-1))
        masks.append(torch.cat(parts, dim=-1))
    m = torch.stack(masks, dim=1).view(batch, stems, n_frames, -1, 2).permute(0, 1, 3, 2, 4)
    summed = torch.zeros(batch, stems, n_bins, n_frames, 2)
    summed.index_add_(2, idx, m.contiguous())
    count = torch.zeros(n_bins).index_add_(0, idx, torch.ones(idx.numel()))
    avg = torch.view_as_complex(summed.contiguous()) / count.view(1, 1, -1, 1)
    out = torch.view_as_complex(zr.contiguous()).unsqueeze(1) * avg
    n_freqs = n_bins // channels
    out = out.view(batch, stems, n_freqs, channels, n_frames).permute(0, 1, 3, 2, 4)
    out = out.reshape(batch * stems * channels, n_freqs, n_frames)
    if cfg.get("zero_dc", True):
        out = out.clone()
        out[:, 0] = 0
    window = torch.hann_window(cfg["stft_win_length"])
    recon = torch.istft(out, n_fft=cfg["stft_n_fft"], hop_length=cfg["stft_hop_length"],
                        win_length=cfg["stft_win_length"], normalized=cfg.get("stft_normalized", False),
                        window=window, return_complex=False, length=length if match_length else None)
    recon = recon.view(batch, stems, channels, -1)
    if complement:
        recon = torch.cat([recon, mix[..., : recon.shape[-1]].unsqueeze(1) - recon], dim=1)
    return recon
