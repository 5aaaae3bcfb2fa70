"""Functional fp32 restatement of ``HTDemucs.forward`` (CPU oracle, test use only).

Every step cites the reference function it restates. Inputs are a reference
layout ``state_dict`` (strict keys of unblend/htdemucs.py's module tree) and the
constructor config. The arithmetic is plain torch on the CPU in float32.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _spec(x: torch.Tensor, nfft: int) -> torch.Tensor:
    """``HTDemucs._spec`` (unblend/htdemucs.py:370-395) + ``spectro`` (unblend/blocks.py:60-88)."""
    hl = nfft // 4
    le = int(math.ceil(x.shape[-1] / hl))
    pad = hl // 2 * 3
    x = F.pad(x, (pad, pad + le * hl - x.shape[-1]), mode="reflect")
    *other, length = x.shape
    z = torch.stft(
        x.reshape(-1, length), nfft, hl, window=torch.hann_window(nfft), win_length=nfft,
        normalized=True, center=True, return_complex=True, pad_mode="reflect",
    )
    z = z.view(*other, z.shape[-2], z.shape[-1])[..., :-1, :]
    return z[..., 2 : 2 + le]


def _ispec(z: torch.Tensor, length: int, nfft: int) -> torch.Tensor:
    """``HTDemucs._ispec`` (unblend/htdemucs.py:397-412) + ``ispectro`` (unblend/blocks.py:165-204)."""
    hl = nfft // 4
    z = F.pad(z, (0, 0, 0, 1))
    z = F.pad(z, (2, 2))
    pad = hl // 2 * 3
    le = hl * int(math.ceil(length / hl)) + 2 * pad
    *other, freqs, frames = z.shape
    x = torch.istft(
        z.reshape(-1, freqs, frames), nfft, hl, window=torch.hann_window(nfft),
        win_length=nfft, normalized=True, length=le, center=True,
    )
    x = x.view(*other, x.shape[-1])
    return x[..., pad : pad + length]


def _dconv(sd: dict, p: str, x: torch.Tensor, depth: int) -> torch.Tensor:
    """``DConv.forward`` (unblend/blocks.py:238-317): x += LS(GLU(GN(1x1(GELU(GN(conv_k3_dil(x)))))))."""
    for d in range(depth):
        q = f"{p}.dconv.layers.{d}"
        dil = 2**d
        y = F.conv1d(x, sd[f"{q}.0.weight"], sd[f"{q}.0.bias"], padding=dil, dilation=dil)
        y = F.gelu(F.group_norm(y, 1, sd[f"{q}.1.weight"], sd[f"{q}.1.bias"], eps=1e-5))
        y = F.conv1d(y, sd[f"{q}.3.weight"], sd[f"{q}.3.bias"])
        y = F.group_norm(y, 1, sd[f"{q}.4.weight"], sd[f"{q}.4.bias"], eps=1e-5)
        y = F.glu(y, dim=1)
        x = x + sd[f"{q}.6.scale"][:, None] * y
    return x


def _dconv_freq(sd: dict, p: str, y: torch.Tensor, depth: int) -> torch.Tensor:
    """DConv over ``[B*Fr, C, T]`` rows of a frequency-branch tensor (unblend/blocks.py:500-506)."""
    B, C, Fr, T = y.shape
    y = y.permute(0, 2, 1, 3).reshape(-1, C, T)
    y = _dconv(sd, p, y, depth)
    return y.view(B, Fr, C, T).permute(0, 2, 1, 3)


def _henc(sd: dict, p: str, x: torch.Tensor, freq: bool, cfg: dict) -> torch.Tensor:
    """``HEncLayer.forward`` (unblend/blocks.py:474-511), norms are Identity at these configs."""
    K, S = cfg["kernel_size"], cfg["stride"]
    if freq:
        y = F.conv2d(x, sd[f"{p}.conv.weight"], sd[f"{p}.conv.bias"], (S, 1), (K // 4, 0))
    else:
        le = x.shape[-1]
        if le % S:
            x = F.pad(x, (0, S - le % S))
        y = F.conv1d(x, sd[f"{p}.conv.weight"], sd[f"{p}.conv.bias"], S, K // 4)
    y = F.gelu(y)
    y = _dconv_freq(sd, p, y, cfg["dconv_depth"]) if freq else _dconv(sd, p, y, cfg["dconv_depth"])
    conv = F.conv2d if freq else F.conv1d
    z = conv(y, sd[f"{p}.rewrite.weight"], sd[f"{p}.rewrite.bias"])
    return F.glu(z, dim=1)


def _hdec(sd: dict, p: str, x: torch.Tensor, skip: torch.Tensor, length: int, freq: bool,
          last: bool, cfg: dict) -> torch.Tensor:
    """``HDecLayer.forward`` (unblend/blocks.py:706-747)."""
    K, S = cfg["kernel_size"], cfg["stride"]
    pad = K // 4
    ctx = cfg["context"]
    x = x + skip
    conv = F.conv2d if freq else F.conv1d
    y = F.glu(conv(x, sd[f"{p}.rewrite.weight"], sd[f"{p}.rewrite.bias"], 1, ctx), dim=1)
    y = _dconv_freq(sd, p, y, cfg["dconv_depth"]) if freq else _dconv(sd, p, y, cfg["dconv_depth"])
    if freq:
        z = F.conv_transpose2d(y, sd[f"{p}.conv_tr.weight"], sd[f"{p}.conv_tr.bias"], (S, 1))
        z = z[..., pad:-pad, :]
    else:
        z = F.conv_transpose1d(y, sd[f"{p}.conv_tr.weight"], sd[f"{p}.conv_tr.bias"], S)
        z = z[..., pad : pad + length]
    if not last:
        z = F.gelu(z)
    return z


def sin_embedding(length: int, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """``create_sin_embedding`` (unblend/transformer.py:18-48) as ``[length, dim]``."""
    pos = torch.arange(length, dtype=torch.float32).view(-1, 1)
    half = dim // 2
    adim = torch.arange(half, dtype=torch.float32).view(1, -1)
    phase = pos / (max_period ** (adim / (half - 1)))
    return torch.cat([torch.cos(phase), torch.sin(phase)], dim=-1)


def sin_embedding_2d(d_model: int, height: int, width: int, max_period: float = 10000.0) -> torch.Tensor:
    """``create_2d_sin_embedding`` (unblend/transformer.py:51-107) as ``[d_model, height, width]``."""
    pe = torch.zeros(d_model, height, width)
    half = d_model // 2
    div = torch.exp(torch.arange(0.0, half, 2) * -(math.log(max_period) / half))
    pos_w = torch.arange(0.0, width).unsqueeze(1)
    pos_h = torch.arange(0.0, height).unsqueeze(1)
    pe[0:half:2] = torch.sin(pos_w * div).t().unsqueeze(1).repeat(1, height, 1)
    pe[1:half:2] = torch.cos(pos_w * div).t().unsqueeze(1).repeat(1, height, 1)
    pe[half::2] = torch.sin(pos_h * div).t().unsqueeze(2).repeat(1, 1, width)
    pe[half + 1 :: 2] = torch.cos(pos_h * div).t().unsqueeze(2).repeat(1, 1, width)
    return pe


def _mha(sd: dict, p: str, q: torch.Tensor, kv: torch.Tensor, heads: int) -> torch.Tensor:
    """``nn.MultiheadAttention`` forward (batch_first, no mask, eval)."""
    w, b = sd[f"{p}.in_proj_weight"], sd[f"{p}.in_proj_bias"]
    d = q.shape[-1]
    Q = F.linear(q, w[:d], b[:d])
    Kt = F.linear(kv, w[d : 2 * d], b[d : 2 * d])
    V = F.linear(kv, w[2 * d :], b[2 * d :])
    B, Lq, _ = Q.shape
    Lk = Kt.shape[1]
    hd = d // heads
    Q = Q.view(B, Lq, heads, hd).transpose(1, 2)
    Kt = Kt.view(B, Lk, heads, hd).transpose(1, 2)
    V = V.view(B, Lk, heads, hd).transpose(1, 2)
    # softmax(Q K^T / sqrt(hd)) V, through torch's fused CPU kernel for that product (the
    # reference's own eval fast path reaches the same kernel).
    o = F.scaled_dot_product_attention(Q, Kt, V, scale=1.0 / math.sqrt(hd)).transpose(1, 2).reshape(B, Lq, d)
    return F.linear(o, sd[f"{p}.out_proj.weight"], sd[f"{p}.out_proj.bias"])


def _ffn(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    """Feed-forward block: linear2(gelu(linear1(x))) (unblend/transformer.py:507-515)."""
    h = F.gelu(F.linear(x, sd[f"{p}.linear1.weight"], sd[f"{p}.linear1.bias"]))
    return F.linear(h, sd[f"{p}.linear2.weight"], sd[f"{p}.linear2.bias"])


def _ln(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), sd[f"{p}.weight"], sd[f"{p}.bias"], 1e-5)


def _norm_out(sd: dict, p: str, x: torch.Tensor) -> torch.Tensor:
    """``MyGroupNorm(1, C)`` over ``[B, T, C]`` (unblend/transformer.py:225-236)."""
    y = F.group_norm(x.transpose(1, 2), 1, sd[f"{p}.norm_out.weight"], sd[f"{p}.norm_out.bias"], 1e-5)
    return y.transpose(1, 2)


def _self_layer(sd: dict, p: str, x: torch.Tensor, heads: int) -> torch.Tensor:
    """``MyTransformerEncoderLayer.forward`` with norm_first and norm_out (unblend/transformer.py:328-359)."""
    h = _ln(sd, f"{p}.norm1", x)
    x = x + sd[f"{p}.gamma_1.scale"] * _mha(sd, f"{p}.self_attn", h, h, heads)
    x = x + sd[f"{p}.gamma_2.scale"] * _ffn(sd, p, _ln(sd, f"{p}.norm2", x))
    return _norm_out(sd, p, x)


def _cross_layer(sd: dict, p: str, q: torch.Tensor, k: torch.Tensor, heads: int) -> torch.Tensor:
    """``CrossTransformerEncoderLayer.forward`` with norm_first and norm_out (unblend/transformer.py:461-481)."""
    kk = _ln(sd, f"{p}.norm2", k)
    x = q + sd[f"{p}.gamma_1.scale"] * _mha(sd, f"{p}.cross_attn", _ln(sd, f"{p}.norm1", q), kk, heads)
    x = x + sd[f"{p}.gamma_2.scale"] * _ffn(sd, p, _ln(sd, f"{p}.norm3", x))
    return _norm_out(sd, p, x)


def _crosstransformer(sd: dict, x: torch.Tensor, xt: torch.Tensor, cfg: dict):
    """``CrossTransformerEncoder.forward`` (unblend/transformer.py:703-742)."""
    p = "crosstransformer"
    heads = cfg["t_heads"]
    B, C, Fr, T1 = x.shape
    pos2 = sin_embedding_2d(C, Fr, T1, cfg["t_max_period"]).permute(2, 1, 0).reshape(1, T1 * Fr, C)
    x = x.permute(0, 3, 2, 1).reshape(B, T1 * Fr, C)
    x = _ln(sd, f"{p}.norm_in", x) + cfg["t_weight_pos_embed"] * pos2
    _, _, T2 = xt.shape
    xt = xt.permute(0, 2, 1)
    pos1 = sin_embedding(T2, C, cfg["t_max_period"])[None]
    xt = _ln(sd, f"{p}.norm_in_t", xt) + cfg["t_weight_pos_embed"] * pos1
    parity = 1 if cfg["t_cross_first"] else 0
    for idx in range(cfg["t_layers"]):
        if idx % 2 == parity:
            x = _self_layer(sd, f"{p}.layers.{idx}", x, heads)
            xt = _self_layer(sd, f"{p}.layers_t.{idx}", xt, heads)
        else:
            old_x = x
            x = _cross_layer(sd, f"{p}.layers.{idx}", x, xt, heads)
            xt = _cross_layer(sd, f"{p}.layers_t.{idx}", xt, old_x, heads)
    x = x.reshape(B, T1, Fr, C).permute(0, 3, 2, 1)
    return x, xt.permute(0, 2, 1)


def forward_core(sd: dict, x: torch.Tensor, xt: torch.Tensor, cfg: dict):
    """``HTDemucs.forward_core`` (unblend/htdemucs.py:585-648)."""
    depth = cfg["depth"]
    saved, saved_t, lengths, lengths_t = [], [], [], []
    for idx in range(depth):
        lengths.append(x.shape[-1])
        lengths_t.append(xt.shape[-1])
        xt = _henc(sd, f"tencoder.{idx}", xt, False, cfg)
        saved_t.append(xt)
        x = _henc(sd, f"encoder.{idx}", x, True, cfg)
        if idx == 0 and cfg["freq_emb"]:
            emb = (sd["freq_emb.embedding.weight"] * cfg["emb_scale"]).t()[None, :, :, None]
            x = x + cfg["freq_emb"] * emb
        saved.append(x)
    if cfg["t_layers"] > 0:
        bottom = cfg["bottom_channels"]
        if bottom:
            b, c, f, t = x.shape
            x = F.conv1d(x.flatten(2), sd["channel_upsampler.weight"], sd["channel_upsampler.bias"])
            x = x.view(b, -1, f, t)
            xt = F.conv1d(xt, sd["channel_upsampler_t.weight"], sd["channel_upsampler_t.bias"])
        x, xt = _crosstransformer(sd, x, xt, cfg)
        if bottom:
            x = F.conv1d(x.flatten(2), sd["channel_downsampler.weight"], sd["channel_downsampler.bias"])
            x = x.view(b, -1, f, t)
            xt = F.conv1d(xt, sd["channel_downsampler_t.weight"], sd["channel_downsampler_t.bias"])
    for idx in range(depth):
        last = idx == depth - 1
        x = _hdec(sd, f"decoder.{idx}", x, saved.pop(-1), lengths.pop(-1), True, last, cfg)
        xt = _hdec(sd, f"tdecoder.{idx}", xt, saved_t.pop(-1), lengths_t.pop(-1), False, last, cfg)
    return x, xt


def normalize_inputs(mix: torch.Tensor, cfg: dict):
    """Spectrogram + per-segment normalisation of both branches (unblend/htdemucs.py:660-678).

    :return: ``(x, xt, (mean, std), (meant, stdt), Fq, T)``.
    """
    z = _spec(mix, cfg["nfft"])
    B, C, Fr, T = z.shape
    x = torch.view_as_real(z).permute(0, 1, 4, 2, 3).reshape(B, C * 2, Fr, T)
    var, mean = torch.var_mean(x, dim=(1, 2, 3), keepdim=True)
    std = torch.sqrt(var)
    x = (x - mean) / (1e-5 + std)
    var_t, meant = torch.var_mean(mix, dim=(1, 2), keepdim=True)
    stdt = torch.sqrt(var_t)
    xt = (mix - meant) / (1e-5 + stdt)
    return x, xt, (mean, std), (meant, stdt)


def segment_length(cfg: dict) -> int:
    """Training length in samples (``HTDemucs.valid_length``, unblend/htdemucs.py:450-467)."""
    return int(round(cfg["segment"] * cfg["samplerate"]))


@torch.no_grad()
def htdemucs_forward(sd: dict, mix: torch.Tensor, cfg: dict) -> torch.Tensor:
    """``HTDemucs.forward`` (unblend/htdemucs.py:650-704) in fp32 on the CPU.

    :param sd: Reference-layout state dict (float32 CPU tensors).
    :param mix: ``[B, C, L]`` with ``L <= segment length``.
    :param cfg: HTDemucs config.
    :return: ``[B, S, C, L]`` separated sources.
    """
    sd = {k: v.float().cpu() for k, v in sd.items()}
    mix = mix.float().cpu()
    T = segment_length(cfg)
    if mix.shape[-1] > T:
        raise ValueError(f"Given length {mix.shape[-1]} is longer than training length {T}")
    length_pre_pad = mix.shape[-1] if mix.shape[-1] < T else None
    if length_pre_pad:
        mix = F.pad(mix, (0, T - length_pre_pad))
    x, xt, (mean, std), (meant, stdt) = normalize_inputs(mix, cfg)
    B, _, Fq, Tf = x.shape
    x, xt = forward_core(sd, x, xt, cfg)
    S = len(cfg["sources"])
    x = x.view(B, S, -1, Fq, Tf) * std[:, None] + mean[:, None]
    x = x.view(B, S, -1, 2, Fq, Tf).permute(0, 1, 2, 4, 5, 3)
    zout = torch.view_as_complex(x.contiguous())
    x = _ispec(zout, T, cfg["nfft"])
    xt = xt.view(B, S, -1, T) * stdt[:, None] + meant[:, None]
    out = xt + x
    if length_pre_pad:
        out = out[..., :length_pre_pad]
    return out
