"""Seeded random-init weights and synthetic audio for the separation path.

Checkpoints and datasets are unavailable offline, so every workload runs on
random-init weights and synthetic audio:

* ``htdemucs_state_dict(config, seed)`` reproduces ``torch.manual_seed(seed)``
  followed by ``HTDemucs(**config)`` (unblend/htdemucs.py:58-368) parameter for
  parameter. It instantiates the same ``torch.nn`` parameter owners in the
  same construction order, so the torch RNG is consumed identically, then
  applies the reference's ``rescale_module`` trick (unblend/blocks.py:207-236)
  and the smoothed frequency embedding (unblend/blocks.py:353-403). The result
  is keyed exactly like the reference ``state_dict`` (strict-loadable).
* ``synth_track(seconds, seed)`` generates the stereo 44.1 kHz test signal:
  8 sinusoids per channel (log-uniform 40-8000 Hz, amplitudes U(0.05, 0.3)),
  pink noise at -20 dB and a decaying impulse train at 120 BPM, normalised to
  0.9 peak.
"""

from __future__ import annotations

import math
from collections import OrderedDict

import numpy as np
import torch
from torch import nn

# Architecture configs of the two HTDemucs registry entries
# (unblend/metadata.json "htdemucs" and "htdemucs_6s" -> "config").
_HTDEMUCS_COMMON = dict(
    audio_channels=2,
    samplerate=44100,
    segment=7.8,
    channels=48,
    growth=2,
    nfft=4096,
    cac=True,
    depth=4,
    rewrite=True,
    freq_emb=0.2,
    emb_scale=10,
    emb_smooth=True,
    kernel_size=8,
    stride=4,
    time_stride=2,
    context=1,
    context_enc=0,
    norm_starts=4,
    norm_groups=4,
    dconv_mode=3,
    dconv_depth=2,
    dconv_comp=8,
    dconv_init=1e-3,
    t_layers=5,
    t_hidden_scale=4.0,
    t_heads=8,
    t_layer_scale=True,
    t_gelu=True,
    t_emb="sin",
    t_max_period=10000.0,
    t_weight_pos_embed=1.0,
    t_norm_in=True,
    t_norm_first=True,
    t_norm_out=True,
    t_cross_first=False,
    rescale=0.1,
)

HTDEMUCS_CONFIGS = {
    "htdemucs": dict(
        _HTDEMUCS_COMMON,
        sources=["drums", "bass", "other", "vocals"],
        bottom_channels=512,
    ),
    "htdemucs_6s": dict(
        _HTDEMUCS_COMMON,
        sources=["drums", "bass", "other", "vocals", "guitar", "piano"],
        bottom_channels=0,
    ),
}


def htdemucs_config(name: str = "htdemucs", **overrides) -> dict:
    """Return a copy of a registry HTDemucs config with ``overrides`` applied.

    :param name: ``"htdemucs"`` or ``"htdemucs_6s"``.
    :param overrides: Fields to replace (e.g. a reduced ``channels`` for tests).
    :return: Config dict with the reference constructor's field names.
    """
    cfg = dict(HTDEMUCS_CONFIGS[name])
    cfg.update(overrides)
    cfg["sources"] = list(cfg["sources"])
    return cfg


def _take(prefix: str, module: nn.Module, out: "OrderedDict[str, torch.Tensor]") -> None:
    """Copy every parameter of ``module`` into ``out`` under ``prefix``."""
    for name, p in module.named_parameters():
        out[f"{prefix}.{name}"] = p.detach().clone()


def _dconv(prefix: str, channels: int, cfg: dict, out, convs: list) -> None:
    """DConv parameters (unblend/blocks.py:238-305), construction order."""
    hidden = int(channels / cfg["dconv_comp"])
    for d in range(cfg["dconv_depth"]):
        dil = 2**d
        c1 = nn.Conv1d(channels, hidden, 3, dilation=dil, padding=dil)
        g1 = nn.GroupNorm(1, hidden)
        c2 = nn.Conv1d(hidden, 2 * channels, 1)
        g2 = nn.GroupNorm(1, 2 * channels)
        p = f"{prefix}.dconv.layers.{d}"
        _take(f"{p}.0", c1, out)
        _take(f"{p}.1", g1, out)
        _take(f"{p}.3", c2, out)
        _take(f"{p}.4", g2, out)
        out[f"{p}.6.scale"] = torch.full((channels,), cfg["dconv_init"])
        convs += [f"{p}.0", f"{p}.3"]


def htdemucs_state_dict(cfg: dict, seed: int) -> "OrderedDict[str, torch.Tensor]":
    """Random-init HTDemucs weights identical to ``manual_seed(seed); HTDemucs(**cfg)``.

    Follows the layer construction loop of unblend/htdemucs.py:216-321, the
    rescale pass of unblend/blocks.py:207-236 and the transformer construction
    of unblend/transformer.py:581-643. Only configurations the registry ships
    are supported (all-frequency encoder layers, CaC, no MultiWrap, no norms
    in the encoder/decoder layers, sinusoidal transformer embedding).

    :param cfg: Config from :func:`htdemucs_config`.
    :param seed: Seed given to ``torch.manual_seed``.
    :return: State dict keyed like the reference module.
    """
    if cfg.get("multi_freqs"):
        raise ValueError("MultiWrap configs are not supported")
    if not cfg["cac"] or cfg["norm_starts"] < cfg["depth"] or cfg["t_emb"] != "sin":
        raise ValueError("only the registry HTDemucs variants are supported")
    state: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    conv_keys: list[str] = []
    rng_state = torch.random.get_rng_state()
    torch.manual_seed(seed)
    try:
        K, S = cfg["kernel_size"], cfg["stride"]
        chin = cfg["audio_channels"]
        chin_z = chin * 2
        chout = chout_z = cfg["channels"]
        freqs = cfg["nfft"] // 2
        nsrc = len(cfg["sources"])
        depth = cfg["depth"]
        ctx = cfg["context"]
        for index in range(depth):
            if freqs <= K:
                raise ValueError("configs that reach a single frequency are not supported")
            # Frequency encoder layer: Conv2d (K,1)/(S,1), 1x1 rewrite, DConv.
            p = f"encoder.{index}"
            _take(f"{p}.conv", nn.Conv2d(chin_z, chout_z, [K, 1], [S, 1], [K // 4, 0]), state)
            _take(f"{p}.rewrite", nn.Conv2d(chout_z, 2 * chout_z, 1, 1, 0), state)
            conv_keys += [f"{p}.conv", f"{p}.rewrite"]
            _dconv(p, chout_z, cfg, state, conv_keys)
            # Time encoder layer.
            p = f"tencoder.{index}"
            _take(f"{p}.conv", nn.Conv1d(chin, chout, K, S, K // 4), state)
            _take(f"{p}.rewrite", nn.Conv1d(chout, 2 * chout, 1, 1, 0), state)
            conv_keys += [f"{p}.conv", f"{p}.rewrite"]
            _dconv(p, chout, cfg, state, conv_keys)
            if index == 0:
                chin = cfg["audio_channels"] * nsrc
                chin_z = chin * 2
            # Decoders are inserted at the front, so layer ``index`` lands at
            # position depth-1-index.
            p = f"decoder.{depth - 1 - index}"
            _take(f"{p}.conv_tr", nn.ConvTranspose2d(chout_z, chin_z, [K, 1], [S, 1]), state)
            _take(f"{p}.rewrite", nn.Conv2d(chout_z, 2 * chout_z, 1 + 2 * ctx, 1, ctx), state)
            conv_keys += [f"{p}.conv_tr", f"{p}.rewrite"]
            _dconv(p, chout_z, cfg, state, conv_keys)
            p = f"tdecoder.{depth - 1 - index}"
            _take(f"{p}.conv_tr", nn.ConvTranspose1d(chout, chin, K, S), state)
            _take(f"{p}.rewrite", nn.Conv1d(chout, 2 * chout, 1 + 2 * ctx, 1, ctx), state)
            conv_keys += [f"{p}.conv_tr", f"{p}.rewrite"]
            _dconv(p, chout, cfg, state, conv_keys)
            chin, chin_z = chout, chout_z
            chout = int(cfg["growth"] * chout)
            chout_z = int(cfg["growth"] * chout_z)
            freqs //= S
            if index == 0 and cfg["freq_emb"]:
                emb = nn.Embedding(freqs, chin_z)
                w = emb.weight.data
                if cfg["emb_smooth"]:
                    w = torch.cumsum(w, dim=0)
                    w = w / torch.arange(1, freqs + 1).to(w).sqrt()[:, None]
                state["freq_emb.embedding.weight"] = (w / cfg["emb_scale"]).clone()
        if cfg["rescale"]:
            for key in conv_keys:
                w = state[f"{key}.weight"]
                scale = (w.std() / cfg["rescale"]) ** 0.5
                state[f"{key}.weight"] = w / scale
                state[f"{key}.bias"] = state[f"{key}.bias"] / scale
        dim = cfg["channels"] * cfg["growth"] ** (depth - 1)
        bottom = cfg["bottom_channels"]
        if bottom:
            for name, (a, b) in (
                ("channel_upsampler", (dim, bottom)),
                ("channel_downsampler", (bottom, dim)),
                ("channel_upsampler_t", (dim, bottom)),
                ("channel_downsampler_t", (bottom, dim)),
            ):
                _take(name, nn.Conv1d(a, b, 1), state)
            dim = bottom
        if cfg["t_layers"] > 0:
            hidden = int(dim * cfg["t_hidden_scale"])
            heads = cfg["t_heads"]
            p = "crosstransformer"
            _take(f"{p}.norm_in", nn.LayerNorm(dim), state)
            _take(f"{p}.norm_in_t", nn.LayerNorm(dim), state)
            parity = 1 if cfg["t_cross_first"] else 0
            for idx in range(cfg["t_layers"]):
                for branch in ("layers", "layers_t"):
                    q = f"{p}.{branch}.{idx}"
                    if idx % 2 == parity:
                        layer = nn.TransformerEncoderLayer(
                            dim, heads, hidden, 0.0, batch_first=True, norm_first=True
                        )
                        _take(q, layer, state)
                        state[f"{q}.norm_out.weight"] = torch.ones(dim)
                        state[f"{q}.norm_out.bias"] = torch.zeros(dim)
                    else:
                        _take(f"{q}.cross_attn", nn.MultiheadAttention(dim, heads, batch_first=True), state)
                        _take(f"{q}.linear1", nn.Linear(dim, hidden), state)
                        _take(f"{q}.linear2", nn.Linear(hidden, dim), state)
                        for n in ("norm1", "norm2", "norm3"):
                            _take(f"{q}.{n}", nn.LayerNorm(dim), state)
                        state[f"{q}.norm_out.weight"] = torch.ones(dim)
                        state[f"{q}.norm_out.bias"] = torch.zeros(dim)
                    state[f"{q}.gamma_1.scale"] = torch.full((dim,), 1e-4)
                    state[f"{q}.gamma_2.scale"] = torch.full((dim,), 1e-4)
    finally:
        torch.random.set_rng_state(rng_state)
    return state


# The standard 62-band split of the 1025 bins of a 2048-point STFT
# (unblend/roformer.py:32-40): 24x2, 12x4, 8x12, 8x24, 8x48, 128, 129.
DEFAULT_FREQS_PER_BANDS = (2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8 + (128, 129)

# BS-RoFormer of the configuration measured here: dim 512, depth 12, 8 heads
# of 64, one time and one frequency transformer per depth, n_fft 2048, hop
# 441, 62 bands, mask estimator depth 2, one stem, 8 s segments.
BSROFORMER_CONFIG = dict(
    dim=512,
    depth=12,
    stereo=True,
    num_stems=1,
    time_transformer_depth=1,
    freq_transformer_depth=1,
    freqs_per_bands=DEFAULT_FREQS_PER_BANDS,
    dim_head=64,
    heads=8,
    stft_n_fft=2048,
    stft_hop_length=441,
    stft_win_length=2048,
    stft_normalized=False,
    zero_dc=True,
    mask_estimator_depth=2,
    mlp_expansion_factor=4,
    skip_connection=False,
)


def bsroformer_config(**overrides) -> dict:
    """Copy of the measured BS-RoFormer constructor config with ``overrides`` applied."""
    cfg = dict(BSROFORMER_CONFIG)
    cfg.update(overrides)
    cfg["freqs_per_bands"] = tuple(cfg["freqs_per_bands"])
    return cfg


def bsroformer_state_dict(cfg: dict, seed: int) -> "OrderedDict[str, torch.Tensor]":
    """Random-init BS-RoFormer weights identical to ``manual_seed(seed); BSRoformer(**cfg)``.

    Follows the construction order of ``_RoformerBase._init_common`` and
    ``BSRoformer.__init__`` (unblend/roformer.py:896-1066, 1207-1310): per depth
    a time then a frequency ``Transformer`` of (gated ``Attention``,
    ``FeedForward``) layers, then ``final_norm``, the per-band ``BandSplit``
    projections and the per-stem, per-band ``MaskEstimator`` MLPs. RMSNorm gains
    start at one and the frozen rotary frequencies are deterministic.

    :param cfg: Config from :func:`bsroformer_config`.
    :param seed: Seed given to ``torch.manual_seed``.
    :return: State dict keyed like the reference module.
    """
    if cfg.get("skip_connection") or cfg.get("linear_transformer_depth", 0):
        raise ValueError("skip connections and linear attention are not supported")
    dim, heads, dh = cfg["dim"], cfg["heads"], cfg["dim_head"]
    inner = heads * dh
    channels = 2 if cfg["stereo"] else 1
    state: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    freqs = 1.0 / (10000.0 ** (torch.arange(0, dh, 2)[: dh // 2].float() / dh))
    rng_state = torch.random.get_rng_state()
    torch.manual_seed(seed)
    try:
        for i in range(cfg["depth"]):
            for axis, tdepth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
                for j in range(tdepth):
                    p = f"layers.{i}.{axis}.layers.{j}"
                    state[f"{p}.0.norm.gamma"] = torch.ones(dim)
                    _take(f"{p}.0.to_qkv", nn.Linear(dim, 3 * inner, bias=False), state)
                    _take(f"{p}.0.to_gates", nn.Linear(dim, heads), state)
                    _take(f"{p}.0.to_out.0", nn.Linear(inner, dim, bias=False), state)
                    state[f"{p}.0.rotary_embed.freqs"] = freqs.clone()
                    state[f"{p}.1.net.0.gamma"] = torch.ones(dim)
                    # FeedForward width is 4 * dim (Transformer's ff_mult).
                    _take(f"{p}.1.net.1", nn.Linear(dim, 4 * dim), state)
                    _take(f"{p}.1.net.4", nn.Linear(4 * dim, dim), state)
        state["final_norm.gamma"] = torch.ones(dim)
        dims_in = [2 * f * channels for f in cfg["freqs_per_bands"]]
        for b, d_in in enumerate(dims_in):
            state[f"band_split.to_features.{b}.0.gamma"] = torch.ones(d_in)
            _take(f"band_split.to_features.{b}.1", nn.Linear(d_in, dim), state)
        hidden = dim * cfg["mlp_expansion_factor"]
        for s in range(cfg["num_stems"]):
            for b, d_in in enumerate(dims_in):
                p = f"mask_estimators.{s}.to_freqs.{b}.0"
                layer_dims = [dim] + [hidden] * (cfg["mask_estimator_depth"] - 1) + [2 * d_in]
                for k, (a_in, a_out) in enumerate(zip(layer_dims[:-1], layer_dims[1:])):
                    _take(f"{p}.{2 * k}", nn.Linear(a_in, a_out), state)
    finally:
        torch.random.set_rng_state(rng_state)
    return state


# Mel-Band RoFormer of the registry's ``melband_roformer_kim`` entry
# (unblend/metadata.json): dim 384, depth 6, 60 mel bands, 8 heads of 64,
# n_fft 2048, hop 441, mask estimator depth 2, one stem, 8 s segments.
MELBAND_KIM_CONFIG = dict(
    dim=384,
    depth=6,
    stereo=True,
    num_stems=1,
    time_transformer_depth=1,
    freq_transformer_depth=1,
    num_bands=60,
    dim_head=64,
    heads=8,
    sample_rate=44100,
    stft_n_fft=2048,
    stft_hop_length=441,
    stft_win_length=2048,
    mask_estimator_depth=2,
    mlp_expansion_factor=4,
)

# MelBandRoformer constructor defaults (unblend/roformer.py:1383-1408) for keys the config may omit.
MELBAND_DEFAULTS = dict(
    stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2, linear_transformer_depth=0,
    num_bands=60, dim_head=64, heads=8, attn_dropout=0.1, ff_dropout=0.1, sample_rate=44100, stft_n_fft=2048,
    stft_hop_length=512, stft_win_length=2048, stft_normalized=False, zero_dc=True, mask_estimator_depth=1,
    mlp_expansion_factor=4, skip_connection=False, match_input_audio_length=False,
)


def melband_config(**overrides) -> dict:
    """Copy of the ``melband_roformer_kim`` constructor config with ``overrides`` applied."""
    cfg = dict(MELBAND_KIM_CONFIG)
    cfg.update(overrides)
    return cfg


def _hz_to_slaney_mel(f: np.ndarray) -> np.ndarray:
    """Slaney's auditory-toolbox mel scale: 200/3 Hz per mel below 1 kHz, log steps of ln(6.4)/27 above."""
    f = np.asarray(f, dtype=np.float64)
    lin = f / (200.0 / 3.0)
    log_mel0 = 1000.0 / (200.0 / 3.0)
    with np.errstate(divide="ignore"):
        logp = log_mel0 + np.log(np.maximum(f, 1000.0) / 1000.0) / (math.log(6.4) / 27.0)
    return np.where(f >= 1000.0, logp, lin)


def _slaney_mel_to_hz(m: np.ndarray) -> np.ndarray:
    m = np.asarray(m, dtype=np.float64)
    log_mel0 = 1000.0 / (200.0 / 3.0)
    return np.where(m >= log_mel0, 1000.0 * np.exp((math.log(6.4) / 27.0) * (m - log_mel0)), m * (200.0 / 3.0))


def mel_band_support(sample_rate: int, n_fft: int, num_bands: int) -> np.ndarray:
    """``[num_bands, n_fft//2 + 1]`` bool: which STFT bins each mel band covers.

    The bands are the triangular filters of a Slaney-normalised mel filter
    bank spanning 0 Hz to Nyquist (``num_bands + 2`` mel-spaced edges, float64);
    a bin belongs to a band where the filter weight is positive. As in the
    reference (unblend/roformer.py:1459-1463), the DC bin is forced into the
    first band and the Nyquist bin into the last.
    """
    n_freqs = n_fft // 2 + 1
    fft_freqs = np.linspace(0.0, sample_rate / 2, n_freqs)
    edges = _slaney_mel_to_hz(np.linspace(0.0, float(_hz_to_slaney_mel(sample_rate / 2)), num_bands + 2))
    widths = np.diff(edges)
    ramps = edges[:, None] - fft_freqs[None, :]
    rising = -ramps[:-2] / widths[:-1, None]
    falling = ramps[2:] / widths[1:, None]
    weights = np.maximum(0.0, np.minimum(rising, falling)) * (2.0 / (edges[2:] - edges[:-2]))[:, None]
    support = weights > 0
    support[0, 0] = True
    support[-1, -1] = True
    return support


def mel_band_layout(sample_rate: int, n_fft: int, num_bands: int, stereo: bool = True):
    """Gather indices and coverage counts of the Mel-Band RoFormer band split.

    :return: ``(freq_indices, freqs_per_band, bands_per_freq)``: the bins of
        band 0, band 1, ... concatenated, as indices into the channel-interleaved
        frequency axis ``(f, channel)`` when stereo (unblend/roformer.py:1472-1477);
        the bin count of each band; how many bands cover each bin.
    """
    support = mel_band_support(sample_rate, n_fft, num_bands)
    if not support.any(axis=0).all():
        raise ValueError("every frequency bin must be covered by at least one mel band")
    idx = np.concatenate([np.nonzero(row)[0] for row in support]).astype(np.int64)
    if stereo:
        idx = (idx[:, None] * 2 + np.arange(2)[None, :]).reshape(-1)
    return (torch.from_numpy(idx), torch.from_numpy(support.sum(axis=1)).long(),
            torch.from_numpy(support.sum(axis=0)).long())


def melband_state_dict(cfg: dict, seed: int) -> "OrderedDict[str, torch.Tensor]":
    """Random-init Mel-Band RoFormer weights identical to ``manual_seed(seed); MelBandRoformer(**cfg)``.

    Construction order of ``_RoformerBase._init_common`` and
    ``MelBandRoformer.__init__`` (unblend/roformer.py:896-1066, 1383-1511): per
    depth a time then a frequency ``Transformer`` (gated ``Attention`` and
    ``FeedForward`` layers, then the output RMSNorm), the per-band ``BandSplit``
    projections over the mel bands, and per stem the per-band ``MaskEstimator``
    MLPs with ``mask_estimator_depth`` hidden layers.
    """
    full = dict(MELBAND_DEFAULTS)
    full.update(cfg)
    cfg = full
    if cfg["skip_connection"] or cfg["linear_transformer_depth"]:
        raise ValueError("skip connections and linear attention are not supported")
    dim, heads, dh = cfg["dim"], cfg["heads"], cfg["dim_head"]
    inner = heads * dh
    channels = 2 if cfg["stereo"] else 1
    _, freqs_per_band, _ = mel_band_layout(cfg["sample_rate"], cfg["stft_n_fft"], cfg["num_bands"], cfg["stereo"])
    state: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    freqs = 1.0 / (10000.0 ** (torch.arange(0, dh, 2)[: dh // 2].float() / dh))
    rng_state = torch.random.get_rng_state()
    torch.manual_seed(seed)
    try:
        for i in range(cfg["depth"]):
            for axis, tdepth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
                for j in range(tdepth):
                    p = f"layers.{i}.{axis}.layers.{j}"
                    state[f"{p}.0.norm.gamma"] = torch.ones(dim)
                    _take(f"{p}.0.to_qkv", nn.Linear(dim, 3 * inner, bias=False), state)
                    _take(f"{p}.0.to_gates", nn.Linear(dim, heads), state)
                    _take(f"{p}.0.to_out.0", nn.Linear(inner, dim, bias=False), state)
                    state[f"{p}.0.rotary_embed.freqs"] = freqs.clone()
                    state[f"{p}.1.net.0.gamma"] = torch.ones(dim)
                    _take(f"{p}.1.net.1", nn.Linear(dim, 4 * dim), state)
                    _take(f"{p}.1.net.4", nn.Linear(4 * dim, dim), state)
                state[f"layers.{i}.{axis}.norm.gamma"] = torch.ones(dim)
        dims_in = [2 * int(f) * channels for f in freqs_per_band.tolist()]
        for b, d_in in enumerate(dims_in):
            state[f"band_split.to_features.{b}.0.gamma"] = torch.ones(d_in)
            _take(f"band_split.to_features.{b}.1", nn.Linear(d_in, dim), state)
        hidden = dim * cfg["mlp_expansion_factor"]
        for s in range(cfg["num_stems"]):
            for b, d_in in enumerate(dims_in):
                p = f"mask_estimators.{s}.to_freqs.{b}.0"
                layer_dims = [dim] + [hidden] * cfg["mask_estimator_depth"] + [2 * d_in]
                for k, (a_in, a_out) in enumerate(zip(layer_dims[:-1], layer_dims[1:])):
                    _take(f"{p}.{2 * k}", nn.Linear(a_in, a_out), state)
    finally:
        torch.random.set_rng_state(rng_state)
    return state


# SCNet registry entries (unblend/metadata.json "scnet_small" and "scnet_xl_wide_v5"):
# architecture, sources, samplerate, segment_samples and the constructor config.
SCNET_CONFIGS = {
    "scnet_small": dict(
        architecture="scnet_masked", sources=["drums", "bass", "other", "vocals"], samplerate=44100,
        segment_samples=485100, audio_channels=2, dims=[4, 32, 64, 128], nfft=4096, hop_size=1024, win_size=4096,
        normalized=True, band_SR=[0.175, 0.392, 0.433], band_stride=[1, 4, 16], band_kernel=[3, 4, 16],
        conv_depths=[3, 2, 1], compress=4, conv_kernel=3, num_dplayer=6, expand=1),
    "scnet_xl_wide_v5": dict(
        architecture="scnet", sources=["drums", "bass", "other", "vocals"], samplerate=44100,
        segment_samples=485100, audio_channels=2, dims=[4, 64, 128, 256], nfft=4096, hop_size=1024, win_size=4096,
        normalized=True, band_SR=[0.23, 0.37, 0.4], band_stride=[1, 4, 4], band_kernel=[3, 4, 4],
        conv_depths=[3, 3, 3], compress=4, conv_kernel=3, num_dplayer=8, expand=1),
}


def scnet_config(name: str = "scnet_small", **overrides) -> dict:
    """SCNet registry config (plus ``architecture``, ``sources``, ``samplerate``, ``segment_samples``)."""
    cfg = {k: (list(v) if isinstance(v, list) else v) for k, v in SCNET_CONFIGS[name].items()}
    cfg.update(overrides)
    return cfg


def scnet_state_dict(cfg: dict, seed: int) -> "OrderedDict[str, torch.Tensor]":
    """Random-init SCNet weights identical to ``manual_seed(seed); SCNet(**cfg)`` (or ``SCNetMasked``).

    Follows the construction order of unblend/scnet.py:616-700: for each stage
    the encoder ``SDblock`` (three band convolutions, the per-band
    ``ConvolutionModule`` stacks, the global 3x3 convolution), then that
    stage's decoder (``FusionLayer`` and ``SUlayer``), which the reference
    inserts at the front of its decoder list; then the dual-path trunk (two
    bidirectional LSTMs, two linears and two GroupNorms per layer); for the
    masked architecture (unblend/scnet.py:800-835) the truncated-normal
    frequency embedding and the mask head.
    """
    torch.manual_seed(seed)
    out: "OrderedDict[str, torch.Tensor]" = OrderedDict()
    dims, S = cfg["dims"], len(cfg["sources"])
    kern, stride = cfg["band_kernel"], cfg["band_stride"]
    stages = len(dims) - 1
    for i in range(stages):
        cin, cout = dims[i], dims[i + 1]
        p = f"encoder.{i}"
        for j in range(3):
            _take(f"{p}.SDlayer.convs.{j}", nn.Conv2d(cin, cout, (kern[j], 1), (stride[j], 1), (0, 0)), out)
        hidden = int(cout / cfg["compress"])
        k = cfg["conv_kernel"]
        for j, depth in enumerate(cfg["conv_depths"]):
            for d in range(abs(depth)):
                q = f"{p}.conv_modules.{j}.layers.{d}"
                _take(f"{q}.0", nn.GroupNorm(1, cout), out)
                _take(f"{q}.1", nn.Conv1d(cout, hidden * 2, k, padding=k // 2), out)
                _take(f"{q}.3", nn.Conv1d(hidden, hidden, k, padding=k // 2, groups=hidden), out)
                _take(f"{q}.4", nn.GroupNorm(1, hidden), out)
                _take(f"{q}.6", nn.Conv1d(hidden, cout, 1), out)
        _take(f"{p}.globalconv", nn.Conv2d(cout, cout, 3, 1, 1), out)
        d_idx = stages - 1 - i  # the reference inserts each stage's decoder at the front
        _take(f"decoder.{d_idx}.0.conv", nn.Conv2d(cout * 2, cout * 2, 3, stride=1, padding=1), out)
        dec_out = cin if i != 0 else cin * S
        for j in range(3):
            _take(f"decoder.{d_idx}.1.convtrs.{j}", nn.ConvTranspose2d(cout, dec_out, [kern[j], 1], [stride[j], 1]),
                  out)
    c = dims[-1]
    for i in range(cfg["num_dplayer"]):
        d_model = c * (2 if i % 2 == 1 else 1)
        hid = d_model * cfg["expand"]
        q = f"separation_net.dp_modules.{i}"
        for j in range(2):
            _take(f"{q}.lstm_layers.{j}", nn.LSTM(d_model, hid, num_layers=1, bidirectional=True), out)
        for j in range(2):
            _take(f"{q}.linear_layers.{j}", nn.Linear(hid * 2, d_model), out)
        for j in range(2):
            _take(f"{q}.norm_layers.{j}", nn.GroupNorm(1, d_model), out)
    if cfg.get("architecture") == "scnet_masked":
        pos = torch.zeros(1, dims[0], cfg["nfft"] // 2 + 1, 1)
        nn.init.trunc_normal_(pos, std=0.02)
        out["pos_embed_f"] = pos
        _take("mask_layer.0", nn.Conv2d(4 * S, 64, kernel_size=3, padding="same"), out)
        _take("mask_layer.2", nn.Conv2d(64, 4 * S, kernel_size=1, padding="same"), out)
    return out


def synth_track(seconds: float, seed: int, samplerate: int = 44100) -> torch.Tensor:
    """Synthetic stereo mixture ``[2, round(seconds * samplerate)]`` in fp32.

    Per channel: 8 sinusoids with log-uniform frequencies over 40-8000 Hz and
    amplitudes U(0.05, 0.3), pink noise at -20 dB relative to the sinusoid RMS,
    and a decaying impulse train at 120 BPM; the mix is normalised to 0.9 peak.

    :param seconds: Duration in seconds.
    :param seed: Generator seed.
    :param samplerate: Sample rate in Hz.
    :return: ``[2, samples]`` float32 tensor.
    """
    rng = np.random.default_rng(seed)
    n = int(round(seconds * samplerate))
    t = np.arange(n, dtype=np.float64) / samplerate
    out = np.zeros((2, n), dtype=np.float64)
    for ch in range(2):
        freqs = np.exp(rng.uniform(math.log(40.0), math.log(8000.0), 8))
        amps = rng.uniform(0.05, 0.3, 8)
        phases = rng.uniform(0, 2 * math.pi, 8)
        tone = np.zeros(n)
        for f, a, ph in zip(freqs, amps, phases):
            tone += a * np.sin(2 * math.pi * f * t + ph)
        # Pink noise: white noise shaped by 1/sqrt(f) in the frequency domain.
        white = rng.standard_normal(n)
        spec = np.fft.rfft(white)
        k = np.arange(spec.shape[0], dtype=np.float64)
        k[0] = 1.0
        pink = np.fft.irfft(spec / np.sqrt(k), n=n)
        tone_rms = np.sqrt(np.mean(tone**2)) + 1e-12
        pink *= (tone_rms * 10 ** (-20 / 20)) / (np.sqrt(np.mean(pink**2)) + 1e-12)
        # Impulse train: one click per beat at 120 BPM with exponential decay.
        clicks = np.zeros(n)
        beat = int(samplerate * 60 / 120)
        decay = np.exp(-np.arange(min(beat, 4410)) / (0.01 * samplerate))
        for start in range(0, n, beat):
            seg = decay[: n - start]
            clicks[start : start + seg.shape[0]] += 0.5 * seg * rng.uniform(0.5, 1.0)
        out[ch] = tone + pink + clicks
    peak = np.abs(out).max()
    if peak > 0:
        out *= 0.9 / peak
    return torch.from_numpy(out.astype(np.float32))
