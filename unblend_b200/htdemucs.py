"""HTDemucs forward on B200: the drop-in model behind ``apply_model``.

``HTDemucsCuda`` keeps the model contract that the reference segment engine
drives (unblend/backends.py:36-59; unblend/apply.py:1201-1202): ``sources``,
``samplerate``, ``audio_channels``, ``max_allowed_segment``,
``_fixed_batch_shape`` and ``forward(mix[B, C, T]) -> [B, S, C, T]``. It is built
from the reference ``state_dict`` (strict keys, unblend/repo.py:138) and its
constructor config, repacks the weights once into kernel layouts on the device,
and runs every step of ``HTDemucs.forward`` (unblend/htdemucs.py:650-704) as
CUDA kernels of ``libunblend_b200.so`` through its C ABI. There is no CPU
path: ``forward`` raises unless its input and weights are on a CUDA device.

Activations are channels-last: the frequency branch is ``[B, F, T, C]`` (T = STFT
frames), the time branch ``[B, rows, C]`` where each level's buffers hold
``4 * ceil(L / 4)`` rows so that encoder outputs and transposed-conv outputs of
a level share one batch stride. Transformer tokens of the frequency branch are
ordered (f, t); the 2-D positional table is laid out to match.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from . import _lib
from ._lib import ACT_GELU, ACT_GLU, ACT_NONE, PRO_ADD, PRO_GN_GELU, PRO_NONE, AttnParams
from .apply import ValidationError
from .convnet import (PRECISIONS, Act, ConvNet, StatsArena, _block_n, _conv_w, _interleave_rows, _key,  # noqa: F401
                      ctypes_byref, split_tf32)
from .synth import HTDEMUCS_CONFIGS


def _moment_width(hid: int) -> int:
    """Hidden width the fused DConv kernels compute with: the true width when even, else rounded up to 4."""
    return hid if hid % 2 == 0 else -(-hid // 4) * 4


def sin_embedding(length: int, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """1-D sinusoidal table ``[length, dim]`` (cos | sin halves), as unblend/transformer.py:18-48."""
    pos = torch.arange(length, dtype=torch.float32).view(-1, 1)
    half = dim // 2
    adim = torch.arange(half, dtype=torch.float32).view(1, -1)
    phase = pos / (max_period ** (adim / (half - 1)))
    return torch.cat([torch.cos(phase), torch.sin(phase)], dim=-1)


def sin_embedding_2d(d_model: int, height: int, width: int, max_period: float = 10000.0) -> torch.Tensor:
    """2-D sinusoidal table ``[d_model, height, width]``, as unblend/transformer.py:51-107."""
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


def _convtr_taps3(w: torch.Tensor) -> torch.Tensor:
    """A stride-4, kernel-8 transposed conv as one 3-tap conv with 4 output phases.

    ``w`` is [Cin, Cout, 8] (or [Cin, Cout, 8, 1]). After the pad-2 crop, output
    row 4p+s receives X[p-1]W[6] + X[p]W[2] (s=0), X[p-1]W[7] + X[p]W[3] (s=1),
    X[p]W[4] + X[p+1]W[0] (s=2), X[p]W[5] + X[p+1]W[1] (s=3). The returned weight
    is [4*Cout, 3 taps (p-1, p, p+1), Cin] with rows ordered (s, cout) and the
    unused tap of each phase zero, so one launch reads every input row once and
    writes all four output rows (channel group s at output row offset s).
    """
    if w.dim() == 4:
        w = w[..., 0]
    wk = w.permute(2, 1, 0)  # [8, Cout, Cin]
    z = torch.zeros_like(wk[0])
    phases = [(wk[6], wk[2], z), (wk[7], wk[3], z), (z, wk[4], wk[0]), (z, wk[5], wk[1])]
    return torch.stack([torch.stack(t, 1) for t in phases], 0).reshape(-1, 3, w.shape[0]).contiguous()


class HTDemucsCuda(ConvNet):
    """HTDemucs separation forward as sm_100a CUDA kernels.

    :param config: HTDemucs constructor config (registry ``config`` fields).
    :param state_dict: Reference-layout weights (strict key set).
    :param precision: ``"fp32"`` (dense layers on tcgen05 tensor cores with the
        3-pass TF32 split, fp32-level accuracy), ``"bf16"`` (bf16 tensor-core
        operands, fp32 accumulation and fp32 activations) or ``"fp32-simt"``
        (every layer on CUDA-core fp32 FMA kernels).
    """

    #: The Separator normalises the track before ``apply_model`` and restores it after
    #: (unblend/api.py:1644, 1706); the RoFormers set this False.
    external_normalization = True

    def __init__(self, config: dict, state_dict: dict, precision: str = "fp32") -> None:
        super().__init__(precision)
        cfg = dict(HTDEMUCS_CONFIGS["htdemucs"])
        cfg.update(config)
        if cfg.get("multi_freqs") or not cfg["cac"] or cfg["norm_starts"] < cfg["depth"]:
            raise ValueError("unsupported HTDemucs variant")
        if cfg["nfft"] != 4096 or cfg["kernel_size"] != 8 or cfg["stride"] != 4 or cfg["t_emb"] != "sin":
            raise ValueError("unsupported HTDemucs geometry")
        self.config = cfg
        # Operand split of the fp32 tensor-core attention: "bf16x3" (kind::f16, 16 dims
        # or keys per MMA) or "tf32x3" (kind::tf32, 8 per MMA).
        self.attention_split = "bf16x3"
        self.sources = list(cfg["sources"])
        self.samplerate = cfg["samplerate"]
        self.audio_channels = cfg["audio_channels"]
        self.max_allowed_segment = cfg["segment"]
        self.segment_length = int(round(cfg["segment"] * cfg["samplerate"]))
        self._fixed_batch_shape = False
        self._eager_tails = False
        self.depth = cfg["depth"]
        self._pack(state_dict)

    @classmethod
    def from_reference(cls, module: nn.Module, precision: str = "fp32") -> "HTDemucsCuda":
        """Build from a reference ``HTDemucs`` instance (its captured init kwargs + state_dict)."""
        args, kwargs = getattr(module, "_init_args_kwargs", ((), {}))
        cfg = dict(kwargs)
        if args:
            cfg["sources"] = args[0]
        return cls(cfg, module.state_dict(), precision=precision)

    # ------------------------------------------------------------------ weights
    def _pack(self, sd: dict) -> None:
        sd = {k: v.detach().float().cpu() for k, v in sd.items()}
        cfg = self.config
        for idx in range(self.depth):
            for pre in (f"encoder.{idx}", f"tencoder.{idx}"):
                self._put(f"{pre}.conv.w", _conv_w(sd[f"{pre}.conv.weight"]))
                self._put(f"{pre}.conv.b", sd[f"{pre}.conv.bias"])
                self._put(f"{pre}.rewrite.w", _interleave_rows(_conv_w(sd[f"{pre}.rewrite.weight"])))
                self._put(f"{pre}.rewrite.b", _interleave_rows(sd[f"{pre}.rewrite.bias"]))
                self._pack_dconv(sd, pre)
            for pre in (f"decoder.{idx}", f"tdecoder.{idx}"):
                self._put(f"{pre}.rewrite.w", _interleave_rows(_conv_w(sd[f"{pre}.rewrite.weight"])))
                self._put(f"{pre}.rewrite.b", _interleave_rows(sd[f"{pre}.rewrite.bias"]))
                self._put(f"{pre}.convtr.w", _convtr_taps3(sd[f"{pre}.conv_tr.weight"]))
                self._put(f"{pre}.convtr.b", sd[f"{pre}.conv_tr.bias"].repeat(4))
                self._pack_dconv(sd, pre)
        if cfg["freq_emb"]:
            self._put("freq_emb", sd["freq_emb.embedding.weight"] * cfg["emb_scale"] * cfg["freq_emb"])
        self.bottom = cfg["bottom_channels"]
        if self.bottom:
            for n in ("channel_upsampler", "channel_downsampler", "channel_upsampler_t", "channel_downsampler_t"):
                self._put(f"{n}.w", sd[f"{n}.weight"][..., 0])
                self._put(f"{n}.b", sd[f"{n}.bias"])
        p = "crosstransformer"
        self.t_layers = cfg["t_layers"]
        if self.t_layers:
            for n in ("norm_in", "norm_in_t"):
                self._put(f"{p}.{n}.weight", sd[f"{p}.{n}.weight"])
                self._put(f"{p}.{n}.bias", sd[f"{p}.{n}.bias"])
            parity = 1 if cfg["t_cross_first"] else 0
            for idx in range(self.t_layers):
                for br in ("layers", "layers_t"):
                    q = f"{p}.{br}.{idx}"
                    attn = "self_attn" if idx % 2 == parity else "cross_attn"
                    for k in (f"{attn}.in_proj_weight", f"{attn}.in_proj_bias", f"{attn}.out_proj.weight",
                              f"{attn}.out_proj.bias", "linear1.weight", "linear1.bias", "linear2.weight",
                              "linear2.bias", "norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias",
                              "norm_out.weight", "norm_out.bias", "gamma_1.scale", "gamma_2.scale"):
                        self._put(f"{q}.{k}", sd[f"{q}.{k}"])
                    if idx % 2 != parity:
                        self._put(f"{q}.norm3.weight", sd[f"{q}.norm3.weight"])
                        self._put(f"{q}.norm3.bias", sd[f"{q}.norm3.bias"])
                        # Query and key/value projections of the cross attention, split once.
                        win, bin_ = sd[f"{q}.cross_attn.in_proj_weight"], sd[f"{q}.cross_attn.in_proj_bias"]
                        d = win.shape[1]
                        self._put(f"{q}.in_q.w", win[:d])
                        self._put(f"{q}.in_q.b", bin_[:d])
                        self._put(f"{q}.in_kv.w", win[d:])
                        self._put(f"{q}.in_kv.b", bin_[d:])
        self.window = None

    def _pack_dconv(self, sd: dict, pre: str) -> None:
        for d in range(self.config["dconv_depth"]):
            q = f"{pre}.dconv.layers.{d}"
            self._put(f"{q}.c1.w", _conv_w(sd[f"{q}.0.weight"]))
            self._put(f"{q}.c1.b", sd[f"{q}.0.bias"])
            self._put(f"{q}.g1.w", sd[f"{q}.1.weight"])
            self._put(f"{q}.g1.b", sd[f"{q}.1.bias"])
            self._put(f"{q}.c2.w", _interleave_rows(_conv_w(sd[f"{q}.3.weight"])))
            self._put(f"{q}.c2.b", _interleave_rows(sd[f"{q}.3.bias"]))
            self._put(f"{q}.g2.w", _interleave_rows(sd[f"{q}.4.weight"]))
            self._put(f"{q}.g2.b", _interleave_rows(sd[f"{q}.4.bias"]))
            self._put(f"{q}.scale", sd[f"{q}.6.scale"])
            self._put_moment_coef(q, sd[f"{q}.3.weight"], sd[f"{q}.3.bias"])
            # Hidden width padded to a multiple of 4 with zero channels (16-byte h
            # rows for the bulk copies of the fused kernels): the padded channels
            # are exactly 0 before and after GELU(GN1) and meet zero weights in W2.
            hid = sd[f"{q}.0.weight"].shape[0]
            hp = -(-hid // 4) * 4
            if hp != hid:
                pad = hp - hid
                c1 = _conv_w(sd[f"{q}.0.weight"])
                self._put(f"{q}.c1p.w", torch.cat([c1, c1.new_zeros((pad,) + tuple(c1.shape[1:]))]))
                self._put(f"{q}.c1p.b", torch.cat([sd[f"{q}.0.bias"], sd[f"{q}.0.bias"].new_zeros(pad)]))
                self._put(f"{q}.g1p.w", torch.cat([sd[f"{q}.1.weight"], sd[f"{q}.1.weight"].new_zeros(pad)]))
                self._put(f"{q}.g1p.b", torch.cat([sd[f"{q}.1.bias"], sd[f"{q}.1.bias"].new_zeros(pad)]))
                c2 = _interleave_rows(_conv_w(sd[f"{q}.3.weight"]))
                self._put(f"{q}.c2p.w", torch.nn.functional.pad(c2, (0, pad)))

    def _put_moment_coef(self, q: str, w2: torch.Tensor, b2: torch.Tensor) -> None:
        """Coefficients turning the moments of a = GELU(GN1(h)) into the sums of z = W2 a + b2 (float64).

        [W2^T 1, W2^T b2, W2^T W2 upper triangle row by row (off-diagonal doubled), sum b2, sum b2^2]
        over the computed hidden width (``_moment_width``; extra columns zero).
        """
        w = w2.reshape(w2.shape[0], -1).double()
        b = b2.double()
        hid = w.shape[1]
        hw = _moment_width(hid)
        if hw != hid:
            w = torch.nn.functional.pad(w, (0, hw - hid))
        g = w.t() @ w
        tri = [g[j, k] * (1.0 if j == k else 2.0) for j in range(hw) for k in range(j, hw)]
        coef = torch.cat([w.sum(0), w.t() @ b, torch.stack(tri), b.sum()[None], (b * b).sum()[None]])
        self.register_buffer(_key(f"{q}.mom_coef"), coef.contiguous(), persistent=False)

    def _tables(self, device: torch.device, F: int, T: int, Lt: int) -> dict:
        """Window, positional and frequency-embedding tables (cached per device and shape)."""
        key = (str(device), F, T, Lt)
        cache = self.__dict__.setdefault("_table_cache", {})
        if key not in cache:
            cfg = self.config
            dim = self.bottom or cfg["channels"] * cfg["growth"] ** (self.depth - 1)
            tabs = {"window": torch.hann_window(cfg["nfft"]).to(device)}
            if self.t_layers:
                pe = sin_embedding_2d(dim, F, T, cfg["t_max_period"])  # [C, F, T]
                pos2 = pe.permute(1, 2, 0).reshape(F * T, dim) * cfg["t_weight_pos_embed"]
                pos1 = sin_embedding(Lt, dim, cfg["t_max_period"]) * cfg["t_weight_pos_embed"]
                tabs["pos2"] = pos2.contiguous().to(device)
                tabs["pos1"] = pos1.contiguous().to(device)
            for v in tabs.values():
                assert v.is_contiguous()
            cache[key] = tabs
        return cache[key]

    def _dconv(self, x: Act, pre: str) -> None:
        """DConv residual branch in place (unblend/blocks.py:238-317)."""
        B, H, W, C = x.B, x.H, x.W, x.C
        hid = int(C / self.config["dconv_comp"])
        per_h = 1 if H > 1 else 0
        groups = B * H
        dev = x.t.device
        x_gs = x.sh if H > 1 else x.sb
        for d in range(self.config["dconv_depth"]):
            q = f"{pre}.dconv.layers.{d}"
            dil = 2**d
            h = Act.freq(B, H, W, hid, dev)
            st1 = self._arena.take(2 * groups, dev)
            conv1_smem = 4 * ((128 + 2 * dil) * (C + 4) + hid * 3 * C)
            # Deep levels (hidden width >= 16): both contractions on the tensor
            # cores, z materialised (these levels hold few rows).
            deep = self.precision != "fp32-simt" and hid % 8 == 0 and hid >= 16
            if deep:
                self._conv(x, self.w(f"{q}.c1.w"), self.w(f"{q}.c1.b"), h, h_out=H, w_out=W, n_out=hid, kw=3,
                           dw=dil, pw=dil, stats=st1, stats_per_h=per_h)
                s1 = self._stats(st1, groups, W * hid)
                a = h.like()
                _lib.call("unblend_group_norm_apply", h.t.data_ptr(), a.t.data_ptr(), s1.data_ptr(),
                          self.w(f"{q}.g1.w").data_ptr(), self.w(f"{q}.g1.b").data_ptr(), groups * W, hid, W,
                          ACT_GELU)
                z = Act.freq(B, H, W, 2 * C, dev)
                st2 = self._arena.take(2 * groups, dev)
                self._conv(a, self.w(f"{q}.c2.w"), self.w(f"{q}.c2.b"), z, h_out=H, w_out=W, n_out=2 * C,
                           stats=st2, stats_per_h=per_h)
                s2 = self._stats(st2, groups, W * 2 * C)
                _lib.call("unblend_dconv_tail", x.t.data_ptr(), z.t.data_ptr(), s2.data_ptr(),
                          self.w(f"{q}.g2.w").data_ptr(), self.w(f"{q}.g2.b").data_ptr(),
                          self.w(f"{q}.scale").data_ptr(), groups, W, C, x_gs)
                continue
            fused = self.precision != "fp32-simt" and conv1_smem <= 220 * 1024 and C % 4 == 0
            hp = -(-hid // 4) * 4
            padded = fused and hp != hid
            pw = (lambda n: self.w(f"{q}.{n[:2]}p.{n[3:]}")) if padded else (lambda n: self.w(f"{q}.{n}"))
            if fused:
                h = Act.freq(B, H, W, hp, dev)
                _lib.call("unblend_dconv_conv1", x.t.data_ptr(), x_gs, groups, W, C, pw("c1.w").data_ptr(),
                          pw("c1.b").data_ptr(), hid, dil, h.t.data_ptr(), st1.data_ptr(),
                          work=6.0 * groups * W * C * hid)
            else:
                self._conv(x, self.w(f"{q}.c1.w"), self.w(f"{q}.c1.b"), h, h_out=H, w_out=W, n_out=hid, kw=3,
                           dw=dil, pw=dil, stats=st1, stats_per_h=per_h)
            s1 = self._stats(st1, groups, W * hid)
            if fused:
                # z = W2 GELU(GN1(h)) is recomputed instead of stored: once for
                # the GN2 statistics, once for the in-place residual update.
                args = (pw("g1.w").data_ptr(), pw("g1.b").data_ptr(), pw("c2.w").data_ptr(),
                        self.w(f"{q}.c2.b").data_ptr())
                # GN2 statistics from the moments of GELU(GN1(h)): no z at all.
                hw = _moment_width(hid)
                mom = self._arena.take(groups * (hw + hw * (hw + 1) // 2), dev)
                # The moments pass also rewrites h in place as a = GELU(GN1(h)) for the apply pass.
                _lib.call("unblend_dconv_moments", h.t.data_ptr(), groups, W, hid, s1.data_ptr(),
                          pw("g1.w").data_ptr(), pw("g1.b").data_ptr(), mom.data_ptr(), h.t.data_ptr(),
                          work=1.0 * groups * W * hw * (hw + 3))
                st2 = torch.empty(2 * groups, device=dev, dtype=torch.float64)
                _lib.call("unblend_dconv_moment_sums", mom.data_ptr(), getattr(self, _key(f"{q}.mom_coef")).data_ptr(),
                          groups, W, hid, st2.data_ptr())
                s2 = self._stats(st2, groups, W * 2 * C)
                _lib.call("unblend_dconv_apply", x.t.data_ptr(), x_gs, h.t.data_ptr(), groups, W, hid, C,
                          s1.data_ptr(), *args, s2.data_ptr(), self.w(f"{q}.g2.w").data_ptr(),
                          self.w(f"{q}.g2.b").data_ptr(), self.w(f"{q}.scale").data_ptr(), 1,
                          work=4.0 * groups * W * C * hid)
                continue
            z = Act.freq(B, H, W, 2 * C, dev)
            st2 = self._arena.take(2 * groups, dev)
            self._conv(h, self.w(f"{q}.c2.w"), self.w(f"{q}.c2.b"), z, h_out=H, w_out=W, n_out=2 * C,
                       prologue=PRO_GN_GELU, pro_stats=s1, pro_gamma=self.w(f"{q}.g1.w"),
                       pro_beta=self.w(f"{q}.g1.b"), pro_per_h=per_h, stats=st2, stats_per_h=per_h)
            s2 = self._stats(st2, groups, W * 2 * C)
            _lib.call("unblend_dconv_tail", x.t.data_ptr(), z.t.data_ptr(), s2.data_ptr(),
                      self.w(f"{q}.g2.w").data_ptr(), self.w(f"{q}.g2.b").data_ptr(),
                      self.w(f"{q}.scale").data_ptr(), groups, W, C, x.sh if H > 1 else x.sb)

    def _enc(self, x: Act, pre: str, freq: bool) -> Act:
        """HEncLayer (unblend/blocks.py:474-511): conv -> GELU -> DConv -> 1x1 rewrite -> GLU."""
        cout = self.w(f"{pre}.conv.b").shape[0]
        dev = x.t.device
        if freq:
            ho, wo = x.H // 4, x.W
            y = Act.freq(x.B, ho, wo, cout, dev)
            self._conv(x, self.w(f"{pre}.conv.w"), self.w(f"{pre}.conv.b"), y, h_out=ho, w_out=wo, n_out=cout,
                       kh=8, sh=4, ph=2, act=ACT_GELU)
        else:
            wo = -(-x.W // 4)
            y = Act.time(x.B, wo, 4 * -(-wo // 4), cout, dev)
            self._conv(x, self.w(f"{pre}.conv.w"), self.w(f"{pre}.conv.b"), y, h_out=1, w_out=wo, n_out=cout,
                       kw=8, sw=4, pw=2, act=ACT_GELU)
        self._dconv(y, pre)
        out = y.like()
        if not freq and out.sb // out.C > out.W:
            # Rows past the logical length are the zero padding the next
            # stride-4 convolution reads (the reference pads to a multiple of 4).
            cap = out.sb // out.C
            _lib.call("unblend_zero_f32", out.t.data_ptr() + 4 * out.W * out.C, (cap - out.W) * out.C, out.B, out.sb)
        # The frequency embedding (added to the first frequency layer's output) rides in the rewrite epilogue.
        post = self.w("freq_emb") if freq and pre == "encoder.0" and "freq_emb" in self.weights else None
        self._conv(y, self.w(f"{pre}.rewrite.w"), self.w(f"{pre}.rewrite.b"), out, h_out=y.H, w_out=y.W,
                   n_out=2 * cout, act=ACT_GLU, post=post)
        return out

    def _dec(self, x: Act, skip: Act, pre: str, freq: bool, last: bool, length: int, skip_in_x: bool = False,
             next_skip: Act | None = None) -> Act:
        """HDecLayer (unblend/blocks.py:706-747): +skip -> 3-tap rewrite -> GLU -> DConv -> convT -> crop -> GELU.

        ``skip_in_x``: the skip connection was already added to ``x`` by the previous
        layer. ``next_skip``: the following decoder layer's skip, added here in the
        ConvTranspose epilogue (``GELU(convT) + skip``, the same single fp32 addition
        the next layer would make) instead of by a separate pass over the activation.
        """
        C = x.C
        y = x.like()
        pro = dict(prologue=PRO_NONE) if skip_in_x else dict(prologue=PRO_ADD, pro_x2=skip)
        if freq:
            self._conv(x, self.w(f"{pre}.rewrite.w"), self.w(f"{pre}.rewrite.b"), y, h_out=x.H, w_out=x.W,
                       n_out=2 * C, kh=3, kw=3, ph=1, pw=1, act=ACT_GLU, **pro)
        else:
            self._conv(x, self.w(f"{pre}.rewrite.w"), self.w(f"{pre}.rewrite.b"), y, h_out=1, w_out=x.W,
                       n_out=2 * C, kw=3, pw=1, act=ACT_GLU, **pro)
        self._dconv(y, pre)
        cout = self._wsel(f"{pre}.convtr.b").shape[0] // 4
        act = ACT_NONE if last else ACT_GELU
        dev = x.t.device
        b = self._wsel(f"{pre}.convtr.b")
        if next_skip is not None:
            want = (4 * x.H * x.W * cout, x.W * cout, cout) if freq else (4 * x.W * cout, 4 * x.W * cout, cout)
            assert (next_skip.sb, next_skip.sh, next_skip.sw, next_skip.C) == want + (cout,), \
                "skip layout differs from the decoder output"
        w = self._wsel(f"{pre}.convtr.w")
        res = None if next_skip is None else next_skip.t
        # One 3-tap launch for the four output phases: channel group s lands at output row 4p + s.
        if freq:
            out = Act.freq(x.B, 4 * x.H, x.W, cout, dev)
            row = out.sh  # stride of one output frequency row
            self._conv(y, w, b, out, h_out=x.H, w_out=x.W, n_out=4 * cout, kh=3, ph=1, act=act, n_group=cout,
                       out_sg=row, out_sh=4 * row, res=res, useful=2.0 / 3.0)
        else:
            cap = 4 * x.W
            out = Act.time(x.B, length, cap, cout, dev)
            self._conv(y, w, b, out, h_out=1, w_out=x.W, n_out=4 * cout, kw=3, pw=1, act=act, n_group=cout,
                       out_sg=cout, out_sw=4 * cout, res=res, useful=2.0 / 3.0)
        return out

    def _linear(self, x: torch.Tensor, B: int, L: int, K: int, w: torch.Tensor, b: torch.Tensor | None,
                out: torch.Tensor, N: int, act: int = ACT_NONE, res: torch.Tensor | None = None,
                res_scale=None, stats: torch.Tensor | None = None) -> None:
        xa = Act(x, B, 1, L, K, L * K, L * K, K)
        oa = Act(out, B, 1, L, N if act != ACT_GLU else N // 2, L * N, L * N, N)
        self._conv(xa, w, b, oa, h_out=1, w_out=L, n_out=N, act=act, res=res, res_scale=res_scale, stats=stats,
                   y_bf16=out.dtype == torch.bfloat16)

    def _ln(self, x: torch.Tensor, rows: int, c: int, name: str, pos: torch.Tensor | None = None,
            pos_rows: int = 1, bf16: bool = False) -> torch.Tensor:
        """LayerNorm of ``rows`` rows; ``bf16``: written as bf16 for rows that only feed bf16 GEMMs."""
        y = torch.empty_like(x, dtype=torch.bfloat16 if bf16 else torch.float32)
        _lib.call("unblend_layer_norm_bf16" if bf16 else "unblend_layer_norm", x.data_ptr(), y.data_ptr(),
                  self.w(f"{name}.weight").data_ptr(), self.w(f"{name}.bias").data_ptr(), _lib.ptr(pos), 1.0,
                  pos_rows, rows, c)
        return y

    def _attn_bf16(self, hd: int, D: int) -> bool:
        """Whether a transformer layer's projections go straight to the bf16 attention kernel."""
        return self.precision == "bf16" and hd in (48, 64) and D % 32 == 0

    def _attention(self, qbuf: torch.Tensor, q_off: int, kvbuf: torch.Tensor, k_off: int, v_off: int, o: int,
                   B: int, heads: int, L: int, Lk: int, hd: int, q_sb: int, q_sr: int, kv_sb: int, kv_sr: int,
                   o_sb: int, o_sr: int, o_bf16: bool = False) -> None:
        """softmax(Q K^T / sqrt(hd)) V for all heads: tensor-core flash attention, or SIMT.

        Q sits at element ``q_off`` of ``qbuf``, K and V at ``k_off`` / ``v_off`` of
        ``kvbuf`` (fp32 projections); strides are in elements. In bf16 precision with
        64-dim heads the projections are rounded to bf16 once and the bf16 kernel runs
        (kind::f16 MMAs, P in bf16); fp32 keeps the 3-pass TF32 kernel.
        """
        work = 4.0 * B * L * Lk * hd * heads
        scale = 1.0 / math.sqrt(hd)
        if qbuf.dtype == torch.bfloat16 or (self.precision == "bf16" and hd in (48, 64) and o % 16 == 0 and
                                            all(v % 8 == 0 for v in (q_off, k_off, v_off, q_sb, q_sr, kv_sb,
                                                                     kv_sr, o_sb, o_sr))):
            if qbuf.dtype == torch.bfloat16:  # projections already rounded by their epilogue
                qb, kvb = qbuf, kvbuf
            else:
                qb = torch.empty(qbuf.numel(), device=qbuf.device, dtype=torch.bfloat16)
                _lib.call("unblend_cast_bf16", qbuf.data_ptr(), qb.data_ptr(), qbuf.numel())
                kvb = qb
                if kvbuf is not qbuf:
                    kvb = torch.empty(kvbuf.numel(), device=kvbuf.device, dtype=torch.bfloat16)
                    _lib.call("unblend_cast_bf16", kvbuf.data_ptr(), kvb.data_ptr(), kvbuf.numel())
            a = AttnParams()
            a.outer, a.inner, a.heads, a.lq, a.lk, a.hd = B, 1, heads, L, Lk, hd
            a.q_so, a.q_si, a.q_sr = q_sb, 8, q_sr
            a.kv_so, a.kv_si, a.kv_sr = kv_sb, 8, kv_sr
            a.out, a.o_so, a.o_si, a.o_sr, a.out_bf16 = o, o_sb, 0, o_sr, 1 if o_bf16 else 0
            a.scale = scale
            _lib.call("unblend_attention_bf16", qb.data_ptr() + 2 * q_off, kvb.data_ptr() + 2 * k_off,
                      kvb.data_ptr() + 2 * v_off, ctypes_byref(a), work=work)
            return
        q, k, v = qbuf.data_ptr() + 4 * q_off, kvbuf.data_ptr() + 4 * k_off, kvbuf.data_ptr() + 4 * v_off
        if self.precision != "fp32-simt" and hd % 4 == 0 and hd <= 64 and all(p % 16 == 0 for p in (q, k, v, o)):
            if self.precision == "fp32":
                mode = 2 if self.attention_split == "bf16x3" else 0
            else:
                mode = 1
            _lib.call("unblend_attention_tc", q, k, v, o, B, heads, L, Lk, hd, q_sb, q_sr, kv_sb, kv_sr, o_sb, o_sr,
                      scale, mode, work=work)
            return
        _lib.call("unblend_attention_f32", q, k, v, o, B, heads, L, Lk, hd, q_sb, q_sr, kv_sb, kv_sr, o_sb, o_sr,
                  scale, work=work)

    def _attn_layer(self, q: str, x: torch.Tensor, kv_src: torch.Tensor | None, B: int, L: int, Lk: int,
                    D: int, cross: bool) -> torch.Tensor:
        """One transformer layer with norm_first, LayerScale and norm_out (unblend/transformer.py:328-359, 461-481)."""
        heads = self.config["t_heads"]
        hd = D // heads
        dev = x.device
        attn = "cross_attn" if cross else "self_attn"
        # bf16 precision: the activations that only feed bf16 GEMMs (LayerNorm outputs, the
        # attention output, the FeedForward hidden layer) are written as bf16 by their
        # producers and loaded as they are; with 48/64-dim heads the projections leave the
        # tensor cores as bf16 for the bf16 attention kernel (no separate rounding pass).
        bf = self.precision == "bf16"
        h = self._ln(x, B * L, D, f"{q}.norm1", bf16=bf)
        pdt = torch.bfloat16 if self._attn_bf16(hd, D) else torch.float32
        att = torch.empty(B * L * D, device=dev, dtype=pdt)
        if not cross:
            win, bin_ = self.w(f"{q}.{attn}.in_proj_weight"), self.w(f"{q}.{attn}.in_proj_bias")
            qkv = torch.empty(B * L * 3 * D, device=dev, dtype=pdt)
            self._linear(h, B, L, D, win, bin_, qkv, 3 * D)
            self._attention(qkv, 0, qkv, D, 2 * D, att.data_ptr(), B, heads, L, L, hd, L * 3 * D,
                            3 * D, L * 3 * D, 3 * D, L * D, D, o_bf16=att.dtype == torch.bfloat16)
        else:
            kvn = self._ln(kv_src, B * Lk, D, f"{q}.norm2", bf16=bf)
            qp = torch.empty(B * L * D, device=dev, dtype=pdt)
            self._linear(h, B, L, D, self.w(f"{q}.in_q.w"), self.w(f"{q}.in_q.b"), qp, D)
            kv = torch.empty(B * Lk * 2 * D, device=dev, dtype=pdt)
            self._linear(kvn, B, Lk, D, self.w(f"{q}.in_kv.w"), self.w(f"{q}.in_kv.b"), kv, 2 * D)
            self._attention(qp, 0, kv, 0, D, att.data_ptr(), B, heads, L, Lk, hd, L * D, D,
                            Lk * 2 * D, 2 * D, L * D, D, o_bf16=att.dtype == torch.bfloat16)
        x_new = torch.empty_like(x)
        self._linear(att, B, L, D, self.w(f"{q}.{attn}.out_proj.weight"), self.w(f"{q}.{attn}.out_proj.bias"),
                     x_new, D, res=x, res_scale=self.w(f"{q}.gamma_1.scale"))
        h2 = self._ln(x_new, B * L, D, f"{q}.norm3" if cross else f"{q}.norm2", bf16=bf)
        hidden = self.w(f"{q}.linear1.bias").shape[0]
        f = torch.empty(B * L * hidden, device=dev, dtype=torch.bfloat16 if bf and hidden % 32 == 0 else torch.float32)
        self._linear(h2, B, L, D, self.w(f"{q}.linear1.weight"), self.w(f"{q}.linear1.bias"), f, hidden,
                     act=ACT_GELU)
        st = self._arena.take(2 * B, dev)
        self._linear(f, B, L, hidden, self.w(f"{q}.linear2.weight"), self.w(f"{q}.linear2.bias"), x_new, D,
                     res=x_new, res_scale=self.w(f"{q}.gamma_2.scale"), stats=st)
        s = self._stats(st, B, L * D)
        _lib.call("unblend_group_norm_apply", x_new.data_ptr(), x_new.data_ptr(), s.data_ptr(),
                  self.w(f"{q}.norm_out.weight").data_ptr(), self.w(f"{q}.norm_out.bias").data_ptr(), B * L, D,
                  L, ACT_NONE)
        return x_new

    def _transformer(self, x: Act, xt: Act, tabs: dict) -> tuple[Act, Act]:
        """Channel up-sampling, CrossTransformerEncoder (unblend/transformer.py:703-742), down-sampling."""
        B, F, T, C0 = x.B, x.H, x.W, x.C
        Lx, Lt = F * T, xt.W
        dev = x.t.device
        D = self.bottom or C0
        p = "crosstransformer"
        # Time rows of this level may sit in a buffer with spare capacity rows.
        xt_rows = xt.t if xt.sb == Lt * C0 else xt.t.view(B, -1)[:, : Lt * C0].contiguous().view(-1)
        if self.bottom:
            xu = torch.empty(B * Lx * D, device=dev, dtype=torch.float32)
            self._linear(x.t, B, Lx, C0, self.w("channel_upsampler.w"), self.w("channel_upsampler.b"), xu, D)
            xtu = torch.empty(B * Lt * D, device=dev, dtype=torch.float32)
            self._linear(xt_rows, B, Lt, C0, self.w("channel_upsampler_t.w"), self.w("channel_upsampler_t.b"), xtu,
                         D)
        else:
            xu, xtu = x.t, xt_rows
        self._trace_tok("up_x", xu, B, Lx, D)
        self._trace_tok("up_xt", xtu, B, Lt, D)
        xs = self._ln(xu, B * Lx, D, f"{p}.norm_in", tabs["pos2"], Lx)
        xts = self._ln(xtu, B * Lt, D, f"{p}.norm_in_t", tabs["pos1"], Lt)
        self._trace_tok("in_x", xs, B, Lx, D)
        self._trace_tok("in_xt", xts, B, Lt, D)
        parity = 1 if self.config["t_cross_first"] else 0
        for idx in range(self.t_layers):
            if idx % 2 == parity:
                xs = self._attn_layer(f"{p}.layers.{idx}", xs, None, B, Lx, Lx, D, False)
                xts = self._attn_layer(f"{p}.layers_t.{idx}", xts, None, B, Lt, Lt, D, False)
            else:
                old = xs
                xs = self._attn_layer(f"{p}.layers.{idx}", xs, xts, B, Lx, Lt, D, True)
                xts = self._attn_layer(f"{p}.layers_t.{idx}", xts, old, B, Lt, Lx, D, True)
            self._trace_tok(f"l{idx}_x", xs, B, Lx, D)
            self._trace_tok(f"l{idx}_xt", xts, B, Lt, D)
        xo = Act.freq(B, F, T, C0, dev)
        xto = Act.time(B, Lt, xt.sb // C0, C0, dev)
        if self.bottom:
            self._linear(xs, B, Lx, D, self.w("channel_downsampler.w"), self.w("channel_downsampler.b"), xo.t, C0)
            xd = torch.empty(B * Lt * C0, device=dev, dtype=torch.float32)
            self._linear(xts, B, Lt, D, self.w("channel_downsampler_t.w"), self.w("channel_downsampler_t.b"), xd, C0)
            xto.t.view(B, -1)[:, : Lt * C0].copy_(xd.view(B, -1))
        else:
            xo.t.copy_(xs)
            xto.t.view(B, -1)[:, : Lt * C0].copy_(xts.view(B, -1))
        return xo, xto

    # ------------------------------------------------------------------ forward
    #: When set to a dict, ``forward`` stores a CPU copy of every stage output
    #: in the reference's channel-first layout (debugging aid, slow).
    trace: dict | None = None

    def _trace_act(self, name: str, a: Act) -> None:
        if self.trace is None:
            return
        if a.H > 1 or a.sb == a.H * a.W * a.C:
            v = a.t.view(a.B, a.H, a.W, a.C).permute(0, 3, 1, 2)
            v = v[:, :, 0] if a.H == 1 else v
        else:
            v = a.t.view(a.B, -1, a.C)[:, : a.W].permute(0, 2, 1)
        self.trace[name] = v.detach().cpu().clone()

    def _trace_tok(self, name: str, t: torch.Tensor, B: int, L: int, D: int) -> None:
        if self.trace is not None:
            self.trace[name] = t.view(B, L, D).detach().cpu().clone()

    def forward(self, mix: torch.Tensor) -> torch.Tensor:
        """Separate ``mix`` [B, C, T<=segment] into ``[B, S, C, T]`` (unblend/htdemucs.py:650-704)."""
        if mix.device.type != "cuda":
            raise RuntimeError("HTDemucsCuda runs on CUDA devices only (no CPU path)")
        wdev = next(iter(self.weights.values())).device
        if wdev != mix.device:
            raise RuntimeError(f"weights are on {wdev}, input on {mix.device}; call .to(device) first")
        T = self.segment_length
        length = mix.shape[-1]
        if length > T:
            raise ValueError(f"Given length {length} is longer than training length {T}")
        mix = mix.float()
        if length < T:
            mix = torch.nn.functional.pad(mix, (0, T - length))
        mix = mix.contiguous()
        graphed = self.__dict__.get("_graphed")
        out = graphed(mix) if graphed is not None else self._forward_arena(mix)
        if length < T:
            out = out[..., :length]
        return out

    # ------------------------------------------------------------------ optional hooks (unblend/backends.py:62-111)
    def prefill_inference_caches(self) -> None:
        """Build the window / positional tables of the segment shape before any graph capture."""
        dev = next(iter(self.weights.values())).device
        if dev.type != "cuda":
            return
        nfft = self.config["nfft"]
        frames = -(-self.segment_length // (nfft // 4))
        lt = self.segment_length
        for _ in range(self.depth):
            lt = -(-lt // 4)
        self._tables(dev, nfft // 2 // 4**self.depth, frames, lt)

    def enable_compiled_core(self) -> None:
        """Replay the forward from CUDA graphs; tails below 7/8 of the captured batch run eagerly, others are zero-padded."""
        from .graphs import GraphedForward

        self.prefill_inference_caches()
        self.__dict__["_graphed"] = GraphedForward(self._forward_arena)
        self._fixed_batch_shape = True
        self._eager_tails = True

    def disable_compiled_core(self) -> None:
        """Back to eager launches; releases the captured graphs."""
        graphed = self.__dict__.pop("_graphed", None)
        if graphed is not None:
            graphed.release()
        self._fixed_batch_shape = False
        self._eager_tails = False

    def select_sources(self, names: list[str] | None) -> "HTDemucsCuda":
        """Materialise only the named stems (all of them when ``names`` is None).

        The stems of HTDemucs part ways only in the last decoder layers: the
        final frequency ConvTranspose emits 4 channels per source (2 audio
        channels x real/imaginary) and the final time ConvTranspose 2 per
        source; everything before is shared. Selecting stems keeps only their
        output rows of those two layers and runs the iSTFT for them alone, so
        ``forward`` returns ``[B, len(names), C, T]`` equal to the matching
        slices of the full output (``SeparatedSources.isolate_stem`` applied
        inside the model). ``self.sources`` becomes ``names``, which is what
        ``apply_model`` reads for the output width.
        """
        full = list(self.config["sources"])
        if names is None:
            names = full
        names = list(names)
        bad = [n for n in names if n not in full]
        if bad or not names or len(set(names)) != len(names):
            raise ValidationError(f"Stems {bad or names!r} are not a selection of this model's sources. "
                                  f"Available stems: {', '.join(full)}")
        graphed = "_graphed" in self.__dict__
        if graphed:
            self.disable_compiled_core()
        idx = [full.index(n) for n in names]
        sel = {}
        if idx != list(range(len(full))):
            last = self.depth - 1
            for pre, per in ((f"decoder.{last}", 4), (f"tdecoder.{last}", 2)):
                b = self.w(f"{pre}.convtr.b")
                cout = b.shape[0] // 4
                ch = torch.tensor([s * per + k for s in idx for k in range(per)], device=b.device)
                rows = torch.cat([ch + ph * cout for ph in range(4)])  # rows are (phase, channel)
                sel[f"{pre}.convtr.w"] = self.w(f"{pre}.convtr.w")[rows].contiguous()
                sel[f"{pre}.convtr.b"] = b[rows].contiguous()
        self.__dict__["_selected"] = sel
        self._tc_cache.clear()
        self.sources = names
        if graphed:
            self.enable_compiled_core()
        return self

    def _wsel(self, name: str) -> torch.Tensor:
        """Weight ``name``, or its stem-selected rows when a selection is active."""
        sel = self.__dict__.get("_selected")
        return sel[name] if sel and name in sel else self.w(name)

    def _forward_arena(self, mix: torch.Tensor) -> torch.Tensor:
        self._arena.begin(mix.device, mix.shape[0])
        try:
            return self._forward_full(mix)
        finally:
            self._arena.end(mix.device)

    def _forward_full(self, mix: torch.Tensor) -> torch.Tensor:
        B, C, T = mix.shape
        if C != 2:
            raise ValueError("stereo input expected")
        dev = mix.device
        S = len(self.sources)
        nfft = self.config["nfft"]
        frames = -(-T // (nfft // 4))
        Fq = nfft // 2
        levels = [T]
        for _ in range(self.depth):
            levels.append(-(-levels[-1] // 4))
        tabs = self._tables(dev, Fq // 4**self.depth, frames, levels[-1])
        # STFT front end and normalisation of both branches.
        spec = Act.freq(B, Fq, frames, 4, dev)
        _lib.call("unblend_stft_cac", mix.data_ptr(), spec.t.data_ptr(), tabs["window"].data_ptr(), B, T, nfft)
        work = torch.empty(4 * B, device=dev, dtype=torch.float64)
        fstats = torch.empty(2 * B, device=dev, dtype=torch.float32)
        tstats = torch.empty(2 * B, device=dev, dtype=torch.float32)
        _lib.call("unblend_mean_std", spec.t.data_ptr(), work.data_ptr(), fstats.data_ptr(), B, Fq * frames * 4)
        _lib.call("unblend_standardize", spec.t.data_ptr(), spec.t.data_ptr(), fstats.data_ptr(),
                  Fq * frames * 4, B)
        _lib.call("unblend_mean_std", mix.data_ptr(), work.data_ptr(), tstats.data_ptr(), B, 2 * T)
        xt = Act.time(B, T, T, 2, dev)
        _lib.call("unblend_time_input", mix.data_ptr(), xt.t.data_ptr(), tstats.data_ptr(), B, T, T)
        x = spec
        self._trace_act("spec", x)
        self._trace_act("xt", xt)
        saved, saved_t = [], []
        for idx in range(self.depth):
            xt = self._enc(xt, f"tencoder.{idx}", False)
            saved_t.append(xt)
            x = self._enc(x, f"encoder.{idx}", True)  # encoder.0 adds the frequency embedding
            saved.append(x)
            self._trace_act(f"tenc{idx}", xt)
            self._trace_act(f"enc{idx}", x)
        if self.t_layers:
            x, xt = self._transformer(x, xt, tabs)
            self._trace_act("tr_x", x)
            self._trace_act("tr_xt", xt)
        for idx in range(self.depth):
            last = idx == self.depth - 1
            skip, skip_t = saved.pop(-1), saved_t.pop(-1)
            # Each ConvTranspose adds the next layer's skip in its epilogue (traced
            # decoder outputs therefore include it).
            nxt, nxt_t = (None, None) if last else (saved[-1], saved_t[-1])
            x = self._dec(x, skip, f"decoder.{idx}", True, last, 0, skip_in_x=idx > 0, next_skip=nxt)
            xt = self._dec(xt, skip_t, f"tdecoder.{idx}", False, last, levels[self.depth - 1 - idx],
                           skip_in_x=idx > 0, next_skip=nxt_t)
            self._trace_act(f"dec{idx}", x)
            self._trace_act(f"tdec{idx}", xt)
        out = torch.empty(B, S, 2, T, device=dev, dtype=torch.float32)
        frames_buf = torch.empty(B * S * 2 * frames * nfft, device=dev, dtype=torch.float32)
        _lib.call("unblend_istft_output", x.t.data_ptr(), xt.t.data_ptr(), xt.sb, fstats.data_ptr(),
                  tstats.data_ptr(), tabs["window"].data_ptr(), frames_buf.data_ptr(), out.data_ptr(), B, S, T,
                  nfft)
        return out
