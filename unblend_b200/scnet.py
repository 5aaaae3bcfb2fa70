"""SCNet forward on B200: the third architecture on the segment engine.

``SCNetCuda`` keeps the model contract that ``apply_model`` drives
(unblend/backends.py:36-59): ``sources``, ``samplerate``, ``audio_channels``,
``max_allowed_segment``, ``_fixed_batch_shape`` and ``forward(mix[B, C, L]) ->
[B, S, C, L]``, plus ``configure_inference`` with the reference's validation
(unblend/scnet.py:700-711). It is built from the reference ``state_dict``
(strict key set) of ``SCNet`` or ``SCNetMasked`` and runs
unblend/scnet.py:746-895 as CUDA kernels of ``libunblend_b200.so``:

* normalised STFT (no window, Hann for the masked variant) of the segment
  padded by ``stft_padding``, frame-major, then swapped to frequency-major
  ``[B, F, T, 4]`` activations (with the masked variant's frequency embedding);
* three ``SDblock`` encoder stages: each band's strided convolution along
  frequency, its ``ConvolutionModule`` stack (GroupNorm, 1x3 convolution with
  GLU, depthwise 1x3 convolution with GroupNorm and Swish, 1x1 convolution,
  residual), GELU into the full band, the global 3x3 convolution;
* the dual-path trunk: GroupNorm, the input projections of both LSTM
  directions as one GEMM, the recurrence kernel, the output projection with
  the residual, first along frequency then along frames; an orthonormal real
  DFT along frames between layers;
* three decoder stages: skip add and the ``FusionLayer`` 3x3 convolution (the
  reference convolves ``cat([x, x])``, i.e. ``x`` with the sum of the two weight
  halves) with GLU; the ``SUlayer`` transposed convolutions (stride 1: the
  flipped-kernel convolution; kernel = stride: one 1x1 convolution emitting
  every output phase) trimmed back to each band's length;
* the mask head (masked variant) and the inverse STFT of mixture x mask (or of
  the decoder output).

Activations are fp32 and channels-last ``[B, F, T, C]``.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import ACT_GELU, ACT_GLU, ACT_NONE, ACT_SWISH, ACT_TANH
from .apply import ValidationError
from .convnet import Act, ConvNet, _conv_w, _interleave_rows


def stft_padding(samples: int, hop: int) -> int:
    """Trailing zeros before the STFT: to a hop boundary, plus one hop when the frame count would be odd."""
    padding = hop - samples % hop
    if (samples + padding) // hop % 2 == 0:
        padding += hop
    return padding


def band_splits(freq: int, band_sr: list[float]) -> list[tuple[int, int]]:
    """Row ranges of the low, mid and high bands of an SD layer."""
    a = math.ceil(freq * band_sr[0])
    b = math.ceil(freq * (band_sr[0] + band_sr[1]))
    return [(0, a), (a, b), (b, freq)]


class SCNetCuda(ConvNet):
    """SCNet / SCNetMasked separation forward as sm_100a CUDA kernels.

    :param config: ``architecture`` (``"scnet"`` or ``"scnet_masked"``), ``sources``,
        ``samplerate``, ``segment_samples`` and the constructor config of the
        registry entry (``unblend_b200.synth.scnet_config``).
    :param state_dict: Reference-layout weights (strict key set).
    :param precision: ``"fp32"`` (every convolution on the fp32 CUDA-core kernel),
        ``"bf16"`` (bf16 tensor-core operands, fp32 accumulation and activations) or
        ``"fp32-simt"`` (same as ``"fp32"``). The LSTM recurrences, DFTs and norms
        run in fp32 in every mode. SCNet has no LayerScale damping its residual
        branches, so the few 1e-5 of output RMS that each 3-pass TF32 tensor-core
        convolution leaves add up over its convolution stages (1.5e-4 of output
        RMS on the xl configuration); fp32 therefore stays on CUDA cores.
    """

    def __init__(self, config: dict, state_dict: dict, precision: str = "fp32") -> None:
        super().__init__(precision)
        cfg = dict(config)
        arch = cfg.get("architecture", "scnet")
        if arch not in ("scnet", "scnet_masked"):
            raise ValidationError(f"Unknown SCNet architecture {arch!r}; expected one of ['scnet', 'scnet_masked'].")
        if cfg.get("audio_channels", 2) != 2 or cfg["nfft"] != 4096 or cfg["win_size"] != cfg["nfft"]:
            raise ValueError("unsupported SCNet geometry (stereo, 4096-point transform, full-length window)")
        if cfg["conv_kernel"] % 2 == 0:
            raise ValidationError(f"SCNet conv kernel must be odd, got {cfg['conv_kernel']}.")
        for k, s in zip(cfg["band_kernel"], cfg["band_stride"]):
            if not (s == 1 or k == s):
                raise ValueError("band convolutions with stride 1 or kernel == stride only")
        self.config = cfg
        self.masked = arch == "scnet_masked"
        self.sources = list(cfg["sources"])
        self.samplerate = int(cfg.get("samplerate", 44100))
        self.audio_channels = 2
        self.max_allowed_segment = cfg.get("segment_samples", 485100) / float(self.samplerate)
        self._fixed_batch_shape = False
        self._eager_tails = False
        self.dims = list(cfg["dims"])
        self._pack({k: v.detach().float().cpu() for k, v in state_dict.items()})
        self.__dict__["_win_cache"] = {}

    def _tc_eligible(self, x: Act, p, prologue: int, out_offset: int) -> bool:
        """Tensor cores for bf16 precision only (fp32 convolutions run on CUDA cores)."""
        return self.precision == "bf16" and super()._tc_eligible(x, p, prologue, out_offset)

    # ------------------------------------------------------------------ contract
    def configure_inference(self, *, sources: list[str], samplerate: int, segment_samples: int) -> None:
        """Attach the checkpoint's stem names, sample rate and segment (unblend/scnet.py:700-711)."""
        if len(sources) != len(self.sources):
            raise ValidationError(f"SCNet checkpoint emits {len(self.sources)} stems; got {len(sources)} source names.")
        self.sources = list(sources)
        self.samplerate = int(samplerate)
        self.max_allowed_segment = segment_samples / float(samplerate)

    # ------------------------------------------------------------------ weights
    def _pack(self, sd: dict) -> None:
        cfg, dims = self.config, self.dims
        S = len(self.sources)
        stages = len(dims) - 1
        for i in range(stages):
            p = f"encoder.{i}"
            for j in range(3):
                self._put(f"{p}.band{j}.w", _conv_w(sd[f"{p}.SDlayer.convs.{j}.weight"]))
                self._put(f"{p}.band{j}.b", sd[f"{p}.SDlayer.convs.{j}.bias"])
                for d in range(abs(cfg["conv_depths"][j])):
                    q = f"{p}.conv_modules.{j}.layers.{d}"
                    self._put(f"{q}.gn0.w", sd[f"{q}.0.weight"])
                    self._put(f"{q}.gn0.b", sd[f"{q}.0.bias"])
                    self._put(f"{q}.c1.w", _interleave_rows(_conv_w(sd[f"{q}.1.weight"])))
                    self._put(f"{q}.c1.b", _interleave_rows(sd[f"{q}.1.bias"]))
                    self._put(f"{q}.dw.w", sd[f"{q}.3.weight"].reshape(sd[f"{q}.3.weight"].shape[0], -1))
                    self._put(f"{q}.dw.b", sd[f"{q}.3.bias"])
                    self._put(f"{q}.gn4.w", sd[f"{q}.4.weight"])
                    self._put(f"{q}.gn4.b", sd[f"{q}.4.bias"])
                    self._put(f"{q}.c6.w", _conv_w(sd[f"{q}.6.weight"]))
                    self._put(f"{q}.c6.b", sd[f"{q}.6.bias"])
            self._put(f"{p}.global.w", _conv_w(sd[f"{p}.globalconv.weight"]))
            self._put(f"{p}.global.b", sd[f"{p}.globalconv.bias"])
        for j in range(stages):
            q = f"decoder.{j}"
            w = sd[f"{q}.0.conv.weight"]
            c = w.shape[1] // 2
            # conv(cat([x, x]), W) = conv(x, W[:, :C] + W[:, C:]).
            self._put(f"{q}.fuse.w", _interleave_rows(_conv_w(w[:, :c] + w[:, c:])))
            self._put(f"{q}.fuse.b", _interleave_rows(sd[f"{q}.0.conv.bias"]))
            for b in range(3):
                wt, bt = sd[f"{q}.1.convtrs.{b}.weight"], sd[f"{q}.1.convtrs.{b}.bias"]  # [Cin, Cout, k, 1]
                k, s = cfg["band_kernel"][b], cfg["band_stride"][b]
                if s == 1:
                    # Transposed conv + symmetric trim = conv with the flipped kernel.
                    flipped = wt[..., 0].flip(-1).permute(1, 2, 0).unsqueeze(2)  # [Cout, k, 1, Cin]
                    self._put(f"{q}.up{b}.w", flipped)
                    self._put(f"{q}.up{b}.b", bt)
                else:
                    # Output row k * i + j of input row i: rows ordered (phase j, channel).
                    phases = wt[..., 0].permute(2, 1, 0).reshape(k * wt.shape[1], 1, 1, wt.shape[0])
                    self._put(f"{q}.up{b}.w", phases)
                    self._put(f"{q}.up{b}.b", bt.repeat(k))
        for i in range(cfg["num_dplayer"]):
            q = f"separation_net.dp_modules.{i}"
            for j in range(2):
                lq = f"{q}.lstm_layers.{j}"
                wih = torch.cat([sd[f"{lq}.weight_ih_l0"], sd[f"{lq}.weight_ih_l0_reverse"]])
                bias = torch.cat([sd[f"{lq}.bias_ih_l0"] + sd[f"{lq}.bias_hh_l0"],
                                  sd[f"{lq}.bias_ih_l0_reverse"] + sd[f"{lq}.bias_hh_l0_reverse"]])
                self._put(f"{q}.ih{j}.w", wih[:, None, None, :])
                self._put(f"{q}.ih{j}.b", bias)
                self._put(f"{q}.hh{j}", torch.stack([sd[f"{lq}.weight_hh_l0"].t(),
                                                     sd[f"{lq}.weight_hh_l0_reverse"].t()]))
                self._put(f"{q}.lin{j}.w", sd[f"{q}.linear_layers.{j}.weight"][:, None, None, :])
                self._put(f"{q}.lin{j}.b", sd[f"{q}.linear_layers.{j}.bias"])
                self._put(f"{q}.gn{j}.w", sd[f"{q}.norm_layers.{j}.weight"])
                self._put(f"{q}.gn{j}.b", sd[f"{q}.norm_layers.{j}.bias"])
        if self.masked:
            self._put("pos", sd["pos_embed_f"][0, :, :, 0])  # [4, max_f]
            self._put("mask0.w", _conv_w(sd["mask_layer.0.weight"]))
            self._put("mask0.b", sd["mask_layer.0.bias"])
            self._put("mask2.w", _conv_w(sd["mask_layer.2.weight"]))
            self._put("mask2.b", sd["mask_layer.2.bias"])
        expected = 4 * S
        if self.w("decoder.%d.up0.b" % (stages - 1)).shape[0] not in (expected, expected * cfg["band_kernel"][0]):
            raise ValueError("decoder output width does not match the sources")

    def _window(self, device: torch.device) -> torch.Tensor:
        """The STFT window scaled by n_fft^-1/2 (normalised transforms): ones, or periodic Hann when masked."""
        key = str(device)
        cache = self.__dict__["_win_cache"]
        if key not in cache:
            n = self.config["nfft"]
            w = torch.hann_window(n, periodic=True) if self.masked else torch.ones(n)
            cache[key] = (w / math.sqrt(n)).to(device)
        return cache[key]

    # ------------------------------------------------------------------ blocks
    def _group_norm(self, x: Act, groups: int, rows_per_group: int, name: str, act: int = ACT_NONE,
                    out: torch.Tensor | None = None) -> torch.Tensor:
        """GroupNorm(1) over contiguous groups of ``rows_per_group`` rows of ``x.C`` channels."""
        n = rows_per_group * x.C
        st = self._arena.take(2 * groups, x.t.device)
        _lib.call("unblend_group_sums", x.t.data_ptr(), st.data_ptr(), groups, n)
        s = self._stats(st, groups, n)
        y = torch.empty_like(x.t) if out is None else out
        _lib.call("unblend_group_norm_apply", x.t.data_ptr(), y.data_ptr(), s.data_ptr(), self.w(f"{name}.w").data_ptr(),
                  self.w(f"{name}.b").data_ptr(), groups * rows_per_group, x.C, rows_per_group, act)
        return y

    def _conv_module(self, y: Act, q0: str, depth: int) -> None:
        """ConvolutionModule (unblend/scnet.py:50-97) in place on the band ``y`` [B, F, T, C]."""
        B, Fb, T, C = y.B, y.H, y.W, y.C
        G = B * Fb
        dev = y.t.device
        for d in range(abs(depth)):
            q = f"{q0}.layers.{d}"
            yn = Act(self._group_norm(y, G, T, f"{q}.gn0"), B, Fb, T, C, y.sb, y.sh, y.sw)
            hid = self.w(f"{q}.dw.b").shape[0]
            z = Act.freq(B, Fb, T, hid, dev)
            self._conv(yn, self.w(f"{q}.c1.w"), self.w(f"{q}.c1.b"), z, h_out=Fb, w_out=T, n_out=2 * hid, kw=3,
                       pw=1, act=ACT_GLU)
            u = Act.freq(B, Fb, T, hid, dev)
            st = torch.empty(2 * G, device=dev, dtype=torch.float64)  # written (not accumulated) per row
            _lib.call("unblend_depthwise3", z.t.data_ptr(), self.w(f"{q}.dw.w").data_ptr(),
                      self.w(f"{q}.dw.b").data_ptr(), u.t.data_ptr(), st.data_ptr(), G, T, hid,
                      work=6.0 * G * T * hid)
            s = self._stats(st, G, T * hid)
            _lib.call("unblend_group_norm_apply", u.t.data_ptr(), u.t.data_ptr(), s.data_ptr(),
                      self.w(f"{q}.gn4.w").data_ptr(), self.w(f"{q}.gn4.b").data_ptr(), G * T, hid, T, ACT_SWISH)
            self._conv(u, self.w(f"{q}.c6.w"), self.w(f"{q}.c6.b"), y, h_out=Fb, w_out=T, n_out=C, res=y.t)

    def _encode(self, x: Act, i: int) -> tuple[Act, Act, list[int], list[int]]:
        """SDblock (unblend/scnet.py:238-330): bands, their convolution modules, GELU, global conv."""
        cfg = self.config
        p = f"encoder.{i}"
        B, F, T, Cin = x.B, x.H, x.W, x.C
        Cout = self.dims[i + 1]
        dev = x.t.device
        bands, orig = [], []
        for j, (s0, e0) in enumerate(band_splits(F, cfg["band_SR"])):
            n = e0 - s0
            stride, k = cfg["band_stride"][j], cfg["band_kernel"][j]
            total = k - stride if stride == 1 else (stride - n % stride) % stride
            fo = (n + total - k) // stride + 1
            xb = Act(x.t[s0 * x.sh:], B, n, T, Cin, x.sb, x.sh, x.sw)
            y = Act.freq(B, fo, T, Cout, dev)
            self._conv(xb, self.w(f"{p}.band{j}.w"), self.w(f"{p}.band{j}.b"), y, h_out=fo, w_out=T, n_out=Cout,
                       kh=k, sh=stride, ph=total // 2)
            self._conv_module(y, f"{p}.conv_modules.{j}", cfg["conv_depths"][j])
            bands.append(y)
            orig.append(n)
        lengths = [b.H for b in bands]
        full = Act.freq(B, sum(lengths), T, Cout, dev)
        row = 0
        for y in bands:
            _lib.call("unblend_act_copy", y.t.data_ptr(), y.sb, full.t.data_ptr() + 4 * row * full.sh, full.sb, B,
                      y.sb, ACT_GELU)
            row += y.H
        out = full.like()
        self._conv(full, self.w(f"{p}.global.w"), self.w(f"{p}.global.b"), out, h_out=full.H, w_out=T, n_out=Cout,
                   kh=3, kw=3, ph=1, pw=1)
        return out, full, lengths, orig

    def _lstm_path(self, x: Act, q: str, j: int, along_freq: bool) -> None:
        """One path of DualPathRNN (unblend/scnet.py:475-500): x += Linear(BiLSTM(GroupNorm(x))), in place."""
        B, F, T, d = x.B, x.H, x.W, x.C
        dev = x.t.device
        y = Act(self._group_norm(x, B, F * T, f"{q}.gn{j}"), B, F, T, d, x.sb, x.sh, x.sw)
        hid = self.w(f"{q}.hh{j}").shape[1]
        xp = Act.freq(B, F, T, 8 * hid, dev)
        self._conv(y, self.w(f"{q}.ih{j}.w"), self.w(f"{q}.ih{j}.b"), xp, h_out=F, w_out=T, n_out=8 * hid)
        h = Act.freq(B, F, T, 2 * hid, dev)
        if along_freq:  # sequences (b, t), steps f
            args = (B * T, F, hid, T, F * T, 1, T)
        else:           # sequences (b, f), steps t
            args = (B * F, T, hid, F, F * T, T, 1)
        n_seq, steps = args[0], args[1]
        # bf16 precision: W_hh h on the tensor cores with bf16 operands (hidden 128 / 256).
        rec = "unblend_lstm_recurrence_bf16" if self.precision == "bf16" and hid in (128, 256) else \
            "unblend_lstm_recurrence"
        _lib.call(rec, xp.t.data_ptr(), self.w(f"{q}.hh{j}").data_ptr(), h.t.data_ptr(), *args,
                  work=2.0 * 2 * n_seq * steps * 4 * hid * hid)
        self._conv(h, self.w(f"{q}.lin{j}.w"), self.w(f"{q}.lin{j}.b"), x, h_out=F, w_out=T, n_out=d, res=x.t)

    def _trunk(self, x: Act) -> Act:
        """SeparationNet (unblend/scnet.py:503-540): dual-path layers with real DFTs along frames between them."""
        dev = x.t.device
        for i in range(self.config["num_dplayer"]):
            q = f"separation_net.dp_modules.{i}"
            self._lstm_path(x, q, 0, True)
            self._trace(f"dp{i}_freq", x)
            self._lstm_path(x, q, 1, False)
            self._trace(f"dp{i}_time", x)
            B, F, T, d = x.B, x.H, x.W, x.C
            if i % 2 == 0:
                y = Act.freq(B, F, T // 2 + 1, 2 * d, dev)
                _lib.call("unblend_rfft_time", x.t.data_ptr(), y.t.data_ptr(), B * F, T, d,
                          work=4.0 * B * F * d * T * (T // 2 + 1))
            else:
                c = d // 2
                y = Act.freq(B, F, 2 * (T - 1), c, dev)
                _lib.call("unblend_irfft_time", x.t.data_ptr(), y.t.data_ptr(), B * F, T, c,
                          work=4.0 * B * F * c * T * 2 * (T - 1))
            x = y
            self._trace(f"fc{i}", x)
        return x

    def _decode(self, x: Act, skip: Act, j: int, lengths: list[int], orig: list[int]) -> Act:
        """FusionLayer + SUlayer (unblend/scnet.py:100-235) of decoder stage ``j``."""
        cfg = self.config
        q = f"decoder.{j}"
        B, F, T, C = x.B, x.H, x.W, x.C
        dev = x.t.device
        _lib.call("unblend_add", x.t.data_ptr(), skip.t.data_ptr(), x.t.data_ptr(), x.t.numel(), x.t.numel(), 1.0)
        y = x.like()
        self._conv(x, self.w(f"{q}.fuse.w"), self.w(f"{q}.fuse.b"), y, h_out=F, w_out=T, n_out=2 * C, kh=3, kw=3,
                   ph=1, pw=1, act=ACT_GLU)
        self._trace(f"fuse{j}", y)
        cout = self.w(f"{q}.up0.b").shape[0]
        out = Act.freq(B, sum(orig), T, cout, dev)
        start = off = 0
        for b in range(3):
            n, o = lengths[b], orig[b]
            k, s = cfg["band_kernel"][b], cfg["band_stride"][b]
            xb = Act(y.t[start * y.sh:], B, n, T, C, y.sb, y.sh, y.sw)
            if s == 1:
                ob = Act(out.t[off * out.sh:], B, o, T, cout, out.sb, out.sh, out.sw)
                self._conv(xb, self.w(f"{q}.up{b}.w"), self.w(f"{q}.up{b}.b"), ob, h_out=n, w_out=T, n_out=cout, kh=k,
                           ph=k - 1 - (k - 1) // 2)
            else:
                tmp = Act.freq(B, k * n, T, cout, dev)
                self._conv(xb, self.w(f"{q}.up{b}.w"), self.w(f"{q}.up{b}.b"), tmp, h_out=n, w_out=T, n_out=k * cout,
                           n_group=cout, out_sg=tmp.sh, out_sh=k * tmp.sh)
                dist = abs(o - k * n) // 2
                _lib.call("unblend_act_copy", tmp.t.data_ptr() + 4 * dist * tmp.sh, tmp.sb,
                          out.t.data_ptr() + 4 * off * out.sh, out.sb, B, o * out.sh, ACT_NONE)
            start += n
            off += o
        return out

    # ------------------------------------------------------------------ forward
    #: When set to a dict, ``forward`` stores a CPU copy of every stage output in
    #: the reference's [B, C, F, T] layout (debugging aid, slow).
    trace: dict | None = None

    def _trace(self, name: str, a: Act) -> None:
        if self.trace is not None:
            self.trace[name] = a.t.view(a.B, a.H, a.W, a.C).permute(0, 3, 1, 2).detach().cpu().clone()

    def forward(self, mix: torch.Tensor) -> torch.Tensor:
        """Separate ``mix`` [B, 2, L] into ``[B, S, 2, L]`` (unblend/scnet.py:746-800, 837-895)."""
        if mix.device.type != "cuda":
            raise RuntimeError("SCNetCuda runs on CUDA devices only (no CPU path)")
        wdev = next(iter(self.weights.values())).device
        if wdev != mix.device:
            raise RuntimeError(f"weights are on {wdev}, input on {mix.device}; call .to(device) first")
        if mix.dim() != 3 or mix.shape[1] != 2:
            raise ValueError("stereo input [B, 2, L] expected")
        mix = mix.float().contiguous()
        graphed = self.__dict__.get("_graphed")
        if graphed is not None:
            return graphed(mix)
        return self._forward_arena(mix)

    def _forward_arena(self, mix: torch.Tensor) -> torch.Tensor:
        self._arena.begin(mix.device, mix.shape[0])
        try:
            return self._forward_full(mix)
        finally:
            self._arena.end(mix.device)

    def _forward_full(self, mix: torch.Tensor) -> torch.Tensor:
        cfg = self.config
        B, _, L = mix.shape
        dev = mix.device
        S = len(self.sources)
        nfft, hop = cfg["nfft"], cfg["hop_size"]
        Lp = L + stft_padding(L, hop)
        if Lp <= nfft // 2:
            raise ValueError(f"segment of {L} samples is too short for the {nfft}-point transform")
        padded = torch.empty(B, 2, Lp, device=dev, dtype=torch.float32)
        _lib.call("unblend_pad_tail", mix.data_ptr(), padded.data_ptr(), 2 * B, L, Lp)
        T = 1 + Lp // hop
        Fq = nfft // 2 + 1
        win = self._window(dev)
        frames = torch.empty(B, T, Fq, 4, device=dev, dtype=torch.float32)
        _lib.call("unblend_stft_frames", padded.data_ptr(), frames.data_ptr(), win.data_ptr(), B, Lp, nfft, hop)
        x = Act.freq(B, Fq, T, 4, dev)
        pos = self.w("pos") if self.masked else None
        _lib.call("unblend_swap_axes", frames.data_ptr(), x.t.data_ptr(), _lib.ptr(pos), B, T, Fq, 1)
        self._trace("spec", x)
        skips, lens, origs = [], [], []
        for i in range(len(self.dims) - 1):
            x, skip, lengths, orig = self._encode(x, i)
            self._trace(f"enc{i}", x)
            self._trace(f"skip{i}", skip)
            skips.append(skip)
            lens.append(lengths)
            origs.append(orig)
        x = self._trunk(x)
        self._trace("trunk", x)
        for j in range(len(self.dims) - 1):
            x = self._decode(x, skips.pop(), j, lens.pop(), origs.pop())
            self._trace(f"dec{j}", x)
        if self.masked:
            h = Act.freq(B, Fq, T, 64, dev)
            self._conv(x, self.w("mask0.w"), self.w("mask0.b"), h, h_out=Fq, w_out=T, n_out=64, kh=3, kw=3, ph=1,
                       pw=1, act=ACT_GELU)
            m = Act.freq(B, Fq, T, 4 * S, dev)
            self._conv(h, self.w("mask2.w"), self.w("mask2.b"), m, h_out=Fq, w_out=T, n_out=4 * S)
            _lib.call("unblend_act_copy", m.t.data_ptr(), 0, m.t.data_ptr(), 0, 1, m.t.numel(), ACT_TANH)
            x = m
        per_stem = torch.empty(S, B, T, Fq, 4, device=dev, dtype=torch.float32)
        _lib.call("unblend_swap_axes", x.t.data_ptr(), per_stem.data_ptr(), None, B, Fq, T, S)
        # The inverse transform runs over the padded length (its frame count follows from the
        # length), then the trailing padding is dropped (unblend/scnet.py:783-784).
        full = torch.empty(B, S, 2, Lp, device=dev, dtype=torch.float32)
        fbuf = torch.empty(B * S * 2 * T * nfft, device=dev, dtype=torch.float32)
        _lib.call("unblend_istft_masked", frames.data_ptr() if self.masked else None, per_stem.data_ptr(),
                  B * T * Fq * 4, win.data_ptr(), None, fbuf.data_ptr(), full.data_ptr(), B, S, 0, Lp, nfft, hop, 0)
        out = torch.empty(B, S, 2, L, device=dev, dtype=torch.float32)
        _lib.call("unblend_act_copy", full.data_ptr(), Lp, out.data_ptr(), L, B * S * 2, L, ACT_NONE)
        return out

    # ------------------------------------------------------------------ optional hooks (unblend/backends.py:62-111)
    def enable_compiled_core(self) -> None:
        """Replay the forward from CUDA graphs; tails below 7/8 of the captured batch run eagerly, others are zero-padded."""
        from .graphs import GraphedForward

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


def build_scnet(architecture: str, config: dict, *, sources: list[str], samplerate: int, segment_samples: int,
                state: dict, precision: str = "fp32") -> SCNetCuda:
    """Mirror of the reference ``build_scnet`` (unblend/scnet.py:905-945) for the CUDA model."""
    if architecture not in ("scnet", "scnet_masked"):
        raise ValidationError(f"Unknown SCNet architecture {architecture!r}; expected one of "
                              "['scnet', 'scnet_masked'].")
    cfg = dict(config, architecture=architecture, sources=list(sources), samplerate=samplerate,
               segment_samples=segment_samples)
    return SCNetCuda(cfg, state, precision=precision)
