"""BS-RoFormer forward on B200: the drop-in model for ``apply_model``.

``BSRoformerCuda`` keeps the reference model contract (unblend/roformer.py:896-1379,
unblend/backends.py:36-59): the constructor takes the reference config dict,
``configure_inference(sources=, samplerate=, segment_samples=)`` attaches the
checkpoint interface (including the single-stem mixture-complement output),
``forward(mix[B, C, L]) -> [B, S, C, L]``. Weights come from a reference-layout
``state_dict`` (strict key set) and are repacked once on the device; every step
of ``BSRoformer.forward`` runs as CUDA kernels of ``libunblend_b200.so`` through
its C ABI. There is no CPU path.

Data layout: STFT features are frame-major ``[B, T, F, C, re/im]``, exactly the
reference's ``b t (f c)`` feature rows; band features and the residual stream are
``[B, T, bands, dim]`` fp32, so the time transformer reads sequences along T with
a (batch, band) two-level batch and the frequency transformer reads each frame's
bands as a contiguous sequence -- no transposes between the axial passes.

Precision: ``"bf16"`` runs the linear layers as bf16 tensor-core GEMMs (operands
written as bf16 by the producing kernel, fp32 accumulation, fp32 residual stream)
and attention as single-pass TF32; ``"fp32"`` runs them with the 3-pass TF32 split
(fp32-level accuracy).
"""

from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _lib
from ._lib import ACT_GELU, ACT_GLU, ACT_NONE, ACT_TANH, AttnParams, GemmGroup, GemmParams
from .apply import ValidationError
from .synth import DEFAULT_FREQS_PER_BANDS, MELBAND_DEFAULTS, mel_band_layout

PRECISIONS = ("fp32", "bf16")

_DEFAULTS = dict(
    stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2, linear_transformer_depth=0,
    freqs_per_bands=DEFAULT_FREQS_PER_BANDS, dim_head=64, heads=8, attn_dropout=0.0, ff_dropout=0.0,
    stft_n_fft=2048, stft_hop_length=512, stft_win_length=2048, stft_normalized=False, zero_dc=True,
    mask_estimator_depth=2, mlp_expansion_factor=4, skip_connection=False,
)


def _interleave_glu(w: torch.Tensor) -> torch.Tensor:
    """Rows (value half | gate half) -> (v0, g0, v1, g1, ...) for the GLU epilogue."""
    c = w.shape[0] // 2
    idx = torch.stack([torch.arange(c), torch.arange(c) + c], dim=1).reshape(-1)
    return w[idx].contiguous()


def split_tf32(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``hi`` = w rounded to TF32 (low 13 mantissa bits clear), ``lo`` = w - hi."""
    w = w.float().contiguous()
    hi = ((w.view(torch.int32) + 0x1000) & ~0x1FFF).view(torch.float32)
    return hi.contiguous(), (w - hi).contiguous()


class _Linear:
    """A (possibly grouped) weight matrix in the tensor-core layout of one precision."""

    def __init__(self, w: torch.Tensor, bias: torch.Tensor | None, groups: list[tuple[int, int, int, int, int]],
                 bf16: bool) -> None:
        self.rows, self.cols = w.shape
        if bf16:
            self.hi, self.lo = w.to(torch.bfloat16).contiguous(), None
        else:
            self.hi, self.lo = split_tf32(w)
        self.bias = None if bias is None else bias.float().contiguous()
        self.groups = groups  # (a_col0, w_row0, n, k, out_col0)
        self.flops_per_row = 2.0 * sum(n * k for _, _, n, k, _ in groups)

    def to(self, device) -> "_Linear":
        for name in ("hi", "lo", "bias"):
            t = getattr(self, name)
            if t is not None:
                setattr(self, name, t.to(device))
        return self


class BSRoformerCuda(nn.Module):
    """BS-RoFormer separation forward as sm_100a CUDA kernels.

    :param config: ``BSRoformer`` constructor kwargs (the registry ``config``).
    :param state_dict: Reference-layout weights (strict key set).
    :param precision: ``"bf16"`` or ``"fp32"`` (see the module docstring).
    """

    _defaults = _DEFAULTS
    #: BS-RoFormer applies one shared ``final_norm``; Mel-Band normalises each transformer's output.
    _norm_each_transformer = False

    def _band_bins(self, cfg: dict) -> tuple[int, ...]:
        """Bins per band: the configured contiguous split (unblend/roformer.py:1286-1293)."""
        fpb = tuple(cfg["freqs_per_bands"])
        if len(fpb) < 2 or sum(fpb) != self.n_fft // 2 + 1:
            raise ValidationError(f"freqs_per_bands must sum to {self.n_fft // 2 + 1} for n_fft={self.n_fft}; "
                                  f"got sum {sum(fpb)} over {len(fpb)} bands.")
        return fpb

    @staticmethod
    def _mask_hidden_layers(depth: int) -> int:
        """Hidden layers of a mask MLP: BS-RoFormer's ``depth`` counts Linears (unblend/roformer.py:1302)."""
        return depth - 1

    def __init__(self, config: dict, state_dict: dict, precision: str = "bf16") -> None:
        super().__init__()
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {PRECISIONS}")
        cfg = dict(self._defaults)
        cfg.update(config)
        if cfg["linear_transformer_depth"] != 0:
            raise ValidationError("linear_transformer_depth != 0 is not supported (no shipped checkpoint uses "
                                  "linear attention).")
        self.config = cfg
        self.precision = precision
        self.stereo = bool(cfg["stereo"])
        self.audio_channels = 2 if self.stereo else 1
        if self.audio_channels != 2:
            raise ValueError("only stereo BS-RoFormer models are supported by the CUDA path")
        self.num_stems = cfg["num_stems"]
        self.dim = cfg["dim"]
        self.heads = cfg["heads"]
        self.dim_head = cfg["dim_head"]
        self.n_fft = cfg["stft_n_fft"]
        self.hop = cfg["stft_hop_length"]
        if cfg["stft_win_length"] != self.n_fft or cfg["stft_normalized"] or self.n_fft not in (2048, 4096):
            raise ValueError("the CUDA STFT supports n_fft 2048/4096, win_length == n_fft, not normalised")
        self.freqs_per_bands = self._band_bins(cfg)
        self.widths = [2 * f * self.audio_channels for f in self.freqs_per_bands]
        self.starts = [sum(self.widths[:b]) for b in range(len(self.widths) + 1)]
        self.bands = len(self.widths)
        self.features = self.starts[-1]
        # Band columns of the band-split GEMM operand: each band starts on a
        # 16-byte boundary of its element type (the TMA row offset), so bands
        # whose width is not a multiple of 8 bf16 values get a zero gap.
        align = 8 if precision == "bf16" else 4
        self.kstarts = [0]
        for w in self.widths:
            self.kstarts.append(-(-(self.kstarts[-1] + w) // align) * align)
        self.kfeatures = self.kstarts[-1]
        # Interface defaults until configure_inference (unblend/roformer.py:1003-1006).
        self.sources = [f"stem_{i}" for i in range(self.num_stems)]
        self.output_complement = False
        # Mel-Band: iSTFT to the exact input length (else to hop * (frames - 1));
        # configure_inference turns it on (unblend/roformer.py:1064, 1524).
        self.match_input_audio_length = bool(cfg.get("match_input_audio_length", False))
        self._fixed_batch_shape = False
        self._eager_tails = False
        self._pack(state_dict)
        self._device = torch.device("cpu")

    # ------------------------------------------------------------------ contract
    @classmethod
    def from_reference(cls, module: nn.Module, config: dict, precision: str = "bf16") -> "BSRoformerCuda":
        """Build from a reference ``BSRoformer`` (its constructor config and state), copying its interface."""
        out = cls(config, module.state_dict(), precision=precision)
        if hasattr(module, "samplerate"):
            out.configure_inference(sources=list(module.sources), samplerate=module.samplerate,
                                    segment_samples=int(round(module.max_allowed_segment * module.samplerate)))
        return out

    def configure_inference(self, *, sources: list[str], samplerate: int, segment_samples: int) -> None:
        """Attach the checkpoint interface (unblend/roformer.py:1008-1064), same validation and semantics."""
        if isinstance(samplerate, bool) or not isinstance(samplerate, int) or samplerate <= 0:
            raise ValidationError(f"samplerate must be a positive integer, got {samplerate}")
        if isinstance(segment_samples, bool) or not isinstance(segment_samples, int) or segment_samples <= 0:
            raise ValidationError(f"segment_samples must be a positive integer, got {segment_samples}")
        if len(sources) == self.num_stems:
            self.output_complement = False
        elif self.num_stems == 1 and len(sources) == 2:
            self.output_complement = True
        else:
            raise ValidationError(f"{len(sources)} source names for a model with {self.num_stems} mask head(s); "
                                  f"expected {self.num_stems} or, for single-stem models, 2.")
        self.sources = list(sources)
        self.samplerate = samplerate
        self.max_allowed_segment = segment_samples / samplerate
        self.match_input_audio_length = True

    def to(self, device, *args, **kwargs):  # noqa: D401 - nn.Module signature
        """Move the packed weights to ``device``."""
        device = torch.device(device)
        for lin in self._linears():
            lin.to(device)
        for k, v in list(self._vec.items()):
            self._vec[k] = v.to(device)
        self._device = device
        self.__dict__["_table_cache"] = {}
        return self

    def cuda(self, device=None):
        return self.to(torch.device("cuda", torch.cuda.current_device() if device is None else device))

    def eval(self):
        return self

    # ------------------------------------------------------------------ weights
    def _pack(self, sd: dict) -> None:
        sd = {k: v.detach().float().cpu() for k, v in sd.items()}
        cfg = self.config
        bf16 = self.precision == "bf16"
        dim, inner = self.dim, self.heads * self.dim_head
        self._vec: dict[str, torch.Tensor] = {}
        self._lin: dict[str, _Linear] = {}
        self._rope_freqs: dict[int, torch.Tensor] = {}
        for i in range(cfg["depth"]):
            for axis, tdepth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
                for j in range(tdepth):
                    p = f"layers.{i}.{axis}.layers.{j}"
                    self._vec[f"{p}.attn.gamma"] = sd[f"{p}.0.norm.gamma"]
                    self._vec[f"{p}.gates.w"] = sd[f"{p}.0.to_gates.weight"]
                    self._vec[f"{p}.gates.b"] = sd[f"{p}.0.to_gates.bias"]
                    self._rope_freqs.setdefault(axis, sd[f"{p}.0.rotary_embed.freqs"])
                    self._lin[f"{p}.qkv"] = _Linear(sd[f"{p}.0.to_qkv.weight"], None,
                                                    [(0, 0, 3 * inner, dim, 0)], bf16)
                    self._lin[f"{p}.out"] = _Linear(sd[f"{p}.0.to_out.0.weight"], None,
                                                    [(0, 0, dim, inner, 0)], bf16)
                    self._vec[f"{p}.ff.gamma"] = sd[f"{p}.1.net.0.gamma"]
                    w1, w2 = sd[f"{p}.1.net.1.weight"], sd[f"{p}.1.net.4.weight"]
                    self._lin[f"{p}.ff1"] = _Linear(w1, sd[f"{p}.1.net.1.bias"], [(0, 0, w1.shape[0], dim, 0)], bf16)
                    self._lin[f"{p}.ff2"] = _Linear(w2, sd[f"{p}.1.net.4.bias"], [(0, 0, dim, w2.shape[1], 0)],
                                                    bf16)
        if self._norm_each_transformer:
            for i in range(cfg["depth"]):
                for axis in (0, 1):
                    self._vec[f"layers.{i}.{axis}.norm.gamma"] = sd[f"layers.{i}.{axis}.norm.gamma"]
        else:
            self._vec["final_norm.gamma"] = sd["final_norm.gamma"]
        # BandSplit: band b's Linear(w_b -> dim) as rows [b*dim, (b+1)*dim) of one
        # zero-padded weight matrix; its RMSNorm gains back to back.
        kpad = -(-max(self.widths) // 64) * 64
        wbs = torch.zeros(self.bands * dim, kpad)
        bbs = torch.zeros(self.bands * dim)
        groups = []
        for b, w in enumerate(self.widths):
            wbs[b * dim:(b + 1) * dim, :w] = sd[f"band_split.to_features.{b}.1.weight"]
            bbs[b * dim:(b + 1) * dim] = sd[f"band_split.to_features.{b}.1.bias"]
            groups.append((self.kstarts[b], b * dim, dim, w, b * dim))
        self._vec["band.gamma"] = torch.cat([sd[f"band_split.to_features.{b}.0.gamma"] for b in range(self.bands)])
        self._vec["band.starts"] = torch.tensor(self.starts, dtype=torch.int32)
        self._vec["band.kstarts"] = torch.tensor(self.kstarts, dtype=torch.int32)
        self._lin["band_split"] = _Linear(wbs, bbs, groups, bf16)
        # MaskEstimator per stem: hidden layers (tanh) as grouped GEMMs with
        # one group per band, then the GLU output layer whose band b writes
        # feature columns [start_b, start_b + w_b) of the mask.
        n_hidden = self._mask_hidden_layers(cfg["mask_estimator_depth"])
        hidden = dim * cfg["mlp_expansion_factor"]
        self.mask_layers: list[list[str]] = []
        for s in range(self.num_stems):
            names = []
            a_in = dim
            for k in range(n_hidden):
                ws = torch.cat([sd[f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}.weight"] for b in range(self.bands)])
                bs = torch.cat([sd[f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}.bias"] for b in range(self.bands)])
                groups = [(b * a_in, b * hidden, hidden, a_in, b * hidden) for b in range(self.bands)]
                name = f"mask.{s}.{k}"
                self._lin[name] = _Linear(ws, bs, groups, bf16)
                names.append(name)
                a_in = hidden
            k = n_hidden
            ws, bs, groups, row = [], [], [], 0
            for b, w in enumerate(self.widths):
                ws.append(_interleave_glu(sd[f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}.weight"]))
                bs.append(_interleave_glu(sd[f"mask_estimators.{s}.to_freqs.{b}.0.{2 * k}.bias"][:, None])[:, 0])
                groups.append((b * a_in, row, 2 * w, a_in, self.starts[b]))
                row += 2 * w
            name = f"mask.{s}.out"
            self._lin[name] = _Linear(torch.cat(ws), torch.cat(bs), groups, bf16)
            names.append(name)
            self.mask_layers.append(names)

    def _linears(self):
        return self._lin.values()

    def _tables(self, T: int) -> dict:
        """Window and rotary (cos, sin) tables for T frames, cached per device."""
        cache = self.__dict__.setdefault("_table_cache", {})
        key = (str(self._device), T)
        if key not in cache:
            tabs = {"window": torch.hann_window(self.n_fft).to(self._device)}
            for axis, seq in ((0, T), (1, self.bands)):
                freqs = self._rope_freqs[axis].float()
                angles = torch.arange(seq, dtype=torch.float32)[:, None] * freqs
                tabs[f"rope{axis}"] = torch.stack([angles.cos(), angles.sin()], dim=-1).contiguous().to(self._device)
            cache[key] = tabs
        return cache[key]

    # ------------------------------------------------------------------ launch helpers
    def _gemm(self, lin: _Linear, a: torch.Tensor, lda: int, rows: int, a_cols: int, out: torch.Tensor, ldo: int,
              act: int = ACT_NONE, res: torch.Tensor | None = None, block_n: int = 256,
              rope: tuple | None = None) -> None:
        mode = _lib.TC_BF16 if self.precision == "bf16" else _lib.TC_TF32X3
        for g0 in range(0, len(lin.groups), _lib.GEMM_MAX_GROUPS):
            chunk = lin.groups[g0:g0 + _lib.GEMM_MAX_GROUPS]
            arr = (GemmGroup * len(chunk))(*[GemmGroup(*g) for g in chunk])
            p = GemmParams()
            p.groups = len(chunk)
            p.group = ctypes.cast(arr, ctypes.POINTER(GemmGroup))
            p.bias = _lib.ptr(lin.bias)
            p.act = act
            p.res = _lib.ptr(res)
            p.ldr = ldo if res is not None else 0
            p.out = out.data_ptr()
            p.ldo = ldo
            p.out_bf16 = 1 if out.dtype == torch.bfloat16 else 0
            if rope is not None:
                table, p.rope_cols, p.rope_hd, p.rope_div, p.rope_mod = rope
                p.rope = table.data_ptr()
            work = rows * 2.0 * sum(n * k for _, _, n, k, _ in chunk)
            _lib.call("unblend_gemm_tc", a.data_ptr(), lda, rows, a_cols, lin.hi.data_ptr(), _lib.ptr(lin.lo),
                      lin.rows, lin.cols, ctypes.byref(p), mode, block_n, work=work)

    def _act_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.precision == "bf16" else torch.float32

    def _attention_layer(self, x: torch.Tensor, p: str, axis: int, B: int, T: int, tabs: dict) -> None:
        """x += Attention(x) (unblend/roformer.py:478-511) over the time (axis 0) or band (axis 1) sequences."""
        nb, dim, H, hd = self.bands, self.dim, self.heads, self.dim_head
        inner = H * hd
        rows = B * T * nb
        dev = x.device
        xn = torch.empty(rows, dim, device=dev, dtype=self._act_dtype())
        gates = torch.empty(rows, H, device=dev, dtype=torch.float32)
        _lib.call("unblend_rms_norm", x.data_ptr(), rows, dim, self._vec[f"{p}.attn.gamma"].data_ptr(),
                  xn.data_ptr(), dim, 1 if xn.dtype == torch.bfloat16 else 0, self._vec[f"{p}.gates.w"].data_ptr(),
                  self._vec[f"{p}.gates.b"].data_ptr(), H, gates.data_ptr())
        bf16 = self.precision == "bf16" and hd == 64
        seq = T if axis == 0 else nb
        rope = tabs[f"rope{axis}"]
        qkv = torch.empty(rows, 3 * inner, device=dev, dtype=torch.bfloat16 if bf16 else torch.float32)
        # bf16 path: the rotary rotation of Q and K is applied in the projection's epilogue.
        self._gemm(self._lin[f"{p}.qkv"], xn, dim, rows, dim, qkv, 3 * inner,
                   rope=(rope, 2 * inner, hd, nb if axis == 0 else 1, seq) if bf16 else None)
        o = torch.empty(rows, inner, device=dev, dtype=self._act_dtype())
        a = AttnParams()
        a.heads, a.hd = H, hd
        q3 = 3 * inner
        if axis == 0:  # sequences along frames, batch (b, band)
            a.outer, a.inner, a.lq, a.lk = B, nb, T, T
            a.q_so, a.q_si, a.q_sr = T * nb * q3, q3, nb * q3
            a.o_so, a.o_si, a.o_sr = T * nb * inner, inner, nb * inner
            a.g_so, a.g_si, a.g_sr = T * nb * H, H, nb * H
        else:  # sequences along bands, batch (b, frame)
            a.outer, a.inner, a.lq, a.lk = B * T, 1, nb, nb
            a.q_so, a.q_si, a.q_sr = nb * q3, 4, q3
            a.o_so, a.o_si, a.o_sr = nb * inner, 0, inner
            a.g_so, a.g_si, a.g_sr = nb * H, 0, H
            if bf16:
                a.q_si = 8
        a.kv_so, a.kv_si, a.kv_sr = a.q_so, a.q_si, a.q_sr
        a.out = o.data_ptr()
        a.out_bf16 = 1 if o.dtype == torch.bfloat16 else 0
        a.gate = gates.data_ptr()
        a.scale = hd ** -0.5
        base = qkv.data_ptr()
        work = 4.0 * a.outer * a.inner * H * seq * seq * hd
        if bf16:
            a.kv_si = a.q_si
            _lib.call("unblend_attention_bf16", base, base + 2 * inner, base + 4 * inner, ctypes.byref(a), work=work)
        else:
            a.rope = rope.data_ptr()
            a.rope_len = seq
            mode = 1 if self.precision == "bf16" else 0
            _lib.call("unblend_attention_tc2", base, base + 4 * inner, base + 8 * inner, ctypes.byref(a), mode,
                      work=work)
        self._gemm(self._lin[f"{p}.out"], o, inner, rows, inner, x, dim, res=x)

    def _ff_layer(self, x: torch.Tensor, p: str, rows: int) -> None:
        """x += FeedForward(x) (unblend/roformer.py:274-308)."""
        dim = self.dim
        dev = x.device
        xn = torch.empty(rows, dim, device=dev, dtype=self._act_dtype())
        _lib.call("unblend_rms_norm", x.data_ptr(), rows, dim, self._vec[f"{p}.ff.gamma"].data_ptr(), xn.data_ptr(),
                  dim, 1 if xn.dtype == torch.bfloat16 else 0, None, None, 0, None)
        lin1 = self._lin[f"{p}.ff1"]
        hidden = lin1.rows
        h = torch.empty(rows, hidden, device=dev, dtype=self._act_dtype())
        self._gemm(lin1, xn, dim, rows, dim, h, hidden, act=ACT_GELU)
        self._gemm(self._lin[f"{p}.ff2"], h, hidden, rows, hidden, x, dim, res=x)

    # ------------------------------------------------------------------ forward
    def forward(self, mix: torch.Tensor) -> torch.Tensor:
        """Separate ``mix`` [B, C, L] into ``[B, S, C, L]`` (unblend/roformer.py:1312-1379)."""
        if mix.device.type != "cuda":
            raise RuntimeError("BSRoformerCuda runs on CUDA devices only (no CPU path)")
        if self._device != mix.device:
            raise RuntimeError(f"weights are on {self._device}, input on {mix.device}; call .to(device) first")
        if mix.dim() != 3:
            raise ValidationError("expected a [batch, channels, samples] mixture")
        B, C, L = mix.shape
        if C != self.audio_channels:
            raise ValidationError(f"Model expects {self.audio_channels} channel(s) (stereo={self.stereo}), got {C}.")
        if L <= self.n_fft // 2:
            raise ValueError(f"input of {L} samples is too short for a {self.n_fft}-point centred STFT")
        in_dtype = mix.dtype
        mix = mix.float().contiguous()
        graphed = self.__dict__.get("_graphed")
        out = graphed(mix) if graphed is not None else self._forward_impl(mix)
        return out if in_dtype == torch.float32 else out.to(in_dtype)

    # ------------------------------------------------------------------ optional hooks (unblend/backends.py:62-111)
    #: The RoFormer calibrator sweeps power-of-two batches (unblend/roformer.py:1075-1078).
    prefers_power_of_two_batch = True
    #: RoFormer consumes the raw mixture (no track-level normalisation by the caller).
    external_normalization = False

    def prefill_inference_caches(self) -> None:
        """Build the window and rotary tables of the configured segment before any graph capture."""
        if self._device.type == "cuda" and hasattr(self, "samplerate"):
            seg = int(round(self.max_allowed_segment * self.samplerate))
            self._tables(1 + seg // self.hop)

    def enable_compiled_core(self) -> None:
        """Replay the forward from CUDA graphs; tails below 7/8 of the captured batch run eagerly, others are zero-padded."""
        from .graphs import GraphedForward

        self.prefill_inference_caches()
        self.__dict__["_graphed"] = GraphedForward(self._forward_impl)
        self._fixed_batch_shape = True
        self._eager_tails = True

    def disable_compiled_core(self) -> None:
        """Back to eager launches; releases the captured graphs."""
        graphed = self.__dict__.pop("_graphed", None)
        if graphed is not None:
            graphed.release()
        self._fixed_batch_shape = False
        self._eager_tails = False

    def _forward_impl(self, mix: torch.Tensor) -> torch.Tensor:
        """The forward on a contiguous fp32 ``[B, 2, L]`` CUDA mixture."""
        B, C, L = mix.shape
        dev = mix.device
        cfg = self.config
        T = 1 + L // self.hop
        nb, dim = self.bands, self.dim
        Fb = self.n_fft // 2 + 1
        tabs = self._tables(T)
        stft = torch.empty(B, T, Fb, 2, 2, device=dev, dtype=torch.float32)
        _lib.call("unblend_stft_frames", mix.data_ptr(), stft.data_ptr(), tabs["window"].data_ptr(), B, L,
                  self.n_fft, self.hop)
        frames = B * T
        # BandSplit: per-band RMSNorm, then the grouped per-band Linear.
        ldf = self.kfeatures if self.precision == "fp32" else -(-self.kfeatures // 8) * 8
        gaps = self.kstarts != self.starts
        # The GEMM reads past each band into its neighbour (zero weights there), so gaps must hold zeros.
        feats = (torch.zeros if gaps else torch.empty)(frames, ldf, device=dev, dtype=self._act_dtype())
        starts = self._vec["band.starts"]
        band_in = self._band_input(stft, frames)
        _lib.call("unblend_band_rms_norm", band_in.data_ptr(), frames, band_in.shape[-1], starts.data_ptr(), nb,
                  self._vec["band.gamma"].data_ptr(), feats.data_ptr(), ldf,
                  1 if feats.dtype == torch.bfloat16 else 0, self._vec["band.kstarts"].data_ptr() if gaps else None)
        x = torch.empty(frames * nb, dim, device=dev, dtype=torch.float32)
        self._gemm(self._lin["band_split"], feats, ldf, frames, self.kfeatures, x, nb * dim)
        # Axial transformers (unblend/roformer.py:1135-1159).
        rows = frames * nb
        store: list[torch.Tensor] = []
        for i in range(cfg["depth"]):
            if cfg["skip_connection"]:
                for prev in store:
                    _lib.call("unblend_add", x.data_ptr(), prev.data_ptr(), x.data_ptr(), x.numel(), x.numel(), 1.0)
            for axis, tdepth in ((0, cfg["time_transformer_depth"]), (1, cfg["freq_transformer_depth"])):
                for j in range(tdepth):
                    p = f"layers.{i}.{axis}.layers.{j}"
                    self._attention_layer(x, p, axis, B, T, tabs)
                    self._ff_layer(x, p, rows)
                last = i == cfg["depth"] - 1 and axis == 1
                if self._norm_each_transformer and not last:
                    # Transformer output RMSNorm (unblend/roformer.py:658, 670), fp32 stream.
                    xn = torch.empty_like(x)
                    _lib.call("unblend_rms_norm", x.data_ptr(), rows, dim,
                              self._vec[f"layers.{i}.{axis}.norm.gamma"].data_ptr(), xn.data_ptr(), dim, 0, None,
                              None, 0, None)
                    x = xn
            if cfg["skip_connection"]:
                store.append(x.clone())
        # The last normalisation (BS: final_norm; Mel-Band: the last transformer's
        # output norm) writes the mask estimators' operand directly.
        last_gamma = (f"layers.{cfg['depth'] - 1}.1.norm.gamma" if self._norm_each_transformer
                      else "final_norm.gamma")
        xf = torch.empty(rows, dim, device=dev, dtype=self._act_dtype())
        _lib.call("unblend_rms_norm", x.data_ptr(), rows, dim, self._vec[last_gamma].data_ptr(),
                  xf.data_ptr(), dim, 1 if xf.dtype == torch.bfloat16 else 0, None, None, 0, None)
        # Mask estimators: [stems, frames, features] complex masks (fp32).
        S = self.num_stems
        mask = torch.empty(S, frames, self.features, device=dev, dtype=torch.float32)
        for s, names in enumerate(self.mask_layers):
            h, ld = xf, nb * dim
            for name in names[:-1]:
                lin = self._lin[name]
                width = lin.rows
                nxt = torch.empty(frames, width, device=dev, dtype=self._act_dtype())
                self._gemm(lin, h, ld, frames, ld, nxt, width, act=ACT_TANH)
                h, ld = nxt, width
            self._gemm(self._lin[names[-1]], h, ld, frames, ld, mask[s], self.features, act=ACT_GLU, block_n=64)
        mask, mask_ld = self._bin_masks(mask, S, frames)
        # Complex masking, DC zeroing, iSTFT, optional complement stem.
        comp = 1 if self.output_complement else 0
        out_len = self._output_length(L)
        out = torch.empty(B, S + comp, 2, out_len, device=dev, dtype=torch.float32)
        fbuf = torch.empty(B * S * 2 * T * self.n_fft, device=dev, dtype=torch.float32)
        _lib.call("unblend_istft_masked", stft.data_ptr(), mask.data_ptr(), frames * mask_ld,
                  tabs["window"].data_ptr(), mix.data_ptr(), fbuf.data_ptr(), out.data_ptr(), B, S, comp, out_len,
                  self.n_fft, self.hop, 1 if cfg["zero_dc"] else 0)
        return out

    # ------------------------------------------------------------------ band layout hooks
    def _band_input(self, stft: torch.Tensor, frames: int) -> torch.Tensor:
        """BandSplit input rows: the STFT feature rows themselves (contiguous bands)."""
        return stft.view(frames, -1)

    def _bin_masks(self, mask: torch.Tensor, S: int, frames: int) -> tuple[torch.Tensor, int]:
        """Per-bin masks for the iSTFT: the band masks already are (contiguous bands)."""
        return mask, self.features

    def _output_length(self, L: int) -> int:
        return L


class MelBandRoformerCuda(BSRoformerCuda):
    """Mel-Band RoFormer forward (unblend/roformer.py:1382-1603) on the BS-RoFormer kernels.

    The bands are the supports of a Slaney mel filter bank and overlap, so the
    band features are gathered from the STFT rows through an index list
    (``unblend_gather_pairs``) and the per-band masks are summed back onto the
    bins and divided by each bin's band count (``unblend_scatter_mean_pairs``)
    before the shared masking iSTFT. Each axial transformer ends with its own
    RMSNorm (no shared ``final_norm``), and the mask MLPs have
    ``mask_estimator_depth`` hidden layers.
    """

    _defaults = MELBAND_DEFAULTS
    _norm_each_transformer = True

    def _band_bins(self, cfg: dict) -> tuple[int, ...]:
        try:
            idx, per_band, per_bin = mel_band_layout(cfg["sample_rate"], self.n_fft, cfg["num_bands"],
                                                     bool(cfg["stereo"]))
        except ValueError as e:
            raise ValidationError("Invalid mel banding: every frequency bin must be covered by at least one "
                                  "band.") from e
        # Gather list and its inverse (destination pair -> gathered positions, ascending).
        self._mel_idx = idx.to(torch.int32)
        order = torch.argsort(idx, stable=True)
        counts = torch.bincount(idx, minlength=(self.n_fft // 2 + 1) * self.audio_channels)
        self._mel_pos = order.to(torch.int32)
        self._mel_off = torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]).to(torch.int32)
        self.bands_per_bin = per_bin
        return tuple(int(v) for v in per_band.tolist())

    @staticmethod
    def _mask_hidden_layers(depth: int) -> int:
        """Mel-Band's ``depth`` counts hidden layers (``depth + 1`` Linears, unblend/roformer.py:1494-1496)."""
        return depth

    def to(self, device, *args, **kwargs):
        super().to(device, *args, **kwargs)
        for name in ("_mel_idx", "_mel_pos", "_mel_off"):
            setattr(self, name, getattr(self, name).to(self._device))
        return self

    def _band_input(self, stft: torch.Tensor, frames: int) -> torch.Tensor:
        g = torch.empty(frames, self.features, device=stft.device, dtype=torch.float32)
        fb4 = stft.shape[2] * 4
        _lib.call("unblend_gather_pairs", stft.data_ptr(), fb4, frames, self._mel_idx.data_ptr(),
                  self._mel_idx.numel(), g.data_ptr(), self.features)
        return g

    def _bin_masks(self, mask: torch.Tensor, S: int, frames: int) -> tuple[torch.Tensor, int]:
        n_bins = (self.n_fft // 2 + 1) * self.audio_channels
        dense = torch.empty(S, frames, 2 * n_bins, device=mask.device, dtype=torch.float32)
        _lib.call("unblend_scatter_mean_pairs", mask.data_ptr(), self.features, S * frames,
                  self._mel_off.data_ptr(), self._mel_pos.data_ptr(), n_bins, dense.data_ptr(), 2 * n_bins)
        return dense, 2 * n_bins

    def _output_length(self, L: int) -> int:
        """torch.istft without ``length`` stops at hop * (frames - 1) unless the model matches the input."""
        return L if self.match_input_audio_length else self.hop * (L // self.hop)


_CUDA_ARCHITECTURES = {"bs_roformer": BSRoformerCuda, "mel_band_roformer": MelBandRoformerCuda}


def build_roformer(architecture: str, config: dict, *, sources: list[str], samplerate: int, segment_samples: int,
                   state: dict, precision: str = "bf16") -> BSRoformerCuda:
    """Counterpart of ``unblend.roformer.build_roformer`` (unblend/roformer.py:1606-1643) for the CUDA path."""
    if architecture not in _CUDA_ARCHITECTURES:
        raise ValidationError(f"architecture {architecture!r} is not built on the CUDA path "
                              f"({', '.join(_CUDA_ARCHITECTURES)})")
    model = _CUDA_ARCHITECTURES[architecture](config, state, precision=precision)
    model.configure_inference(sources=sources, samplerate=samplerate, segment_samples=segment_samples)
    return model
