"""Shared machinery of the convolutional models: channels-last activation views,
the per-forward statistics arena and the convolution launcher that picks the
tcgen05 tensor-core kernel or the CUDA-core one for each layer.

``ConvNet`` holds a model's repacked weights (``nn.ParameterDict``) and turns
a convolution described on :class:`Act` views into one ``UnblendConvParams``
launch of ``libunblend_b200.so``: the tensor-core kernel (3-pass TF32 in fp32
precision, bf16 operands in bf16 precision) when the layer meets its layout
rules, else the fp32 SIMT kernel. There is no PyTorch fallback.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import nn

from . import _lib
from ._lib import ACT_GLU, ACT_NONE, PRO_ADD, PRO_NONE, ConvParams


def _key(name: str) -> str:
    return name.replace(".", "__")


@dataclass
class Act:
    """A channels-last activation view: ``t`` holds [B, H, W, C] with strides sb/sh/sw."""

    t: torch.Tensor
    B: int
    H: int
    W: int
    C: int
    sb: int
    sh: int
    sw: int

    @staticmethod
    def freq(B: int, F: int, T: int, C: int, device) -> "Act":
        t = torch.empty(B * F * T * C, device=device, dtype=torch.float32)
        return Act(t, B, F, T, C, F * T * C, T * C, C)

    @staticmethod
    def time(B: int, rows: int, cap: int, C: int, device) -> "Act":
        t = torch.empty(B * cap * C, device=device, dtype=torch.float32)
        return Act(t, B, 1, rows, C, cap * C, cap * C, C)

    def like(self) -> "Act":
        return Act(torch.empty_like(self.t), self.B, self.H, self.W, self.C, self.sb, self.sh, self.sw)


class StatsArena:
    """The float64 GroupNorm / DConv statistics sums of one forward, zeroed by one launch.

    Every statistics buffer of a forward is a slice of one device buffer per
    (device, batch) key, zeroed by a single ``unblend_zero_f64`` at the start of
    the forward instead of one fill per buffer. The first forward of a key
    learns the size it needs (its slices are separate zeroed buffers); later
    forwards of that key take slices of the arena. Arenas are never freed while
    the model lives, so captured CUDA graphs can keep referring to them.
    """

    def __init__(self) -> None:
        self.bufs: dict = {}
        self.retired: list = []
        self.key = None
        self.cur: torch.Tensor | None = None
        self.pos = 0

    def begin(self, device: torch.device, batch: int) -> None:
        self.key = (str(device), batch)
        self.cur = self.bufs.get(self.key)
        self.pos = 0
        if self.cur is not None:
            _lib.call("unblend_zero_f64", self.cur.data_ptr(), self.cur.numel())

    def take(self, n: int, device: torch.device) -> torch.Tensor:
        """``n`` zeroed doubles on ``device`` (16-byte aligned slices of the arena inside a forward)."""
        size = n + (n & 1)
        if self.cur is not None and self.cur.device == device and self.pos + size <= self.cur.numel():
            t = self.cur[self.pos:self.pos + n]
        else:
            t = torch.empty(size, device=device, dtype=torch.float64)
            _lib.call("unblend_zero_f64", t.data_ptr(), size)
            t = t[:n]
        if self.key is not None:
            self.pos += size
        return t

    def end(self, device: torch.device) -> None:
        if self.cur is None or self.cur.numel() < self.pos:
            if self.cur is not None:
                self.retired.append(self.cur)
            self.bufs[self.key] = torch.empty(max(self.pos, 2), device=device, dtype=torch.float64)
        self.cur = None
        self.key = None


def _interleave_rows(t: torch.Tensor) -> torch.Tensor:
    """Reorder the 2C output rows (value half, gate half) to (v0, g0, v1, g1, ...)."""
    c = t.shape[0] // 2
    idx = torch.stack([torch.arange(c), torch.arange(c) + c], dim=1).reshape(-1)
    return t[idx].contiguous()


def _conv_w(w: torch.Tensor) -> torch.Tensor:
    """Conv weight to [Cout, KH, KW, Cin] (Conv1d kernels become KH=1)."""
    if w.dim() == 3:
        return w.permute(0, 2, 1).unsqueeze(1).contiguous()
    return w.permute(0, 2, 3, 1).contiguous()


def split_tf32(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Split fp32 ``w`` into ``hi`` (rounded to TF32, low 13 mantissa bits clear) and ``lo = w - hi``."""
    w = w.float().contiguous()
    hi = ((w.view(torch.int32) + 0x1000) & ~0x1FFF).view(torch.float32)
    return hi.contiguous(), (w - hi).contiguous()


def split_bf16(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Split fp32 ``w`` into bf16 ``hi`` = round(w) and ``lo`` = round(w - hi) (round to nearest even)."""
    w = w.float().contiguous()
    hi = w.to(torch.bfloat16)
    return hi.contiguous(), (w - hi.float()).to(torch.bfloat16).contiguous()


PRECISIONS = ("fp32", "bf16", "fp32-simt")


def _m_tiles(batch: int, h_out: int, w_out: int) -> int:
    """128-row output tiles of the tensor-core convolution (rows of W split into 128s, or into the
    largest multiple of 8 in [64, 128] that divides W when 128 does not, e.g. 336 = 3 x 112)."""
    mv = 128
    if w_out % 128 and h_out > 1:
        mv = next((m for m in range(128, 63, -8) if w_out % m == 0), 128)
    return batch * h_out * -(-w_out // mv)


def _block_n(n_out: int, bn256_min: int, m_tiles: int = 1 << 20, sms: int = 148, max_bn: int = 256) -> int:
    """Output-channel tile of the tensor-core convolution.

    Candidates 64, 96, 128, 192 (and 256 from ``bn256_min`` channels on). The persistent
    kernel runs ``m_tiles * ceil(n_out / bn)`` tiles over ``sms`` CTAs, so a launch costs
    about ceil(tiles / sms) waves of (64 + bn) column-units per tile (the MMA issue time
    of a 128-row tile: ~48 cycles per instruction at N = 64 against 128 at N = 256, and
    the width-independent A loads and operand conversion). The cheapest candidate wins,
    ties going to the wider tile (fewer re-reads of the input rows): with many tiles that
    is the fewest padded columns; with few (small batches) it trades width for fuller waves.
    """
    cands = [bn for bn in [64, 96, 128, 192] + ([256] if n_out >= bn256_min else []) if bn <= max_bn]
    best = None
    for bn in cands:
        tiles = m_tiles * -(-n_out // bn)
        key = (-(-tiles // sms) * (64 + bn), -bn)
        if best is None or key < best[0]:
            best = (key, bn)
    return best[1]


def _subtaps_pay(n_out: int, bn256_min: int) -> bool:
    """Whether a 3-wide kernel row of the 3-pass bf16 split runs faster with its three taps sharing one
    A load and operand split (tiles of <= 128 columns) than on the widest tiles without sharing.

    Worth it up to 1.5x the tiles of the widest choice (HTDemucs decoder 3x3 rewrites at 32 segments:
    48 -> 96 channels 3.37 -> 2.33 ms, 192 -> 384 1.59 -> 1.36 ms; not 96 -> 192 on 96-column tiles,
    1.63 -> 1.73 ms, nor 384 -> 768 on 128-column tiles, 1.22 -> 1.37 ms). Depends on the layer only.
    """
    full = -(-n_out // _block_n(n_out, bn256_min))
    shared = -(-n_out // _block_n(n_out, bn256_min, max_bn=128))
    return 2 * shared <= 3 * full


class ConvNet(nn.Module):
    """Weights and convolution launches shared by the HTDemucs and SCNet models.

    :param precision: ``"fp32"`` (3-pass tensor-core layers, operands split into
        hi / lo parts), ``"bf16"``
        (bf16 tensor-core operands, fp32 accumulation and activations) or
        ``"fp32-simt"`` (CUDA-core fp32 kernels only).
    """

    def __init__(self, precision: str = "fp32") -> None:
        super().__init__()
        if precision not in PRECISIONS:
            raise ValueError(f"precision must be one of {PRECISIONS}")
        self.precision = precision
        self._tc_cache: dict = {}
        self._sm_count: dict = {}
        # Output widths from which the 256-column tile is used (per tensor-core mode).
        self._bn256_min = {_lib.TC_TF32X3: 512, _lib.TC_BF16: 512, _lib.TC_BF16X3: 512}
        # Operand split of the fp32 tensor-core convolutions: "bf16x3" (hi/lo bf16
        # parts, kind::f16: 16 K channels per MMA, on tiles of 192 and 256 columns)
        # or "tf32x3" (hi/lo TF32 parts, kind::tf32: 8 per MMA, every tile). Both
        # hold the fp32 parity bound on the registry models; bf16x3 issues half the MMAs.
        self.fp32_split = "bf16x3"
        # With the bf16x3 split, 3-wide kernel rows (stride 1) run on tiles of <= 128
        # columns whose three taps share one A load and one operand split, where that pays.
        self.fp32_subtaps = True
        self.weights = nn.ParameterDict()
        self._arena = StatsArena()

    def _put(self, name: str, t: torch.Tensor) -> None:
        self.weights[_key(name)] = nn.Parameter(t.detach().float().contiguous().clone(), requires_grad=False)

    def w(self, name: str) -> torch.Tensor:
        return self.weights[_key(name)]

    # ------------------------------------------------------------------ launch helpers
    def _conv(self, x: Act, w: torch.Tensor, b: torch.Tensor | None, out: Act, *, h_out: int, w_out: int,
              n_out: int, kh: int = 1, kw: int = 1, sh: int = 1, sw: int = 1, dh: int = 1, dw: int = 1,
              ph: int = 0, pw: int = 0, act: int = ACT_NONE, prologue: int = PRO_NONE,
              pro_stats: torch.Tensor | None = None, pro_gamma=None, pro_beta=None, pro_per_h: int = 0,
              pro_x2: Act | None = None, res: torch.Tensor | None = None, res_scale=None,
              stats: torch.Tensor | None = None, stats_per_h: int = 0, n_group: int | None = None,
              out_sg: int = 0, out_offset: int = 0, out_sh: int | None = None, out_sw: int | None = None,
              useful: float = 1.0, post: torch.Tensor | None = None, y_bf16: bool = False) -> None:
        p = ConvParams()
        p.batch, p.h_in, p.w_in, p.c_in = x.B, x.H, x.W, x.C
        p.in_sb, p.in_sh, p.in_sw = x.sb, x.sh, x.sw
        p.h_out, p.w_out, p.n_out = h_out, w_out, n_out
        p.kh, p.kw, p.sh, p.sw, p.dh, p.dw, p.ph, p.pw = kh, kw, sh, sw, dh, dw, ph, pw
        p.out_sb = out.sb
        p.out_sh = out.sh if out_sh is None else out_sh
        p.out_sw = out.sw if out_sw is None else out_sw
        p.out_sg = out_sg
        n_final = n_out // 2 if act == ACT_GLU else n_out
        p.n_group = n_group if n_group is not None else n_final
        p.act, p.prologue = act, prologue
        p.pro_stats, p.pro_gamma, p.pro_beta = _lib.ptr(pro_stats), _lib.ptr(pro_gamma), _lib.ptr(pro_beta)
        p.pro_group_per_h = pro_per_h
        if pro_x2 is not None:
            assert (pro_x2.sb, pro_x2.sh, pro_x2.sw) == (x.sb, x.sh, x.sw)
            p.pro_x2 = pro_x2.t.data_ptr()
        p.res = _lib.ptr(res)
        p.res_scale = _lib.ptr(res_scale)
        p.stats = _lib.ptr(stats)
        p.stats_per_h = stats_per_h
        y = out.t.data_ptr() + 4 * out_offset
        # Algorithmic FLOPs (``useful``: the fraction of the kernel's taps that are not structural zeros).
        flops = 2.0 * x.B * h_out * w_out * n_out * kh * kw * x.C * useful
        if self._tc_eligible(x, p, prologue, out_offset):
            if prologue == PRO_ADD:
                # Fold the decoder skip connection into its input (consumed only here).
                _lib.call("unblend_add", x.t.data_ptr(), pro_x2.t.data_ptr(), x.t.data_ptr(), x.t.numel(),
                          x.t.numel(), 1.0)
                p.prologue, p.pro_x2 = PRO_NONE, None
            if post is not None:
                # post [h_out, n_final]: added per (output row, channel) after the activation.
                p.post, p.post_sh = post.data_ptr(), post.shape[1]
            p.y_bf16 = 1 if y_bf16 else 0
            if self.precision == "fp32":
                # The bf16 split halves the MMAs; layers whose many-tile width is <= 128 columns
                # keep the TF32 split, whose A operand sits in TMEM (A-from-TMEM MMAs issue faster
                # at those widths: decoder.3's 3x3 rewrite 851 us against 923 us with the bf16
                # split in shared memory), unless their three taps along w share one A load and
                # operand split (bf16 split, tiles of <= 128 columns; 3.37 -> 2.33 ms for that
                # layer at 32 segments). The split and the tap grouping depend on the layer only,
                # not on the batch (the tile width does not change any output's rounding; the
                # split and the K order do).
                bn256 = self._bn256_min[_lib.TC_TF32X3]
                subtap = self.fp32_subtaps and kw == 3 and sw == 1 and dw * 2 <= 8 and _subtaps_pay(n_out, bn256)
                wide = _block_n(n_out, bn256) >= 192
                if self.fp32_split == "bf16x3" and subtap:
                    mode = _lib.TC_BF16X3_TAPS
                else:
                    mode = _lib.TC_BF16X3 if self.fp32_split == "bf16x3" and wide else _lib.TC_TF32X3
                block_n = _block_n(n_out, bn256, _m_tiles(x.B, h_out, w_out), self._sms(x),
                                   max_bn=128 if mode == _lib.TC_BF16X3_TAPS else 256)
            else:
                mode = _lib.TC_BF16
                if x.t.dtype == torch.bfloat16:
                    # Activations a producer wrote as bf16 for this layer: loaded as they are.
                    mode, p.x_bf16 = _lib.TC_BF16_ACT, 1
                bn256 = self._bn256_min[_lib.TC_BF16]
                if kw == 3 and sw == 1 and dw * 2 <= 8:
                    # 3-wide kernel rows: tiles of <= 192 columns share one A load across the three taps.
                    bn256 = 1 << 30
                block_n = _block_n(n_out, bn256, _m_tiles(x.B, h_out, w_out), self._sms(x))
            wmode = {_lib.TC_BF16_ACT: _lib.TC_BF16, _lib.TC_BF16X3_TAPS: _lib.TC_BF16X3}.get(mode, mode)
            whi, wlo = self._tc_weight(w, wmode)
            _lib.call("unblend_conv2d_tc", x.t.data_ptr(), whi.data_ptr(), _lib.ptr(wlo), _lib.ptr(b), y,
                      ctypes_byref(p), mode, block_n, work=flops)
            return
        assert not y_bf16 and x.t.dtype == torch.float32, "bf16 activations need the tensor-core path"
        _lib.call("unblend_conv2d_f32", x.t.data_ptr(), w.data_ptr(), _lib.ptr(b), y, ctypes_byref(p), work=flops)
        if post is not None:
            # CUDA-core path: the same add as a separate pass over the dense output.
            assert out_offset == 0 and out.sb == h_out * w_out * n_final and out.sw == n_final
            table = post[:, None, :].expand(h_out, w_out, n_final).contiguous()
            _lib.call("unblend_add", y, table.data_ptr(), y, out.B * table.numel(), table.numel(), 1.0)

    def _sms(self, x: Act) -> int:
        """Streaming multiprocessors of the device holding ``x`` (cached)."""
        dev = x.t.device
        n = self._sm_count.get(dev.index)
        if n is None:
            n = self._sm_count[dev.index] = torch.cuda.get_device_properties(dev).multi_processor_count
        return n

    def _tc_eligible(self, x: Act, p: ConvParams, prologue: int, out_offset: int) -> bool:
        """Whether this convolution meets the tensor-core kernel's layout requirements."""
        if self.precision == "fp32-simt" or prologue not in (PRO_NONE, PRO_ADD):
            return False
        if x.C % 8 or x.C < 16 or x.sw != x.C or x.sh % 4 or x.sb % 4:
            return False
        if x.t.dtype == torch.bfloat16 and (self.precision != "bf16" or p.sw != 1 or x.sh % 8 or x.sb % 8):
            return False
        if p.sw != 1:
            cap = x.sb // x.C
            if not (p.sw == 4 and p.kw == 8 and p.pw == 2 and p.kh == 1 and x.H == 1 and x.sb % (4 * x.C) == 0
                    and cap >= 4 * -(-x.W // 4) and (2 * x.C) % 32 == 0):
                return False
        if p.act == ACT_GLU and p.n_out % 4:
            return False
        return all(v % 4 == 0 for v in (p.n_group, p.out_sb, p.out_sh, p.out_sw, p.out_sg, out_offset))

    def _tc_weight(self, w: torch.Tensor, mode: int) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Tensor-core copy of a packed weight: (hi, lo) TF32 or bf16 split, or (bf16, None), cached."""
        key = (w.data_ptr(), tuple(w.shape), mode)
        hit = self._tc_cache.get(key)
        if hit is None:
            flat = w.reshape(w.shape[0], -1)
            if mode == _lib.TC_TF32X3:
                hit = split_tf32(flat)
            elif mode == _lib.TC_BF16X3:
                hit = split_bf16(flat)
            else:
                hit = (flat.to(torch.bfloat16).contiguous(), None)
            self._tc_cache[key] = hit
        return hit

    def _stats(self, stats: torch.Tensor, groups: int, count: float) -> torch.Tensor:
        out = torch.empty(2 * groups, device=stats.device, dtype=torch.float32)
        _lib.call("unblend_stats_finalize", stats.data_ptr(), out.data_ptr(), groups, float(count), 1e-5, 0, 0)
        return out



def ctypes_byref(p: ConvParams):
    return ctypes.byref(p)
