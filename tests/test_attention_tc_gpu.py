"""The tcgen05 flash-attention kernel against a PyTorch fp32 reference."""

from __future__ import annotations

import math

import pytest
import torch

from conftest import rel_err
from unblend_b200 import _lib

pytestmark = pytest.mark.gpu

# mode 0: 3-pass TF32 (fp32 accuracy); mode 1: single-pass TF32; mode 2: 3-pass
# bf16 (16 significant bits per operand). On these unit-variance inputs a score's
# error is ~2^-16 of |q| |k| and enters the exponent as is, so mode 2 reaches
# 1.6e-4 of the RMS on the 2688-key rows (mode 0: 1e-5); in the HTDemucs forward
# the attention output passes a 1e-4 LayerScale, and the model-level tests hold
# the 1e-4 x RMS parity bound against the reference with this mode.
TOL = {0: 2e-5, 1: 1e-2, 2: 3e-4}


def _ref(q, k, v, heads, hd):
    B, lq, _ = q.shape
    lk = k.shape[1]
    qh = q.view(B, lq, heads, hd).transpose(1, 2).double()
    kh = k.view(B, lk, heads, hd).transpose(1, 2).double()
    vh = v.view(B, lk, heads, hd).transpose(1, 2).double()
    att = torch.softmax(qh @ kh.transpose(-1, -2) / math.sqrt(hd), -1) @ vh
    return att.transpose(1, 2).reshape(B, lq, heads * hd).float()


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("lq,lk,heads,hd", [(100, 70, 3, 64), (130, 64, 2, 48), (9, 200, 4, 8), (300, 257, 2, 64),
                                            (1344, 2688, 1, 64)])
def test_attention_tc_matches_reference(mode, lq, lk, heads, hd):
    B, D = 2, heads * hd
    g = torch.Generator(device="cuda").manual_seed(lq * 7 + lk)
    q = torch.randn(B, lq, D, device="cuda", generator=g)
    k = torch.randn(B, lk, D, device="cuda", generator=g)
    v = torch.randn(B, lk, D, device="cuda", generator=g)
    o = torch.empty(B, lq, D, device="cuda")
    _lib.call("unblend_attention_tc", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, heads, lq, lk, hd,
              lq * D, D, lk * D, D, lq * D, D, 1.0 / math.sqrt(hd), mode)
    torch.cuda.synchronize()
    assert _lib.error_flag() == 0
    ref = _ref(q, k, v, heads, hd)
    err = rel_err(o, ref)
    if mode in (0, 2):
        # fp32 modes: as accurate as the fp32 SIMT kernel (long rows average
        # thousands of values, so fp32 accumulation alone reaches ~1e-4 of RMS).
        o32 = torch.empty_like(o)
        _lib.call("unblend_attention_f32", q.data_ptr(), k.data_ptr(), v.data_ptr(), o32.data_ptr(), B, heads, lq,
                  lk, hd, lq * D, D, lk * D, D, lq * D, D, 1.0 / math.sqrt(hd))
        assert err < max(TOL[mode], 4 * rel_err(o32, ref))
    else:
        assert err < TOL[mode]


def test_attention_tc_interleaved_qkv_rows():
    """Self-attention reads Q, K and V out of one [L, 3D] projection."""
    B, L, heads, hd = 2, 200, 8, 64
    D = heads * hd
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, L, 3 * D, device="cuda", generator=g)
    o = torch.empty(B, L, D, device="cuda")
    base = qkv.data_ptr()
    _lib.call("unblend_attention_tc", base, base + 4 * D, base + 8 * D, o.data_ptr(), B, heads, L, L, hd,
              L * 3 * D, 3 * D, L * 3 * D, 3 * D, L * D, D, 1.0 / math.sqrt(hd), 0)
    q, k, v = (qkv[..., i * D:(i + 1) * D].contiguous() for i in range(3))
    ref = _ref(q, k, v, heads, hd)
    # The fp32 SIMT kernel on the same rows sets the accuracy floor (as in the test above).
    o32 = torch.empty_like(o)
    _lib.call("unblend_attention_f32", q.data_ptr(), k.data_ptr(), v.data_ptr(), o32.data_ptr(), B, heads, L, L, hd,
              L * D, D, L * D, D, L * D, D, 1.0 / math.sqrt(hd))
    floor = 4 * rel_err(o32, ref)
    assert rel_err(o, ref) < max(TOL[0], floor)
    o2 = torch.empty_like(o)
    _lib.call("unblend_attention_tc", base, base + 4 * D, base + 8 * D, o2.data_ptr(), B, heads, L, L, hd,
              L * 3 * D, 3 * D, L * 3 * D, 3 * D, L * D, D, 1.0 / math.sqrt(hd), 2)
    assert rel_err(o2, ref) < max(TOL[2], floor)
    assert _lib.error_flag() == 0
