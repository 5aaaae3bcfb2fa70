"""Host-side launch choices of the tensor-core convolution (no GPU needed)."""

from __future__ import annotations

import pytest

from unblend_b200.convnet import _block_n, _m_tiles, _subtaps_pay


@pytest.mark.parametrize("n_out,bn", [(48, 64), (64, 64), (96, 96), (128, 128), (192, 192), (384, 192),
                                      (768, 256), (1536, 256), (2048, 256), (200, 128)])
def test_many_tile_width_minimises_padded_columns(n_out, bn):
    assert _block_n(n_out, 512) == bn


def test_few_tiles_trade_width_for_fuller_waves():
    # 4 segments of the transformer's 2688 tokens x 512 -> 1536: 84 row tiles; the choice is the
    # cheapest of (waves x (64 + width)) over the candidate widths.
    m = _m_tiles(4, 1, 2688)
    assert m == 21 * 4
    bn = _block_n(1536, 512, m, 148)
    cost = lambda c: -(-(m * -(-1536 // c)) // 148) * (64 + c)  # noqa: E731
    assert cost(bn) == min(cost(c) for c in (64, 96, 128, 192, 256))
    # One row tile: two 64-column tiles still fit one wave and cost less than one 96-column tile.
    assert _block_n(96, 512, 1, 148) == 64


def test_max_bn_caps_the_candidates():
    for n in (96, 192, 384, 768, 1536):
        assert _block_n(n, 512, max_bn=128) <= 128
    assert _block_n(1536, 512, max_bn=128) == 128


@pytest.mark.parametrize("n_out,shared", [(64, True), (96, True), (128, True), (192, False), (256, True),
                                          (384, True), (768, False), (1536, False)])
def test_shared_tap_loads_only_where_the_tile_count_stays_within_1_5x(n_out, shared):
    assert _subtaps_pay(n_out, 512) is shared
