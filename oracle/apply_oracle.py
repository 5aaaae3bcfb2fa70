"""Restatement of the overlapping-segment loop (CPU oracle, test use only).

Restates ``apply_model_multi`` / ``_apply_model_multi_unshifted``
(unblend/apply.py:567-1333) for plain models: centred zero-padded chunks
(``TensorChunk.padded``, unblend/apply.py:278-311), the triangular cross-fade
(``_split_weight``, unblend/apply.py:406-432), weighted overlap-add with a
weight sum and the final divide (unblend/apply.py:1219-1238, 1329), and shift
averaging over ``random.randint`` offsets (unblend/apply.py:877-995).
Chunk-to-batch grouping does not change any chunk's result, so chunks are
run in input order in groups of ``chunk_batch_size``.
"""

from __future__ import annotations

import random
from typing import Callable

import torch
import torch.nn.functional as F


def split_weight(segment_length: int, transition_power: float = 1.0) -> torch.Tensor:
    """Triangular cross-fade weight (unblend/apply.py:406-432)."""
    half = segment_length // 2
    rising = torch.arange(1, half + 1, dtype=torch.float32)
    falling = torch.arange(segment_length - half, 0, -1, dtype=torch.float32)
    w = torch.cat([rising, falling])
    return (w / w.max()) ** transition_power


def padded_chunk(mix: torch.Tensor, offset: int, length: int, target: int) -> torch.Tensor:
    """``TensorChunk(mix, offset, length).padded(target)`` (unblend/apply.py:233-311)."""
    total = mix.shape[-1]
    length = min(total - offset, length)
    delta = target - length
    start = offset - delta // 2
    end = start + target
    cs, ce = max(0, start), min(total, end)
    return F.pad(mix[..., cs:ce], (cs - start, end - ce))


def center_trim(t: torch.Tensor, ref: int) -> torch.Tensor:
    """``center_trim`` (unblend/blocks.py:17-36)."""
    delta = t.shape[-1] - ref
    if delta:
        t = t[..., delta // 2 : -(delta - delta // 2)]
    return t


def apply_unshifted(model: Callable[[torch.Tensor], torch.Tensor], mix: torch.Tensor, n_sources: int,
                    segment_length: int, overlap: float = 0.25, chunk_batch_size: int = 1,
                    transition_power: float = 1.0) -> torch.Tensor:
    """One mix ``[1, C, L]`` through ``_apply_model_multi_unshifted`` (unblend/apply.py:1009-1333)."""
    stride = int((1 - overlap) * segment_length)
    L = mix.shape[-1]
    weight = split_weight(segment_length, transition_power)
    out = torch.zeros(mix.shape[0], n_sources, mix.shape[-2], L)
    sum_w = torch.zeros(L)
    offsets = list(range(0, L, stride))
    for i in range(0, len(offsets), chunk_batch_size):
        group = offsets[i : i + chunk_batch_size]
        batch = torch.cat([padded_chunk(mix, o, segment_length, segment_length) for o in group])
        y = model(batch)
        for j, o in enumerate(group):
            n = min(L - o, segment_length)
            chunk_out = center_trim(y[j : j + 1], n)
            w = weight[:n]
            out[..., o : o + n] += chunk_out * w
            sum_w[o : o + n] += w
    return out / sum_w


def shift_offsets(n_mixes: int, shifts: int, samplerate: int, seed: int | None = None) -> list[list[int]]:
    """Round-major ``random.randint(0, max_shift)`` draws (unblend/apply.py:877-888)."""
    if seed is not None:
        random.seed(seed)
    max_shift = int(0.5 * samplerate)
    return [[random.randint(0, max_shift) for _ in range(n_mixes)] for _ in range(shifts)]


def apply_model(model: Callable[[torch.Tensor], torch.Tensor], mix: torch.Tensor, n_sources: int,
                segment_length: int, samplerate: int, shifts: int = 0, overlap: float = 0.25,
                chunk_batch_size: int = 1, offsets: list[int] | None = None) -> torch.Tensor:
    """``apply_model`` (unblend/apply.py:500-564, 877-995) for one ``[1, C, L]`` mix.

    :param offsets: Per-round shift offsets; drawn with ``random`` when ``None``.
    """
    if not shifts:
        return apply_unshifted(model, mix, n_sources, segment_length, overlap, chunk_batch_size)
    max_shift = int(0.5 * samplerate)
    if offsets is None:
        offsets = [r[0] for r in shift_offsets(1, shifts, samplerate)]
    L = mix.shape[-1]
    acc = None
    for off in offsets:
        padded = padded_chunk(mix, 0, L, L + 2 * max_shift)
        shifted = padded[..., off : off + L + max_shift - off]
        part = apply_unshifted(model, shifted, n_sources, segment_length, overlap, chunk_batch_size)
        part = part[..., max_shift - off :][..., :L]
        acc = part.clone() if acc is None else acc + part
    return acc / shifts
