"""Overlapping-segment engine on the GPU (mirror of ``unblend.apply.apply_model``).

Same arguments and semantics as the reference (unblend/apply.py:500-1333) for
plain models: the track is split into segments of
``round(model.samplerate * model.max_allowed_segment)`` samples at stride
``int((1 - overlap) * segment)``; each chunk is centred and zero-padded to the
segment length, batched ``chunk_batch_size`` at a time through
``model(batch)``, centre-trimmed, weighted by the triangular cross-fade and
overlap-added with a running weight sum; the result is ``out / sum_weight``.
``shifts > 0`` averages rounds over ``random.randint(0, samplerate // 2)``
offsets drawn round-major, as the reference does.

Chunk gather, weighted overlap-add and the final divide are CUDA kernels of
``libunblend_b200.so``; the track and accumulators stay resident on the device
and nothing synchronises per batch unless a progress callback is attached.
"""

from __future__ import annotations

import random
from typing import Any, Callable

import torch

from . import _lib


class ValidationError(ValueError):
    """Invalid argument (same role as the reference's ``ValidationError``, a ``ValueError``)."""


def _segment_plan(model: Any, overlap: float) -> tuple[int, int]:
    segment = int(round(model.samplerate * model.max_allowed_segment))
    stride = int((1 - overlap) * segment)
    if stride < 1:
        raise ValidationError(f"split overlap {overlap} produces an invalid stride for segment length {segment}")
    return segment, stride


def _accumulate(model: Callable, mix: torch.Tensor, n_sources: int, segment: int, offsets: list[int],
                off_dev: torch.Tensor, chunk_batch_size: int, acc: torch.Tensor, sum_w: torch.Tensor,
                progress: Callable[[int], None] | None = None) -> None:
    """Separate the chunks starting at ``offsets`` and overlap-add them into ``acc``/``sum_w``.

    ``acc`` is ``[S*C, L]`` and ``sum_w`` ``[L]`` over the whole track (only the
    positions the chunks touch are written); ``off_dev`` holds ``offsets`` as
    int64 on the device (unblend/apply.py:1155-1238).
    """
    C, L = mix.shape
    dev = mix.device
    fixed = bool(getattr(model, "_fixed_batch_shape", False))
    total = len(offsets)
    for i in range(0, total, chunk_batch_size):
        n = min(chunk_batch_size, total - i)
        rows = chunk_batch_size if fixed else n
        batch = torch.zeros(rows, C, segment, device=dev, dtype=torch.float32) if rows > n else \
            torch.empty(rows, C, segment, device=dev, dtype=torch.float32)
        offp = off_dev.data_ptr() + 8 * i
        _lib.call("unblend_gather_chunks", mix.data_ptr(), C, L, offp, n, segment, batch.data_ptr())
        with torch.inference_mode():
            y = model(batch)
        y = y.float().contiguous()
        if y.shape[0] != rows or y.shape[-1] != segment:
            raise RuntimeError(f"model returned {tuple(y.shape)} for a batch of {rows} x {segment}")
        lo = offsets[i]
        hi = min(L, offsets[i + n - 1] + segment)
        _lib.call("unblend_overlap_add", y.data_ptr(), n, n_sources * C, segment, offp, L, lo, hi,
                  acc.data_ptr(), sum_w.data_ptr())
        if progress is not None:
            progress(n)


def _apply_unshifted(model: Callable, mix: torch.Tensor, n_sources: int, segment: int, stride: int,
                     chunk_batch_size: int, progress_callback: Callable | None) -> torch.Tensor:
    """One ``[C, L]`` device track -> ``[S, C, L]`` (unblend/apply.py:1009-1333)."""
    C, L = mix.shape
    dev = mix.device
    offsets = list(range(0, L, stride))
    off_dev = torch.tensor(offsets, device=dev, dtype=torch.int64)
    acc = torch.zeros(n_sources * C, L, device=dev, dtype=torch.float32)
    sum_w = torch.zeros(L, device=dev, dtype=torch.float32)
    total = len(offsets)
    progress = None
    if progress_callback:
        progress_callback("processing_start", {"total_chunks": total, "total_inputs": 1,
                                               "input_total_chunks": [total]})
        done = [0]

        def progress(n: int) -> None:
            torch.cuda.synchronize(dev)
            for _ in range(n):
                done[0] += 1
                progress_callback("chunk_complete", {"completed_chunks": done[0], "total_chunks": total,
                                                     "input_index": 0, "input_completed_chunks": done[0],
                                                     "input_total_chunks": total})
    _accumulate(model, mix, n_sources, segment, offsets, off_dev, chunk_batch_size, acc, sum_w, progress)
    out = torch.empty_like(acc)
    _lib.call("unblend_divide", acc.data_ptr(), sum_w.data_ptr(), out.data_ptr(), n_sources * C, L)
    if progress_callback:
        progress_callback("processing_complete", {"total_chunks": total, "total_inputs": 1,
                                                  "input_total_chunks": [total]})
    return out.view(n_sources, C, L)


def apply_model(model: Any, mix: torch.Tensor, device: torch.device | str | None = None, shifts: int = 0,
                overlap: float = 0.25, transition_power: float = 1.0,
                progress_callback: Callable[[str, dict[str, Any]], None] | None = None,
                chunk_batch_size: int = 1, shift_offsets: list[int] | None = None) -> torch.Tensor:
    """Separate ``mix`` ([C, L] or [B, C, L]) with ``model`` over overlapping segments.

    :param model: Object with ``sources``, ``samplerate``, ``max_allowed_segment`` and a
        CUDA ``__call__(batch[B, C, T]) -> [B, S, C, T]`` (e.g. :class:`HTDemucsCuda`).
    :param mix: Mixture on any device; it is staged to ``device`` once.
    :param device: CUDA device (defaults to the mix's device, or the current CUDA device).
    :param shifts: Number of random-shift rounds to average (0 = none).
    :param overlap: Segment overlap in [0, 1).
    :param transition_power: Cross-fade exponent; only 1.0 is implemented.
    :param progress_callback: Optional ``(event, payload)`` callback; attaching one
        synchronises the device after each batch (as the reference's CUDA path does).
    :param chunk_batch_size: Segments per forward.
    :param shift_offsets: Explicit per-round offsets (one track) instead of ``random`` draws.
    :return: ``[B, S, C, L]`` (or ``[S, C, L]`` for a 2-D mix) on the mix's original device.
    """
    if not 0.0 <= overlap < 1.0:
        raise ValidationError(f"overlap must be in [0, 1), got {overlap}")
    if transition_power != 1.0:
        raise ValidationError("only transition_power=1.0 is implemented")
    if chunk_batch_size < 1:
        raise ValidationError("chunk_batch_size must be >= 1")
    orig_device = mix.device
    if device is None:
        device = mix.device if mix.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise ValidationError("the B200 segment engine runs on CUDA devices only")
    squeeze = mix.dim() == 2
    mixes = mix[None] if squeeze else mix
    segment, stride = _segment_plan(model, overlap)
    S = len(model.sources)
    max_shift = int(0.5 * model.samplerate)
    results = []
    with torch.cuda.device(device):
        for row in range(mixes.shape[0]):
            track = mixes[row].to(device, dtype=torch.float32, non_blocking=True).contiguous()
            C, L = track.shape
            if not shifts:
                results.append(_apply_unshifted(model, track, S, segment, stride, chunk_batch_size,
                                                progress_callback))
                continue
            offs = list(shift_offsets) if shift_offsets is not None else \
                [random.randint(0, max_shift) for _ in range(shifts)]
            acc = None
            padded = torch.nn.functional.pad(track, (max_shift, max_shift))
            for off in offs:
                shifted = padded[:, off : L + max_shift].contiguous()
                part = _apply_unshifted(model, shifted, S, segment, stride, chunk_batch_size, progress_callback)
                part = part[..., max_shift - off :][..., :L]
                acc = part.clone() if acc is None else acc.add_(part)
            results.append(acc / len(offs))
    out = torch.stack(results)
    if squeeze:
        out = out[0]
    if orig_device.type == "cpu":
        # Page-locked staging (torch's caching host allocator): the device->host
        # copy runs at full PCIe/C2C bandwidth instead of through pageable memory.
        host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        host.copy_(out, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        return host
    return out.to(orig_device)
