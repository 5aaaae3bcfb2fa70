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

import math
import random
from numbers import Real
from typing import Any, Callable

import torch

from . import _lib


class ValidationError(ValueError):
    """Invalid argument (same role as the reference's ``ValidationError``, a ``ValueError``)."""


def _finite_number(v: Any) -> bool:
    return not isinstance(v, bool) and isinstance(v, Real) and math.isfinite(float(v))


class ModelEnsemble:
    """Weighted ensemble of separation models (mirror of unblend/apply.py:63-219).

    ``apply_model`` runs every member over the same segments and shift offsets,
    scales each member's stem ``k`` by ``weights[m][k]`` and divides the sum by
    the per-stem weight totals (``htdemucs_ft``: four specialists with one-hot
    rows). Members must agree on sources, sample rate, channel count and the
    external-normalisation contract; ``segment`` caps every member's segment.

    :param models: Member models (e.g. :class:`~unblend_b200.htdemucs.HTDemucsCuda`).
    :param weights: ``len(models)`` rows of one weight per source (all ones when None).
    :param segment: Optional segment length override in seconds.
    """

    def __init__(self, models: list, weights: list[list[float]] | None = None,
                 segment: float | None = None) -> None:
        if not models:
            raise ValidationError("ModelEnsemble requires at least one model.")
        if segment is not None and not (_finite_number(segment) and segment > 0):
            raise ValidationError(f"segment must be a finite positive number, got {segment}")
        first = models[0]
        norm = getattr(first, "external_normalization", True)
        for i, other in enumerate(models):
            for attr in ("sources", "samplerate", "audio_channels"):
                if getattr(other, attr) != getattr(first, attr):
                    raise ValidationError(f"Ensemble model {i} has {attr} {getattr(other, attr)}, "
                                          f"expected {getattr(first, attr)}.")
            if getattr(other, "external_normalization", True) != norm:
                raise ValidationError("Ensemble members must share the same external_normalization contract.")
            maximum = float(other.max_allowed_segment)
            if not math.isfinite(maximum) or maximum <= 0:
                raise ValidationError(f"Ensemble model {i} has invalid max_allowed_segment {other.max_allowed_segment}.")
            if segment is not None:
                other.max_allowed_segment = min(float(segment), maximum)
        self.models = list(models)
        self.sources = first.sources
        self.samplerate = first.samplerate
        self.audio_channels = first.audio_channels
        self.external_normalization = norm
        if weights is None:
            weights = [[1.0] * len(first.sources) for _ in models]
        self.weights = [list(row) for row in weights]
        self.validated_weight_totals()
        self.weights = [[float(v) for v in row] for row in self.weights]

    @property
    def max_allowed_segment(self) -> float:
        return min(float(m.max_allowed_segment) for m in self.models)

    def validated_weight_totals(self) -> list[float]:
        """Check the weight matrix and return the per-source totals (finite, non-zero)."""
        if len(self.weights) != len(self.models):
            raise ValidationError(f"weights must have one row per model ({len(self.models)}), "
                                  f"got {len(self.weights)}.")
        for i, row in enumerate(self.weights):
            if len(row) != len(self.sources):
                raise ValidationError(f"weights row {i} must contain {len(self.sources)} source weights, "
                                      f"got {len(row)}.")
            for k, v in enumerate(row):
                if not _finite_number(v):
                    raise ValidationError(f"weights[{i}][{k}] must be a finite number.")
        totals = [sum(float(row[k]) for row in self.weights) for k in range(len(self.sources))]
        for name, total in zip(self.sources, totals):
            if not math.isfinite(total) or total == 0:
                raise ValidationError(f"Ensemble weights for source '{name}' must have a finite, non-zero total.")
        return totals

    def specialist_for(self, stem: str | None) -> int | None:
        """Index of the member whose row is one-hot on ``stem`` while every other row is 0 there
        (unblend/apply.py:730-760), else None."""
        if stem is None or stem not in self.sources:
            return None
        k = self.sources.index(stem)
        for i, row in enumerate(self.weights):
            if (abs(row[k] - 1.0) < 1e-6 and all(abs(w) < 1e-6 for j, w in enumerate(row) if j != k)
                    and all(o == i or abs(other[k]) < 1e-6 for o, other in enumerate(self.weights))):
                return i
        return None

    def __call__(self, *args, **kwargs):
        raise NotImplementedError("Call `apply_model` on this.")


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
                chunk_batch_size: int = 1, shift_offsets: list[int] | None = None,
                use_only_stem: str | None = None) -> torch.Tensor:
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
    :param use_only_stem: For a :class:`ModelEnsemble` of specialists, run only the member whose
        weight row is one-hot on this stem (its output still holds every source); no effect otherwise.
    :return: ``[B, S, C, L]`` (or ``[S, C, L]`` for a 2-D mix) on the mix's original device.
    """
    members = getattr(model, "models", None)
    if members is not None and hasattr(model, "weights"):
        return _apply_ensemble(model, mix, device, shifts, overlap, transition_power, progress_callback,
                               chunk_batch_size, shift_offsets, use_only_stem)
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
    rows_offs = _shift_plan(shifts, mixes.shape[0], max_shift, shift_offsets)
    results = []
    with torch.cuda.device(device):
        for row in range(mixes.shape[0]):
            track = mixes[row].to(device, dtype=torch.float32, non_blocking=True).contiguous()
            C, L = track.shape
            if not shifts:
                results.append(_apply_unshifted(model, track, S, segment, stride, chunk_batch_size,
                                                progress_callback))
                continue
            offs = rows_offs[row]
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
        return _to_host(out)
    return out.to(orig_device)


def _to_host(out: torch.Tensor) -> torch.Tensor:
    """Copy a device result into page-locked host memory (torch's caching host
    allocator), so the device->host copy runs at full link bandwidth instead of
    through pageable memory."""
    host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream(out.device).synchronize()
    return host


def _shift_plan(shifts: int, rows: int, max_shift: int, shift_offsets: list[int] | None) -> list[list[int]]:
    """Per-row shift offsets, drawn round-major then row-minor as the reference does
    (unblend/apply.py:722-727); ``shift_offsets`` (one list for every row) replaces the draws."""
    if not shifts:
        return [[] for _ in range(rows)]
    if shift_offsets is not None:
        return [list(shift_offsets) for _ in range(rows)]
    draws = [[random.randint(0, max_shift) for _ in range(rows)] for _ in range(shifts)]
    return [[draws[r][row] for r in range(shifts)] for row in range(rows)]


def _apply_ensemble(ens: Any, mix: torch.Tensor, device, shifts: int, overlap: float, transition_power: float,
                    progress_callback, chunk_batch_size: int, shift_offsets, use_only_stem) -> torch.Tensor:
    """Weighted sum of the members' separations over shared shift offsets (unblend/apply.py:722-867)."""
    totals = ens.validated_weight_totals()
    if shifts and mix.dim() == 3 and mix.shape[0] > 1:
        # One draw for the whole ensemble (round-major, mix-minor), then row by row
        # so every member sees the same shifted rounds of each mix.
        plan = _shift_plan(shifts, mix.shape[0], int(0.5 * ens.samplerate), shift_offsets)
        return torch.stack([_apply_ensemble(ens, mix[r], device, shifts, overlap, transition_power,
                                            progress_callback, chunk_batch_size, plan[r], use_only_stem)
                            for r in range(mix.shape[0])])
    if shifts and shift_offsets is None:
        shift_offsets = _shift_plan(shifts, 1, int(0.5 * ens.samplerate), None)[0]
    pick = ens.specialist_for(use_only_stem) if hasattr(ens, "specialist_for") else None
    kw = dict(device=device, shifts=shifts, overlap=overlap, transition_power=transition_power,
              progress_callback=progress_callback, chunk_batch_size=chunk_batch_size, shift_offsets=shift_offsets)
    if pick is not None:
        return apply_model(ens.models[pick], mix, **kw)
    acc = None
    for member, row in zip(ens.models, ens.weights):
        out = apply_model(member, mix, **kw)
        w = torch.tensor([float(v) for v in row], dtype=out.dtype, device=out.device)
        part = out * w.view(-1, 1, 1) if out.dim() == 3 else out * w.view(1, -1, 1, 1)
        acc = part if acc is None else acc.add_(part)
    t = torch.tensor(totals, dtype=acc.dtype, device=acc.device)
    return acc / (t.view(-1, 1, 1) if acc.dim() == 3 else t.view(1, -1, 1, 1))
