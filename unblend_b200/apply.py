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
import time
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


def _looks_like_cuda_oom(exc: BaseException) -> bool:
    """Whether ``exc`` reports exhausted device memory (the test of unblend/apply.py:32-53).

    Covers torch's ``OutOfMemoryError`` and the ``RuntimeError`` this library's
    launchers raise for ``cudaErrorMemoryAllocation`` ("CUDA out of memory in ...").
    """
    if isinstance(exc, torch.cuda.OutOfMemoryError):
        return True
    text = str(exc).lower()
    return any(m in text for m in ("out of memory", "cudaerrormemoryallocation", "cublas_status_alloc_failed"))


# Accumulators stay on the device when every mix's track, accumulator and weight
# sum fit this fraction of the free device memory, after a reserve for the
# forward's working set (unblend/apply.py:330-400); otherwise they live on the host
# and each batch's weighted output is copied back, bounding device memory by
# the model and one batch for arbitrarily long audio.
_GPU_ACCUM_VRAM_FRACTION = 0.3
_GPU_ACCUM_VRAM_RESERVE_BYTES = 2 * 1024**3


# Free device memory as last queried per device: (time, free bytes, this process's
# reserved bytes then). cudaMemGetInfo costs milliseconds per call on this driver,
# so a query younger than _FREE_QUERY_MAX_AGE_S is reused, corrected by what this
# process's allocator reserved or released since (other processes' changes within
# that window are not seen).
_FREE_QUERY: dict[int, tuple[float, int, int]] = {}
_FREE_QUERY_MAX_AGE_S = 1.0


def _free_device_bytes(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    now = time.monotonic()
    reserved = torch.cuda.memory_reserved(idx)
    hit = _FREE_QUERY.get(idx)
    if hit is not None and now - hit[0] < _FREE_QUERY_MAX_AGE_S:
        return max(0, hit[1] - (reserved - hit[2]))
    free, _ = torch.cuda.mem_get_info(idx)
    _FREE_QUERY[idx] = (now, free, reserved)
    return free


def _gpu_accum_budget_bytes(device: torch.device, forward_reserve_bytes: int | None = None) -> int:
    """Device bytes available for resident tracks and accumulators (0 if unknown)."""
    try:
        free = _free_device_bytes(device)
    except Exception:
        return 0
    slack = torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    reserve = max(_GPU_ACCUM_VRAM_RESERVE_BYTES, forward_reserve_bytes or 0)
    return max(0, int(_GPU_ACCUM_VRAM_FRACTION * (free + max(0, slack) - reserve)))


def _gpu_accum_bytes_needed(batch_dim: int, n_sources: int, channels: int, length: int) -> int:
    """fp32 bytes of one mix's resident state: the track, the ``[S, C, L]`` accumulator and the weight sum."""
    return (batch_dim * channels * (n_sources + 1) * length + length) * 4


def _split_weight_host(segment: int, power: float) -> torch.Tensor:
    """The triangular cross-fade weight on the host (unblend/apply.py:406-432), for host accumulation."""
    half = segment // 2
    w = torch.cat([torch.arange(1, half + 1, dtype=torch.float32),
                   torch.arange(segment - half, 0, -1, dtype=torch.float32)])
    return (w / w.max()) ** power


def _segment_plan(model: Any, overlap: float) -> tuple[int, int]:
    segment = int(round(model.samplerate * model.max_allowed_segment))
    stride = int((1 - overlap) * segment)
    if stride < 1:
        raise ValidationError(f"split overlap {overlap} produces an invalid stride for segment length {segment}")
    return segment, stride


def _pools(counts: list[int], chunk_batch_size: int) -> tuple[list[tuple[int, int]], list[tuple[int, int]]]:
    """Split every mix's chunks into the full-batch pool and the cross-mix tail pool.

    Items are ``(mix index, chunk index)``. Each mix contributes its first
    ``chunk_batch_size * (n // chunk_batch_size)`` chunks to the full pool and the
    rest to the tail pool, so the tails of all mixes share batches
    (unblend/apply.py:1102-1155). Within each pool a mix's chunks are contiguous
    and ascending.
    """
    full, tail = [], []
    for m, n in enumerate(counts):
        n_full = (n // chunk_batch_size) * chunk_batch_size
        full += [(m, k) for k in range(n_full)]
        tail += [(m, k) for k in range(n_full, n)]
    return full, tail


def _runs(items: list[tuple[int, int]]) -> list[tuple[int, int, int, int]]:
    """Group a batch's items into ``(mix, first chunk, count, first batch row)`` runs of consecutive chunks."""
    runs: list[list[int]] = []
    for row, (m, k) in enumerate(items):
        if runs and runs[-1][0] == m and runs[-1][1] + runs[-1][2] == k:
            runs[-1][2] += 1
        else:
            runs.append([m, k, 1, row])
    return [tuple(r) for r in runs]  # type: ignore[misc]


def _drain(pool: list, run_batch: Callable[[list], list], batch_size: Callable[[], int],
           backoff: dict | None, fixed_shape: bool, after_oom: Callable[[], None],
           emit: Callable[[list], None]) -> None:
    """Run ``pool`` in slices of ``batch_size()`` items, halving on device OOM (unblend/apply.py:1264-1306).

    Backoff applies only when the caller passed a ``backoff`` dict, the model
    accepts any batch shape and the failure looks like an OOM; the halved size
    sticks in ``backoff["chunk_batch_size"]``; at size 1 the error propagates.
    ``run_batch`` returns progress payloads, emitted only once its batch has
    committed, so a raising callback is not mistaken for a batch failure.
    """
    idx = 0
    while idx < len(pool):
        batch = pool[idx: idx + batch_size()]
        try:
            pending = run_batch(batch)
        except RuntimeError as exc:
            current = batch_size()
            if backoff is None or fixed_shape or current <= 1 or not _looks_like_cuda_oom(exc):
                raise
            backoff["chunk_batch_size"] = max(1, current // 2)
            after_oom()
            continue
        idx += len(batch)
        emit(pending)


class _MixState:
    """One mix's chunk plan and accumulators inside a pooled run."""

    def __init__(self, track: torch.Tensor, offsets: list[int], off_dev: torch.Tensor, acc: torch.Tensor,
                 sum_w: torch.Tensor) -> None:
        self.track = track  # [C, L]: on the device in resident mode, else on the host
        self.C, self.L = track.shape
        self.offsets = offsets
        self.off_dev = off_dev  # the offsets as int64 on the device
        self.acc = acc  # [S*C, L]
        self.sum_w = sum_w  # [L]

    @classmethod
    def plan(cls, track: torch.Tensor, stride: int, n_sources: int, resident: bool,
             device: torch.device) -> "_MixState":
        """Chunks at ``range(0, L, stride)`` and zeroed accumulators (device or host)."""
        C, L = track.shape
        offsets = list(range(0, L, stride))
        off_dev = torch.tensor(offsets, device=device, dtype=torch.int64)
        if resident:
            acc = torch.empty(n_sources * C, L, device=device, dtype=torch.float32)
            sum_w = torch.empty(L, device=device, dtype=torch.float32)
            _lib.call("unblend_zero_f32", acc.data_ptr(), acc.numel(), 1, 0)
            _lib.call("unblend_zero_f32", sum_w.data_ptr(), sum_w.numel(), 1, 0)
        else:
            acc = torch.zeros(n_sources * C, L, dtype=torch.float32)
            sum_w = torch.zeros(L, dtype=torch.float32)
        return cls(track, offsets, off_dev, acc, sum_w)


class _PooledRun:
    """``_apply_model_multi_unshifted`` (unblend/apply.py:1009-1333) on the B200 kernels.

    Full batches run first, then the pooled tails of all mixes. Resident mode
    gathers chunks on the device (``unblend_gather_chunks``) and overlap-adds
    there (``unblend_overlap_add``); host mode gathers on the host, runs the
    batch on the device, weights the trimmed outputs there
    (``unblend_weight_chunks``) and adds them into host accumulators. A batch
    commits only after everything that can fail has run, so a retried batch is
    never counted twice.
    """

    def __init__(self, model: Callable, mixes: list[_MixState], device: torch.device, segment: int,
                 n_sources: int, chunk_batch_size: int, transition_power: float, backoff: dict | None,
                 progress_callback: Callable | None, resident: bool) -> None:
        self.model, self.device, self.segment, self.S = model, device, segment, n_sources
        self.cbs, self.power = chunk_batch_size, float(transition_power)
        self.backoff, self.progress, self.resident = backoff, progress_callback, resident
        self.fixed = bool(getattr(model, "_fixed_batch_shape", False))
        self.mixes = mixes
        self.C = mixes[0].C if mixes else 0
        self.weight = None if resident else _split_weight_host(segment, self.power)
        self.totals = [len(m.offsets) for m in mixes]
        self.done = 0
        self.done_per = [0] * len(mixes)

    def _batch_size(self) -> int:
        if self.backoff is not None:
            return max(1, int(self.backoff["chunk_batch_size"]))
        return self.cbs

    def _forward(self, batch: torch.Tensor, n: int) -> torch.Tensor:
        with torch.inference_mode():
            y = self.model(batch)
        y = y.float().contiguous()
        if y.shape[0] != batch.shape[0] or y.shape[-1] != self.segment or y.shape[1] != self.S:
            raise RuntimeError(f"model returned {tuple(y.shape)} for a batch of {tuple(batch.shape)}")
        return y

    def _rows(self, n: int) -> int:
        # Captured CUDA graphs replay one batch shape: tails are zero-padded up to it
        # (unblend/apply.py:1189-1196). Models whose graphs leave smaller batches to eager
        # launches (``_eager_tails``) are padded only when the tail is within an eighth of
        # the full batch; a smaller tail runs at its own size instead of computing padding.
        if not self.fixed or n >= self.cbs:
            return n
        if getattr(self.model, "_eager_tails", False) and 8 * n < 7 * self.cbs:
            return n
        return self.cbs

    def run_batch(self, items: list[tuple[int, int]]) -> list[dict]:
        n, C, seg, S = len(items), self.C, self.segment, self.S
        rows = self._rows(n)
        runs = _runs(items)
        if self.resident:
            batch = torch.empty(rows, C, seg, device=self.device, dtype=torch.float32)
            if rows > n:
                _lib.call("unblend_zero_f32", batch.data_ptr() + 4 * n * C * seg, (rows - n) * C * seg, 1, 0)
            for m, k0, cnt, b0 in runs:
                st = self.mixes[m]
                _lib.call("unblend_gather_chunks", st.track.data_ptr(), C, st.L, st.off_dev.data_ptr() + 8 * k0,
                          cnt, seg, batch.data_ptr() + 4 * b0 * C * seg)
            y = self._forward(batch, n)
            # Commit: in-place accumulations only, nothing left that allocates.
            for m, k0, cnt, b0 in runs:
                st = self.mixes[m]
                lo, hi = st.offsets[k0], min(st.L, st.offsets[k0 + cnt - 1] + seg)
                _lib.call("unblend_overlap_add", y.data_ptr() + 4 * b0 * S * C * seg, cnt, S * C, seg,
                          st.off_dev.data_ptr() + 8 * k0, st.L, lo, hi, self.power, st.acc.data_ptr(),
                          st.sum_w.data_ptr())
            if self.progress is not None:
                torch.cuda.synchronize(self.device)
        else:
            host = torch.zeros(rows, C, seg, dtype=torch.float32, pin_memory=True)
            for row, (m, k) in enumerate(items):
                st = self.mixes[m]
                o = st.offsets[k]
                ln = min(st.L - o, seg)
                start = o - (seg - ln) // 2
                a, b = max(0, start), min(st.L, start + seg)
                host[row, :, a - start:b - start] = st.track[:, a:b]
            y = self._forward(host.to(self.device, non_blocking=True), n)
            for m, k0, cnt, b0 in runs:
                st = self.mixes[m]
                _lib.call("unblend_weight_chunks", y.data_ptr() + 4 * b0 * S * C * seg, cnt, S * C, seg,
                          st.off_dev.data_ptr() + 8 * k0, st.L, self.power)
            out = torch.empty(n, S * C, seg, dtype=torch.float32, pin_memory=True)
            out.copy_(y[:n].view(n, S * C, seg), non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            for row, (m, k) in enumerate(items):
                st = self.mixes[m]
                o = st.offsets[k]
                ln = min(st.L - o, seg)
                trim = (seg - ln) // 2
                st.acc[:, o:o + ln] += out[row, :, trim:trim + ln]
                st.sum_w[o:o + ln] += self.weight[:ln]
        pending = []
        for m, _ in items:
            self.done += 1
            self.done_per[m] += 1
            pending.append({"completed_chunks": self.done, "total_chunks": sum(self.totals), "input_index": m,
                            "input_completed_chunks": self.done_per[m], "input_total_chunks": self.totals[m]})
        return pending

    def _emit(self, pending: list[dict]) -> None:
        if self.progress is not None:
            for payload in pending:
                self.progress("chunk_complete", payload)

    def _after_oom(self) -> None:
        torch.cuda.empty_cache()

    def run(self, pools: tuple[list, list] | None = None) -> None:
        full, tail = pools if pools is not None else _pools(self.totals, self.cbs)
        for pool in (full, tail):
            _drain(pool, self.run_batch, self._batch_size, self.backoff, self.fixed, self._after_oom, self._emit)

    def results(self) -> list[torch.Tensor]:
        """``out / sum_w`` per mix as ``[S, C, L]`` (on the device when resident, else on the host)."""
        outs = []
        for st in self.mixes:
            if self.resident:
                out = torch.empty_like(st.acc)
                _lib.call("unblend_divide", st.acc.data_ptr(), st.sum_w.data_ptr(), out.data_ptr(), st.acc.shape[0],
                          st.L)
            else:
                out = st.acc / st.sum_w
            outs.append(out.view(self.S, st.C, st.L))
        return outs


def _accumulate(model: Callable, mix: torch.Tensor, n_sources: int, segment: int, offsets: list[int],
                off_dev: torch.Tensor, chunk_batch_size: int, acc: torch.Tensor, sum_w: torch.Tensor,
                transition_power: float = 1.0) -> None:
    """Separate one device track's chunks at ``offsets`` into the given device ``acc``/``sum_w``.

    Used by the sharded engine, whose ranks each own a contiguous run of a
    track's chunks (``offsets`` ascending, ``off_dev`` the same values on the device).
    """
    st = _MixState(mix, list(offsets), off_dev, acc, sum_w)
    run = _PooledRun(model, [st], mix.device, segment, n_sources, chunk_batch_size, transition_power, None, None,
                     True)
    run.run(([(0, k) for k in range(len(offsets))], []))


def _resident(model: Any, lengths: list[int], channels: int, device: torch.device) -> bool:
    """Whether the tracks and accumulators of ``lengths`` fit the device budget."""
    need = sum(_gpu_accum_bytes_needed(1, len(model.sources), channels, n) for n in lengths)
    return need <= _gpu_accum_budget_bytes(device, getattr(model, "_forward_reserve_bytes", None))


def _unshifted(model: Any, tracks: list[torch.Tensor], device: torch.device, segment: int, stride: int,
               chunk_batch_size: int, transition_power: float, backoff: dict | None,
               progress: Callable | None, resident: bool) -> list[torch.Tensor]:
    """Pooled separation of ``[C, L]`` tracks (unblend/apply.py:1009-1333), resident or host accumulation."""
    S = len(model.sources)
    staged = [t.to(device, dtype=torch.float32, non_blocking=True).contiguous() if resident
              else t.to("cpu", dtype=torch.float32).contiguous() for t in tracks]
    mixes = [_MixState.plan(t, stride, S, resident, device) for t in staged]
    run = _PooledRun(model, mixes, device, segment, S, chunk_batch_size, transition_power, backoff, progress,
                     resident)
    run.run()
    return run.results()


def _validate_device(device: Any, mixes: list[torch.Tensor]) -> torch.device:
    if device is None:
        first = mixes[0].device if mixes else torch.device("cpu")
        if first.type == "cuda":
            return first
        if not torch.cuda.is_available():
            raise ValidationError("the B200 segment engine runs on CUDA devices only")
        return torch.device("cuda", torch.cuda.current_device())
    try:
        device = torch.device(device)
    except (TypeError, RuntimeError, ValueError) as e:
        raise ValidationError(f"Invalid device {device!r}: {e}") from e
    if device.type != "cuda":
        raise ValidationError("the B200 segment engine runs on CUDA devices only")
    if not torch.cuda.is_available():
        raise ValidationError("Device 'cuda' requested but CUDA is not available in this PyTorch build/environment.")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif device.index >= torch.cuda.device_count():
        raise ValidationError(f"Device 'cuda:{device.index}' requested but only {torch.cuda.device_count()} "
                              "CUDA device(s) are available.")
    return device


def apply_model_multi(model: Any, mixes: list[torch.Tensor], device: torch.device | str | None = None,
                      shifts: int = 0, overlap: float = 0.25, transition_power: float = 1.0,
                      progress_callback: Callable[[str, dict[str, Any]], None] | None = None,
                      use_only_stem: str | None = None, chunk_batch_size: int = 1,
                      oom_backoff_state: dict[str, int] | None = None, *,
                      _shift_offsets: list[list[int]] | None = None) -> list[torch.Tensor]:
    """Separate several mixes, pooling their tail chunks into shared batches (unblend/apply.py:567-1006).

    Each mix is chunked independently; the full batches of every mix run first,
    then the leftover chunks of all mixes are drained together, so every
    forward but the last holds ``chunk_batch_size`` chunks. Shift rounds draw
    one offset per mix per round (round-major). A :class:`ModelEnsemble` runs
    every member over the same offsets (or only the one-hot specialist for
    ``use_only_stem``) and weights the members' stems.

    :param mixes: ``[C, L]`` or ``[B, C, L]`` tensors on any device (rows of a
        batched mix are separated as separate mixes and restacked).
    :param oom_backoff_state: ``{"chunk_batch_size": n}`` opts into halving the
        batch on device out-of-memory; halvings persist in the dict. ``None``
        lets an OOM propagate.
    :return: One ``[S, C, L]`` (or ``[B, S, C, L]``) result per mix, on the mix's
        original device (page-locked host memory for host mixes).
    """
    if not 0.0 <= overlap < 1.0:
        raise ValidationError(f"overlap must be in [0, 1), got {overlap}")
    if not (_finite_number(transition_power) and transition_power >= 1):
        raise ValidationError(f"transition_power must be a finite number >= 1, got {transition_power}")
    if chunk_batch_size < 1:
        raise ValidationError("chunk_batch_size must be >= 1")
    device = _validate_device(device, list(mixes))
    if not mixes:
        return []
    # Batched mixes are separated row by row inside one pooled run.
    rows: list[torch.Tensor] = []
    spans: list[tuple[int, bool]] = []
    for mix in mixes:
        if mix.dim() == 2:
            rows.append(mix)
            spans.append((1, True))
        elif mix.dim() == 3:
            rows += [mix[b] for b in range(mix.shape[0])]
            spans.append((mix.shape[0], False))
        else:
            raise ValidationError(f"expected [C, L] or [B, C, L] mixes, got {tuple(mix.shape)}")
    if shifts and _shift_offsets is None:
        max_shift = int(0.5 * model.samplerate)
        _shift_offsets = [[random.randint(0, max_shift) for _ in rows] for _ in range(shifts)]
    with torch.cuda.device(device):
        flat = _separate_rows(model, rows, device, shifts, overlap, transition_power, progress_callback,
                              use_only_stem, chunk_batch_size, oom_backoff_state, _shift_offsets)
    out, i = [], 0
    for n, squeeze in spans:
        part = flat[i] if squeeze else torch.stack(flat[i:i + n])
        i += n
        orig = mixes[len(out)].device
        out.append(_to_host(part) if orig.type == "cpu" and part.device.type == "cuda" else part.to(orig))
    return out


def _separate_rows(model: Any, rows: list[torch.Tensor], device: torch.device, shifts: int, overlap: float,
                   transition_power: float, progress: Callable | None, use_only_stem: str | None,
                   chunk_batch_size: int, backoff: dict | None, shift_offsets: list[list[int]] | None
                   ) -> list[torch.Tensor]:
    """``[C, L]`` rows -> ``[S, C, L]`` results on the device (ensembles, shifts, pooling)."""
    if getattr(model, "models", None) is not None and hasattr(model, "weights"):
        return _separate_ensemble(model, rows, device, shifts, overlap, transition_power, progress,
                                  use_only_stem, chunk_batch_size, backoff, shift_offsets)
    segment, stride = _segment_plan(model, overlap)
    counts = _planned_counts(model, rows, shifts, overlap, shift_offsets)
    inner = progress
    if progress is not None:
        state = {"done": 0, "per": [0] * len(rows)}

        def inner(event: str, data: dict) -> None:
            if event != "chunk_complete":
                return
            m = int(data["input_index"])
            state["done"] += 1
            state["per"][m] += 1
            progress("chunk_complete", {"completed_chunks": state["done"], "total_chunks": sum(counts),
                                        "input_index": m, "input_completed_chunks": state["per"][m],
                                        "input_total_chunks": counts[m]})
        progress("processing_start", {"total_chunks": sum(counts), "total_inputs": len(rows),
                                      "input_total_chunks": counts})
    C = rows[0].shape[0]
    if not shifts:
        resident = _resident(model, [t.shape[-1] for t in rows], C, device)
        res = _unshifted(model, rows, device, segment, stride, chunk_batch_size, transition_power, backoff, inner,
                         resident)
    else:
        max_shift = int(0.5 * model.samplerate)
        resident = _resident(model, [t.shape[-1] + 2 * max_shift for t in rows], C, device)
        home = device if resident else torch.device("cpu")
        padded = [torch.nn.functional.pad(t.to(home, dtype=torch.float32), (max_shift, max_shift)) for t in rows]
        acc: list[torch.Tensor | None] = [None] * len(rows)
        for offs in shift_offsets:
            shifted = [p[:, off:p.shape[-1] - max_shift] for p, off in zip(padded, offs)]
            parts = _unshifted(model, shifted, device, segment, stride, chunk_batch_size, transition_power,
                               backoff, inner, resident)
            for i, (part, off) in enumerate(zip(parts, offs)):
                trimmed = part[..., max_shift - off:][..., :rows[i].shape[-1]]
                acc[i] = trimmed.clone() if acc[i] is None else acc[i].add_(trimmed)
        res = [a / len(shift_offsets) for a in acc]  # type: ignore[operator]
    if progress is not None:
        progress("processing_complete", {"total_chunks": sum(counts), "total_inputs": len(rows),
                                         "input_total_chunks": counts})
    return res


def _planned_counts(model: Any, rows: list[torch.Tensor], shifts: int, overlap: float,
                    shift_offsets: list[list[int]] | None) -> list[int]:
    """Exact chunk count per row over all shift rounds (unblend/apply.py:434-475)."""
    _, stride = _segment_plan(model, overlap)
    if not shifts:
        return [-(-t.shape[-1] // stride) for t in rows]
    max_shift = int(0.5 * model.samplerate)
    return [sum(-(-(t.shape[-1] + max_shift - offs[i]) // stride) for offs in shift_offsets)
            for i, t in enumerate(rows)]


def _separate_ensemble(ens: Any, rows: list[torch.Tensor], device: torch.device, shifts: int, overlap: float,
                       transition_power: float, progress: Callable | None, use_only_stem: str | None,
                       chunk_batch_size: int, backoff: dict | None, shift_offsets: list[list[int]] | None
                       ) -> list[torch.Tensor]:
    """Weighted member sum over shared offsets, or the lone one-hot specialist (unblend/apply.py:722-867)."""
    totals = ens.validated_weight_totals()
    args = (device, shifts, overlap, transition_power)
    pick = ens.specialist_for(use_only_stem) if hasattr(ens, "specialist_for") else None
    if pick is not None:
        return _separate_rows(ens.models[pick], rows, *args, progress, None, chunk_batch_size, backoff,
                              shift_offsets)
    per_member = [_planned_counts(m, rows, shifts, overlap, shift_offsets) for m in ens.models]
    agg = [sum(c[i] for c in per_member) for i in range(len(rows))]
    sub = None
    if progress is not None:
        progress("processing_start", {"total_chunks": sum(agg), "total_inputs": len(rows),
                                      "input_total_chunks": agg})
        state = {"member": 0}

        def sub(event: str, data: dict) -> None:
            if event != "chunk_complete":
                return
            m = int(data["input_index"])
            before = per_member[:state["member"]]
            progress("chunk_complete", {
                "completed_chunks": sum(sum(c) for c in before) + int(data["completed_chunks"]),
                "total_chunks": sum(agg), "input_index": m,
                "input_completed_chunks": sum(c[m] for c in before) + int(data["input_completed_chunks"]),
                "input_total_chunks": agg[m]})
    acc: list[torch.Tensor] | None = None
    for i, (member, wrow) in enumerate(zip(ens.models, ens.weights)):
        if sub is not None:
            state["member"] = i
        outs = _separate_rows(member, rows, *args, sub, None, chunk_batch_size, backoff, shift_offsets)
        w = torch.tensor([float(v) for v in wrow], dtype=torch.float32, device=outs[0].device).view(-1, 1, 1)
        outs = [o * w.to(o.device) for o in outs]
        acc = outs if acc is None else [a.add_(o) for a, o in zip(acc, outs)]
    t = torch.tensor(totals, dtype=torch.float32).view(-1, 1, 1)
    res = [a / t.to(a.device) for a in acc]  # type: ignore[union-attr]
    if progress is not None:
        progress("processing_complete", {"total_chunks": sum(agg), "total_inputs": len(rows),
                                         "input_total_chunks": agg})
    return res


def apply_model(model: Any, mix: torch.Tensor, device: torch.device | str | None = None, shifts: int = 0,
                overlap: float = 0.25, transition_power: float = 1.0,
                progress_callback: Callable[[str, dict[str, Any]], None] | None = None,
                use_only_stem: str | None = None, chunk_batch_size: int = 1,
                oom_backoff_state: dict[str, int] | None = None,
                shift_offsets: list[int] | None = None) -> torch.Tensor:
    """Separate ``mix`` ([C, L] or [B, C, L]) with ``model`` over overlapping segments (unblend/apply.py:500-564).

    :param model: Object with ``sources``, ``samplerate``, ``max_allowed_segment`` and a
        CUDA ``__call__(batch[B, C, T]) -> [B, S, C, T]`` (e.g. :class:`HTDemucsCuda`), or a
        :class:`ModelEnsemble` of them.
    :param mix: Mixture on any device; it is staged to ``device`` once (or kept on the host
        with host accumulators when the accumulators would not fit the device).
    :param device: CUDA device (defaults to the mix's device, or the current CUDA device).
    :param shifts: Number of random-shift rounds to average (0 = none).
    :param overlap: Segment overlap in [0, 1).
    :param transition_power: Exponent of the triangular cross-fade (>= 1).
    :param progress_callback: Optional ``(event, payload)`` callback; attaching one
        synchronises the device after each batch (as the reference's CUDA path does).
    :param use_only_stem: For a :class:`ModelEnsemble` of specialists, run only the member whose
        weight row is one-hot on this stem (its output still holds every source); no effect otherwise.
    :param chunk_batch_size: Segments per forward.
    :param oom_backoff_state: ``{"chunk_batch_size": n}`` to halve the batch on device OOM.
    :param shift_offsets: Explicit per-round offsets applied to every row instead of ``random`` draws.
    :return: ``[B, S, C, L]`` (or ``[S, C, L]`` for a 2-D mix) on the mix's original device.
    """
    plan = None
    if shifts and shift_offsets is not None:
        rows = 1 if mix.dim() == 2 else mix.shape[0]
        plan = [[off] * rows for off in shift_offsets]
    return apply_model_multi(model, [mix], device=device, shifts=shifts, overlap=overlap,
                             transition_power=transition_power, progress_callback=progress_callback,
                             use_only_stem=use_only_stem, chunk_batch_size=chunk_batch_size,
                             oom_backoff_state=oom_backoff_state, _shift_offsets=plan)[0]


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
