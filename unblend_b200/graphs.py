"""CUDA-graph replay of a model's fixed-shape forward (the ``enable_compiled_core`` hook).

The reference compiles its hot core with ``torch.compile(mode="reduce-overhead")``
(unblend/htdemucs.py:553-583), i.e. CUDA graphs over a fixed batch shape, and
sets ``_fixed_batch_shape`` so ``apply_model`` zero-pads tail batches
(unblend/apply.py:1189-1196). Here the launch sequence of the CUDA forward is
captured as-is into a ``torch.cuda.CUDAGraph`` per input shape: the first call
with a shape runs the forward once eagerly (lazy kernel attributes, tables),
then captures it; later calls copy the input into the captured buffer and
replay the graph, so a forward costs one graph launch on the host instead of a
few hundred kernel launches. A batch smaller than one already captured (a tail)
runs eagerly at its own size; ``apply_model`` pads such tails up to the captured
shape only when they are within an eighth of it (``_eager_tails``).
"""

from __future__ import annotations

from typing import Callable

import torch

from . import _lib


class GraphedForward:
    """Replays ``fn`` (a ``[B, C, T] -> tensor`` CUDA forward) from CUDA graphs, one per input shape."""

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor]) -> None:
        self.fn = fn
        self.graphs: dict = {}

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        key = (tuple(x.shape), x.dtype, x.device)
        entry = self.graphs.get(key)
        if entry is None and any(k[0][1:] == key[0][1:] and k[0][0] > x.shape[0] and k[1:] == key[1:]
                                 for k in self.graphs):
            # A tail batch smaller than a captured one: eager launches at its own size
            # (a graph per tail size would hold a private memory pool each).
            return self.fn(x)
        if entry is None:
            static_in = x.clone()
            side = torch.cuda.Stream(device=x.device)
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                self.fn(static_in)  # eager warm-up: lazy attributes and cached tables
            torch.cuda.current_stream(x.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            before = _lib.counters["launches"]
            with torch.cuda.graph(graph, capture_error_mode="relaxed"):
                static_out = self.fn(static_in)
            # Kernels of this library inside the graph: counted again on every replay.
            kernels = _lib.counters["launches"] - before
            _lib.counters["launches"] = before
            entry = self.graphs[key] = (graph, static_in, static_out, kernels)
        graph, static_in, static_out, kernels = entry
        static_in.copy_(x)
        graph.replay()
        _lib.counters["launches"] += kernels
        return static_out.clone()

    def release(self) -> None:
        """Drop every captured graph and its private memory pool."""
        self.graphs.clear()
