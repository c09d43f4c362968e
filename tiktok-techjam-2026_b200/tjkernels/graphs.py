"""Whole-forward CUDA graph capture.

Same contract as the reference's ``tjkernels/graphs.py`` (:30-91): a captured
forward is bound to one input shape / dtype / mask presence; every ``run``
copies the live input (and mask) into the captured static buffers, replays,
and returns a clone of the static output, so results are correct for any
input, not only the captured one.  Warm-up runs on a side stream before
capture so that any lazy initialisation (kernel attributes, tensor-map
encoder lookup, allocator growth) happens outside the capture.
"""

from __future__ import annotations

from typing import Callable, Dict, Optional, Tuple

import torch

Forward = Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor]


class CapturedGraph:
    """One captured forward."""

    def __init__(self, fn: Forward, x: torch.Tensor, mask: Optional[torch.Tensor],
                 warmup: int = 2) -> None:
        self.static_x = x.clone()
        self.static_mask = None if mask is None else mask.clone()
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(self.static_x, self.static_mask)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_out = fn(self.static_x, self.static_mask)

    def run(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        self.static_x.copy_(x)
        if self.static_mask is not None and mask is not None:
            self.static_mask.copy_(mask)
        self.graph.replay()
        return self.static_out.clone()

    def replay_into(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        """Like ``run`` but returns the static output without cloning (valid
        until the next replay)."""
        self.static_x.copy_(x)
        if self.static_mask is not None and mask is not None:
            self.static_mask.copy_(mask)
        self.graph.replay()
        return self.static_out


class GraphCache:
    """Captured graphs keyed by everything that changes the captured work."""

    def __init__(self) -> None:
        self._graphs: Dict[Tuple, CapturedGraph] = {}

    def get(self, key: Tuple, fn: Forward, x: torch.Tensor,
            mask: Optional[torch.Tensor]) -> CapturedGraph:
        graph = self._graphs.get(key)
        if graph is None:
            graph = CapturedGraph(fn, x, mask)
            self._graphs[key] = graph
        return graph

    def clear(self) -> None:
        self._graphs.clear()

    def __len__(self) -> int:
        return len(self._graphs)
