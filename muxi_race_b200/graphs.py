"""CUDA-graph capture of a fused MoE call.

Every library entry point is stream-ordered, keeps its block counts on the device and reuses a
cached workspace, so one call (alignment, gather, both grouped GEMMs) can be captured into a
CUDA graph and replayed with one launch: the per-kernel host launch cost (seven launches per call)
disappears, which is what dominates small, decode-sized calls.

    g = GraphedMoE(lambda x, ids, w, out: fused_moe(x, w13, w2, ids, w, out=out), x, ids, w, out)
    x.copy_(new_x); ids.copy_(new_ids); w.copy_(new_w)   # the captured buffers are the inputs
    g.replay()                                             # out holds the result

The first, uncaptured call done by the constructor sets the library's one-time per-kernel state
(shared-memory attributes, occupancy queries) that must not happen during a capture.
"""
from __future__ import annotations

from typing import Callable

import torch


class GraphedMoE:
    def __init__(self, fn: Callable, *buffers: torch.Tensor, warmup: int = 2):
        """``fn(*buffers)`` is one call on fixed device buffers (inputs then output)."""
        if not buffers or any(not t.is_cuda for t in buffers):
            raise ValueError("GraphedMoE needs CUDA buffers")
        self.fn = fn
        self.buffers = buffers
        side = torch.cuda.Stream(buffers[0].device)
        side.wait_stream(torch.cuda.current_stream(buffers[0].device))
        with torch.cuda.stream(side):
            for _ in range(max(warmup, 1)):
                fn(*buffers)
        torch.cuda.current_stream(buffers[0].device).wait_stream(side)
        torch.cuda.synchronize(buffers[0].device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            fn(*buffers)

    def replay(self) -> None:
        self.graph.replay()
