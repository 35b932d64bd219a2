"""CUDA-graph replay for calls with fixed shapes and buffers.

At the reference's task shapes (tens of tokens) a call is a handful of short
kernels, and host-side launch work (Python, ctypes, allocator) is most of its
time. ``GraphCache`` runs a function eagerly the first time it sees a given
set of input tensors (shapes, dtypes, devices and data pointers), captures the
same call into a CUDA graph right after, and from then on replays the graph:
one launch. The replay reads whatever the input buffers hold at that moment,
so new values in the same tensors give new results; any other tensor (a new
pointer, shape or dtype) takes the eager path again and re-captures. Every call
returns new tensors, as the reference's ``ModelNew`` does
(``fused_moe/v1/fused_moe.py:320-341``): a replay copies the graph's own output
buffers, which the next replay rewrites, into fresh ones (one device copy per
output), so a result held by the caller never changes under a later call.
"""

from __future__ import annotations

from typing import Callable

import torch


def _fresh(out):
    if isinstance(out, torch.Tensor):
        return out.clone()
    return type(out)(_fresh(o) for o in out)


class GraphCache:
    def __init__(self, fn: Callable[..., torch.Tensor]):
        self.fn = fn
        self._key = None
        self._graph = None
        self._out = None
        self.replays = 0

    @staticmethod
    def _key_of(args):
        return tuple((t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype, t.device) if isinstance(t, torch.Tensor)
                     else ("v", t) for t in args)

    def __call__(self, *args):
        if not all(t.is_cuda for t in args if isinstance(t, torch.Tensor)):
            return self.fn(*args)  # the ops themselves reject host tensors
        key = self._key_of(args)
        if key == self._key and self._graph is not None:
            self._graph.replay()
            self.replays += 1
            return _fresh(self._out)
        out = self.fn(*args)  # eager: this call's result, and warm-up of every lazy setup
        dev = next(t.device for t in args if isinstance(t, torch.Tensor))
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                static_out = self.fn(*args)
        torch.cuda.current_stream(dev).wait_stream(side)
        self._key, self._graph, self._out = key, g, static_out
        return out
