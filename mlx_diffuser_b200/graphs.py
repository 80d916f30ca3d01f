"""CUDA-graph capture of a fixed-topology forward pass.

A diffusion sampler runs the same sparse network on the same coordinates at every step: once the
kernel maps, row schedules and downsample coordinates sit in the SparseTensor cache, the forward
pass is a fixed sequence of kernel launches whose only inputs are feature values. Capturing that
sequence once and replaying it removes the per-launch host cost (Python, ctypes, torch dispatch),
which dominates at the SLat model's sizes (tens of thousands of voxels, 128 channels).

Everything this package launches inside a forward pass is capturable after one eager run:
convolutions, row norms, pooling and gathers take their scratch from torch's allocator and their
one-off host setup (kernel attributes, tensor-map entry point) happens on the first call.
Topology work (neighbour maps, plans, downsample sorting) synchronises the host and must therefore
already be cached when capture starts, which the warm-up runs ensure.
"""

from __future__ import annotations

from typing import Callable

import torch

from . import _native as N


class CapturedForward:
    """``fn(*tensors) -> tensor | tuple of tensors`` replayed from a CUDA graph.

    The first call copies its arguments into static buffers, runs ``fn`` ``warmup`` times on a
    side stream (filling every cache) and captures one more run. Later calls copy the new
    argument values into the static buffers and replay. Shapes, dtypes and devices must not
    change between calls; the returned tensors are the graph's static outputs, overwritten by
    the next call (clone them to keep them).
    """

    def __init__(self, fn: Callable[..., torch.Tensor | tuple], warmup: int = 2):
        self.fn = fn
        self.warmup = max(int(warmup), 1)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.static_inputs: tuple[torch.Tensor, ...] = ()
        self.static_outputs = None
        self.signature = None

    @staticmethod
    def _signature(inputs) -> tuple:
        return tuple((t.shape, t.dtype, t.device) for t in inputs)

    def capture(self, *inputs: torch.Tensor) -> None:
        if not inputs or not all(isinstance(t, torch.Tensor) and t.is_cuda for t in inputs):
            raise ValueError("CapturedForward needs CUDA tensor arguments")
        dev = inputs[0].device
        N.status_word(dev)  # allocated outside the graph's memory pool
        self.static_inputs = tuple(t.detach().clone() for t in inputs)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(self.warmup):
                self.fn(*self.static_inputs)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        N.check_device_status(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.static_outputs = self.fn(*self.static_inputs)
        self.graph = graph
        self.signature = self._signature(inputs)

    def __call__(self, *inputs: torch.Tensor):
        if self.graph is None:
            self.capture(*inputs)
        elif self._signature(inputs) != self.signature:
            raise ValueError("CapturedForward: argument shapes, dtypes or devices changed")
        for static, new in zip(self.static_inputs, inputs):
            if new is not static:
                static.copy_(new)
        self.graph.replay()
        return self.static_outputs

    def release(self) -> None:
        """Free the graph and its memory pool."""

        self.graph = None
        self.static_inputs = ()
        self.static_outputs = None


__all__ = ["CapturedForward"]
