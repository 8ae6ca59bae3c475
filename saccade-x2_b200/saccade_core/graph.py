"""CapturedStep: replay a fixed sequence of C-TARQ calls as one CUDA graph.

Decode-sized C-TARQ calls run for a few microseconds each, less than a host launch
costs, so a serving loop captures one step (host->device copies of the inputs, every
layer's sc_forward_ws, device->host copies of the outputs) once and replays it.  Every
library entry point used on the forward path is capturable: no host synchronisation,
no allocation (workspaces come from saccade_core.op.WORKSPACES, sized by a warm-up call
made before capture), and completion counters that each call returns to zero.
"""
from __future__ import annotations

import contextlib
import gc
from typing import Callable, Optional

import torch

from .op import flush_deferred


@contextlib.contextmanager
def no_gc():
    """Collects garbage, then keeps the collector off: a destructor that frees device memory must not
    run inside a CUDA graph capture (it would invalidate the capture)."""
    gc.collect()
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


class CapturedStep:
    def __init__(self, fn: Callable[[], None], device: Optional[torch.device] = None, warmup: int = 1):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.Stream(device=self.device)
        self.fn = fn
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            for _ in range(warmup):
                fn()  # sizes workspaces and sets kernel attributes outside the capture
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.device(self.device), no_gc():
            with torch.cuda.graph(self.graph, stream=self.stream):
                fn()
        self.stream.synchronize()
        flush_deferred()

    def replay(self) -> None:
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            self.graph.replay()

    def synchronize(self) -> None:
        self.stream.synchronize()
