"""Prepared programs: a recorded sequence of operator calls replayed as one
CUDA graph.

The reference prepares programs of attention / statistics steps and replays
them (compute-cuda/src/program/builder_attention.rs:3-75,
program/statistics_launch.rs:17-214).  Here any Python callable that issues
this library's operators (convolution included) on the current stream is
captured once with CUDA graph capture and replayed with a single launch:
host-side validation, tensor-map encoding and per-kernel launch cost are paid
at capture time only.

Capture rules (the same hold for a C-ABI caller capturing its own stream):
  * one eager call on the capture stream first, so that the library's
    per-(device, stream) scratch buffers exist before capture (allocation is
    not permitted while a stream is capturing);
  * no calls that synchronise (``device_status``, host reads) inside the
    captured region;
  * the captured program reads and writes the same device buffers on every
    replay: inputs are refreshed in place, outputs are read after replay.
"""

from __future__ import annotations

from typing import Any, Callable

import torch


class Program:
    """``Program(fn, *args)`` runs ``fn(*args)`` once eagerly (warm-up) and
    once under capture; ``run()`` replays the graph and returns the captured
    call's result (the same tensors every time)."""

    def __init__(self, fn: Callable[..., Any], *args: Any, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.Stream(device=self.device)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            fn(*args)  # warm-up: scratch for this stream, kernel attributes, lazy library state
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.result = fn(*args)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def run(self) -> Any:
        """Replays the program on the current stream."""
        self.graph.replay()
        return self.result
