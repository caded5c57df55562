"""Prepared programs: a recorded sequence of operator calls replayed as one
CUDA graph launch, through the C ABI's ``fb_program_*`` entry points.

The reference prepares typed programs and replays them, optionally as a
captured CUDA graph, with the same buffers (compute-cuda/src/program.rs:1-60,
program/graph.rs, program/execution.rs:20-150; attention and statistics steps
in program/builder_attention.rs:3-75 and program/statistics_launch.rs:17-214).
Here any Python callable that issues this library's operators (convolution
included) on the current stream is recorded once by ``fb_program_begin`` /
``fb_program_end`` and replayed by ``fb_program_launch``: host-side
validation, tensor-map encoding and per-kernel launch cost are paid while
recording only.  A failed replay poisons the program, as in the reference.

Recording rules (the same hold for a C-ABI caller):
  * the callable runs once eagerly on the recording stream first, so the
    library's per-(device, stream) scratch exists before recording (nothing
    is allocated while recording);
  * nothing that synchronises (``device_status``, host reads) inside it;
  * it may allocate only the tensors it returns (kept alive by the program):
    a temporary freed inside it would hand memory the graph still writes to
    back to torch's allocator, so the program counts the allocations made
    while recording and refuses any beyond the returned tensors;
  * every replay reads and writes the same device buffers: inputs are
    refreshed in place, outputs are read after a replay.
"""

from __future__ import annotations

import ctypes as C
from typing import Any, Callable

import torch

from . import api


def _storages(obj) -> list:
    """Distinct device storages of the tensors in a (nested) result."""
    found, seen = [], set()

    def walk(o):
        if isinstance(o, torch.Tensor):
            key = o.untyped_storage().data_ptr()
            if o.is_cuda and key not in seen:
                seen.add(key)
                found.append(o)
        elif isinstance(o, (list, tuple)):
            for x in o:
                walk(x)
        elif isinstance(o, dict):
            for x in o.values():
                walk(x)
        elif hasattr(o, "__dict__"):
            for x in vars(o).values():
                walk(x)

    walk(obj)
    return found


class Program:
    """``Program(fn, *args)`` runs ``fn(*args)`` once eagerly and once while
    recording; ``run()`` replays the recording on the current stream and
    returns the recorded call's result (the same tensors every time)."""

    def __init__(self, fn: Callable[..., Any], *args: Any, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._lib = api.lib()
        self.handle = None
        self.stream = torch.cuda.Stream(device=self.device)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            fn(*args)  # eager: scratch for this stream, kernel attributes, lazy library state
            self.stream.synchronize()
            s = C.c_void_p(self.stream.cuda_stream)
            allocs0 = torch.cuda.memory_stats(self.device).get("allocation.all.allocated", 0)
            api._check(self._lib.fb_program_begin(s))
            try:
                self.result = fn(*args)
            except BaseException:
                h = C.c_void_p()
                if self._lib.fb_program_end(s, C.byref(h)) == 0:
                    self._lib.fb_program_destroy(h)
                raise
            h = C.c_void_p()
            api._check(self._lib.fb_program_end(s, C.byref(h)))
            self.handle = h
            allocs = torch.cuda.memory_stats(self.device).get("allocation.all.allocated", 0) - allocs0
        if allocs > len(_storages(self.result)):
            raise api.TensorError(38, f"the recorded call allocated {allocs} device blocks but returns "
                                      f"{len(_storages(self.result))}: temporaries cannot live in a replayed program")
        torch.cuda.current_stream(self.device).wait_stream(self.stream)

    def stats(self) -> dict:
        """This library's kernels in the recording, graph nodes, poisoned flag."""
        k, n, p = C.c_uint64(), C.c_uint64(), C.c_int32()
        api._check(self._lib.fb_program_stats(self.handle, C.byref(k), C.byref(n), C.byref(p)))
        return {"kernel_launches": k.value, "graph_nodes": n.value, "poisoned": bool(p.value)}

    def run(self) -> Any:
        """Replays the program on the current stream."""
        with torch.cuda.device(self.device):
            api._check(self._lib.fb_program_launch(self.handle, C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return self.result

    def close(self) -> None:
        if self.handle is not None:
            self._lib.fb_program_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
