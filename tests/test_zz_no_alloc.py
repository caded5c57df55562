"""The global-sum partial that allocates nothing (fb_sum_partial_f64_static).

Some callers cannot let a library call cudaMalloc: engines that reserve the
device's memory up front and route every allocation through their own pool,
and latency-critical paths that cannot absorb cudaMalloc's implicit device-wide
synchronisation.  This entry point keeps its scratch in a static device array
instead; it must give the allocating entry point's result, call after call.
Collected last on purpose, so a stop-at-first-failure run has already run
every other test if this one fails.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from forma_b200 import _lib, api

pytestmark = pytest.mark.gpu


def _sum(lib, fn, t, out):
    d = api.describe(t)
    rc = fn(C.byref(d), C.c_void_p(out.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.fb_last_error().decode()


def test_static_scratch_sum_matches_allocating_entry_point(cuda):
    lib = _lib.load()
    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(4096, 1000, device=cuda, generator=g)
    for t in (x, x.t(), x[:, :999], torch.randn(65536, 4096, device=cuda, generator=g)):
        for _ in range(2):  # two calls in a row: the shared array is re-armed each call
            want = torch.zeros((), dtype=torch.float64, device=cuda)
            got = torch.full((), float("nan"), dtype=torch.float64, device=cuda)
            _sum(lib, lib.fb_sum_partial_f64, t, want)
            _sum(lib, lib.fb_sum_partial_f64_static, t, got)
            torch.cuda.synchronize()
            a, b = want.item(), got.item()
            assert abs(a - b) <= 1e-9 * max(abs(a), 1.0), (a, b)
    assert api.device_status() == 0


def test_static_scratch_sum_rejects_oversized_input(cuda):
    lib = _lib.load()
    limit = lib.fb_sum_static_max_elements()
    assert limit == 8160 * 2**18  # (65536 - 256) / 8 partials, one per 2^18 elements
    d = _lib.FbTensor()
    d.data = 0x10000  # never dereferenced: the size check precedes any launch
    d.dtype = _lib.F32
    d.rank = 1
    d.dims[0] = limit + 1
    d.strides[0] = 1
    d.storage_len = limit + 1
    out = torch.zeros((), dtype=torch.float64, device=cuda)
    rc = lib.fb_sum_partial_f64_static(C.byref(d), C.c_void_p(out.data_ptr()), None)
    assert rc == 32 and b"at most" in lib.fb_last_error()
