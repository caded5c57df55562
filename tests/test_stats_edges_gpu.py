"""The reference's CUDA statistics edge cases (compute-cuda/tests/
cuda_tensor.rs:861-880 and :204-233), restated through this backend's API.

More rows than a bounded grid holds, a narrowed and transposed view (offset,
non-unit strides), values on a 1e8 common offset, and the chain moments ->
layer_norm -> softmax -> sum with every call enqueued before the first read.
The reference's tolerances are kept: close(actual, expected, atol, rtol)
accepts |a - e| <= atol + rtol * |e| (cuda_tensor.rs:14-22)."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ReduceOp

pytestmark = pytest.mark.gpu


def close(actual, expected, atol, rtol):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    assert a.shape == e.shape
    assert np.isfinite(a).all()
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), (int(np.argmax(bad)), a[bad][:4], e[bad][:4])


def test_statistics_large_grid_offset_transpose_chain(cuda):
    rows = 2051
    i = np.arange(rows * 19)
    row, col = i // 19, i % 19
    values = np.where((col == 0) | (col == 18), 99.0,
                      1e8 + (row % 5).astype(np.float32) * 64.0 + (col.astype(np.float32) - 9.0) * 8.0)
    values = values.astype(np.float32)
    backing = torch.from_numpy(values.reshape(rows, 19)).to(cuda)
    before = backing.clone()
    view = backing.narrow(1, 1, 17).permute(1, 0)  # [17, 2051], offset 1, strides (1, 19)
    moments = api.moments(view, [0])
    normalized = api.layer_norm(view, [0], 0.25)
    probabilities = api.softmax(normalized, [0])
    totals = api.reduce_f32(ReduceOp.Sum, probabilities, [0])
    # all enqueued before the first read
    close(moments.mean.cpu().numpy(), 1e8 + (np.arange(rows) % 5) * 64.0, 0.0, 0.0)
    close(moments.variance.cpu().numpy(), np.full(rows, 1536.0), 0.0, 0.0)
    close(totals.cpu().numpy(), np.ones(rows), 2e-6, 0.0)
    expected = np.repeat((np.arange(17) - 8.0) * 8.0 / np.sqrt(1536.25), rows)
    close(normalized.cpu().numpy(), expected, 2e-7, 2e-7)
    assert torch.equal(backing, before)
    assert api.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_low_statistics_offset_transpose(cuda, dtype):
    rows = 2053
    i = np.arange(rows * 9)
    values = np.where((i % 9 == 0) | (i % 9 == 8), 99.0, (i // 9 % 16) + (i % 9) - 4.0).astype(np.float32)
    backing = api.cast_to_low(torch.from_numpy(values.reshape(rows, 9)).to(cuda), dtype)
    bits = backing.view(torch.int16).clone()
    x = backing.narrow(1, 1, 7).permute(1, 0)  # [7, 2053] over 16-bit storage
    for _ in range(2):
        m = api.moments_low_f32(x, [0])
        assert np.array_equal(m.mean.cpu().numpy(), (np.arange(rows) % 16).astype(np.float32))
        assert np.array_equal(m.variance.cpu().numpy(), np.full(rows, 4.0, np.float32))
        normalized = api.layer_norm_low_f32(x, [0], 0.25)
        expected = np.repeat((np.arange(7) - 3.0) / np.sqrt(4.25), rows)
        close(normalized.cpu().numpy(), expected, 1e-7, 2e-6)
        sums = api.reduce_f32(ReduceOp.Sum, api.softmax_low_f32(x, [0]), [0])
        close(sums.cpu().numpy(), np.ones(rows), 2e-6, 2e-6)
    assert torch.equal(backing.view(torch.int16), bits)
    assert api.device_status() == 0
