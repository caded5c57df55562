"""The reference's conformance fixtures, restated for this backend's tests.

Each builder follows the cited reference suite: same shapes, the same
deterministic dyadic ``data()`` values, the same views (permutations,
broadcasts) and the same tolerances.  Expected values come from the C oracle.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from oracle import oracle as orc

F32_MAX = float(np.finfo(np.float32).max)


@dataclass
class Host:
    """conformance Host<T> (conformance/attention.rs:4-25): physical values,
    an optional permutation and (conv only) an optional broadcast."""

    dims: list
    values: np.ndarray
    permutation: Optional[list] = None
    broadcast: Optional[list] = None

    def logical(self) -> np.ndarray:
        a = np.asarray(self.values).reshape(self.dims)
        if self.permutation is not None:
            a = np.transpose(a, self.permutation)
        if self.broadcast is not None:
            a = np.broadcast_to(a, self.broadcast)
        return np.ascontiguousarray(a)

    def to_device(self, torch, device, dtype=None):
        t = torch.as_tensor(np.asarray(self.values).reshape(self.dims)).to(device)
        if dtype is not None:
            t = t.to(dtype)
        if self.permutation is not None:
            t = t.permute(*self.permutation)
        if self.broadcast is not None:
            t = t.expand(*self.broadcast)
        return t


def data(dims, seed) -> Host:
    return Host(list(dims), orc.data(list(dims), seed).reshape(-1))


# ------------------------------------------------------------- convolution

@dataclass
class ConvCase:
    input: Host
    weight: Host
    strides: list
    dilations: list
    padding_before: list
    padding_after: list
    groups: int = 1


def conv_cases() -> list:
    """cases() of conformance/convolution.rs:77-178."""
    r = [
        ConvCase(data([2, 2, 9], 1), data([3, 2, 3], 2), [2], [2], [1], [2]),
        ConvCase(data([1, 3, 6, 5], 3), data([6, 1, 2, 3], 4), [1, 2], [2, 1], [0, 1], [1, 0], 3),
        ConvCase(data([1, 4, 4, 5, 6], 5), data([6, 2, 2, 2, 3], 6), [1, 2, 2], [2, 1, 1], [1, 0, 2], [0, 1, 0], 2),
        ConvCase(data([1, 2, 265], 7), data([3, 2, 257], 8), [1], [1], [0], [0]),
    ]
    for kernel in (255, 256, 257, 513):
        r.append(ConvCase(data([1, 1, kernel + 4], kernel), data([3, 1, kernel], kernel + 1), [1], [1], [0], [0]))
    i = data([2, 7, 4, 5], 9)
    i.permutation = [0, 2, 3, 1]
    w = data([2, 3, 6, 2], 10)
    w.permutation = [2, 0, 1, 3]
    r.append(ConvCase(i, w, [2, 1], [1, 2], [1, 2], [0, 1], 2))
    i = data([1, 1, 5, 1], 11)
    i.broadcast = [2, 4, 5, 7]
    w = data([1, 1, 3, 2], 12)
    w.broadcast = [6, 2, 3, 2]
    r.append(ConvCase(i, w, [1, 1], [1, 1], [0, 0], [0, 0], 2))
    for ind, wd in (([0, 2, 7], [4, 2, 3]), ([2, 2, 7], [0, 2, 3]), ([2, 0, 7], [4, 0, 3]), ([2, 2, 1], [3, 2, 3])):
        r.append(ConvCase(data(ind, 13), data(wd, 14), [1], [1], [0], [0]))
    r.append(ConvCase(data([2, 2, 0, 3], 15), data([4, 2, 2, 2], 16), [1, 1], [1, 1], [2, 1], [1, 0]))
    return r


def conv_expected(case: ConvCase, narrow=None) -> np.ndarray:
    x, w = case.input.logical(), case.weight.logical()
    if narrow is not None:
        x, w = narrow(x), narrow(w)
    return orc.conv(x, w, case.strides, case.dilations, case.padding_before, case.padding_after, case.groups)


# --------------------------------------------------------------- attention

@dataclass
class AttnCase:
    q: Host
    k: Host
    v: Host
    mask_kind: Optional[str] = None  # "keep" | "additive"
    mask: Optional[Host] = None
    scale: Optional[float] = None
    causal: Optional[int] = None


def attention_cases() -> list:
    """check_attention_backend (conformance/attention.rs:256-473)."""
    r = []
    for m, n, d, dv in ((3, 5, 7, 9), (33, 65, 17, 67), (2, 257, 65, 3), (1, 4097, 3, 5)):
        r.append(AttnCase(data([m, d], 1), data([n, d], 2), data([n, dv], 3)))
    r.append(AttnCase(data([2, 1, 6, 3, 5], 1), data([1, 3, 2, 7, 5], 2), data([3, 2, 7, 9], 3)))
    q = data([2, 5, 4, 3], 1)
    q.permutation = [0, 2, 3, 1]
    k = data([1, 7, 2, 5], 2)
    k.permutation = [0, 2, 1, 3]
    v = data([2, 9, 7], 3)
    v.permutation = [0, 2, 1]
    keep = Host([7, 3], np.array([0 if (i % 3 == 0 or i % 5 == 0) else 0xFFFFFFFF for i in range(21)], np.uint32),
                permutation=[1, 0])
    r.append(AttnCase(q, k, v, "keep", keep))
    for causal in (None, 0, 4, -2, -(2**31), 2**31 - 1):
        r.append(AttnCase(data([2, 4, 3, 5], 1), data([1, 2, 7, 5], 2), data([1, 2, 7, 4], 3), causal=causal))
    masks = [
        ("keep", Host([], np.array([0], np.uint32))),
        ("additive", Host([3, 7], np.array([-np.inf if (i // 7 == 1 or i % 4 == 0) else float(i % 5) - 2.0
                                            for i in range(21)], np.float32))),
        ("keep", Host([7], np.array([0, 1, 0xFFFFFFFF, 0, 7, 0, 1], np.uint32))),
    ]
    for kind, mask in masks:
        r.append(AttnCase(data([4, 3, 5], 1), data([2, 7, 5], 2), data([2, 7, 3], 3), kind, mask, scale=-0.5, causal=1))
    for scale in (0.0, 2.0, None):
        q = data([3, 1], 1)
        q.values = np.array([1.0, -1.0, 0.0], np.float32)
        k = data([65, 1], 2)
        k.values = np.array([10000.0 + (i % 7) for i in range(65)], np.float32)
        r.append(AttnCase(q, k, data([65, 5], 3), scale=scale))
    for m, d, large in ((1, 3, 1e30), (1, 64, F32_MAX), (17, 64, F32_MAX)):
        q = data([m, d], 1)
        q.values = np.zeros_like(q.values)
        k = data([65, d], 2)
        k.values = np.zeros_like(k.values)
        v = data([65, d], 3)
        v.values = np.full_like(v.values, large)
        r.append(AttnCase(q, k, v))
    q = data([1, 1], 1)
    q.values = np.ones(1, np.float32)
    k = data([65, 1], 2)
    k.values = np.array([0.0 if i < 32 else 200.0 for i in range(65)], np.float32)
    v = data([65, 1], 3)
    v.values = np.array([F32_MAX if i < 32 else 1.0 for i in range(65)], np.float32)
    r.append(AttnCase(q, k, v))
    q = data([1, 1], 1)
    q.values = np.zeros(1, np.float32)
    v = data([65, 1], 3)
    v.values = np.array([F32_MAX if i < 32 else 1.0 for i in range(65)], np.float32)
    keep = Host([65], np.array([1 if i >= 32 else 0 for i in range(65)], np.uint32))
    r.append(AttnCase(q, data([65, 1], 2), v, "keep", keep))
    for m in (1, 17):
        keep = Host([m, 65], np.array([0 if i // 65 == 0 else 1 for i in range(m * 65)], np.uint32))
        r.append(AttnCase(data([1, 4, m, 64], 1), data([1, 2, 65, 64], 2), data([1, 2, 65, 64], 3), "keep", keep))
    for m, n, dv in ((0, 3, 5), (3, 0, 5), (3, 5, 0)):
        r.append(AttnCase(data([m, 4], 1), data([n, 4], 2), data([n, dv], 3)))
    r.append(AttnCase(data([0, 4, 3, 5], 1), data([1, 2, 7, 5], 2), data([2, 7, 3], 3)))
    return r


def attention_expected(case: AttnCase, narrow=None) -> np.ndarray:
    q, k, v = case.q.logical(), case.k.logical(), case.v.logical()
    if narrow is not None:
        q, k, v = narrow(q), narrow(k), narrow(v)
    mask = None
    if case.mask is not None:
        m = case.mask.logical()
        if case.mask_kind == "keep":
            mask = np.where(m.astype(np.uint32) == 0, -np.inf, 0.0)
        else:
            mask = m.astype(np.float64)
    return orc.attention(q, k, v, mask, case.scale, case.causal)


# ------------------------------------------------------------- reductions

def reduce_float_values() -> np.ndarray:
    """conformance/reduction.rs:84-92."""
    return np.array([-1.0 if i % 5 == 0 else 1.0 + (i % 3) / 32.0 for i in range(30)], np.float32)


def reduce_uint_values() -> np.ndarray:
    """conformance/reduction.rs:93."""
    return np.array([(0xFFFFFFFF - i * 17) & 0xFFFFFFFF for i in range(30)], np.uint32)


def axis_masks():
    """axes for mask 0..8 in the suite's order (conformance/reduction.rs:103-107)."""
    for mask in range(8):
        yield [a for a in (2, 1, 0) if mask & (1 << a)]


def stats_values() -> np.ndarray:
    """conformance/statistics.rs:388."""
    return np.array([(i % 13) / 4.0 - 1.5 for i in range(30)], np.float32)


def huge_offset_rows() -> list:
    """conformance/statistics.rs:413-427."""
    fmax_bits = np.float32(F32_MAX).view(np.uint32)
    near = [np.array([fmax_bits - s * 65536], np.uint32).view(np.float32)[0] for s in (0, 1, 2, 4, 8)]
    return [
        np.full(257, 1e30, np.float32),
        np.array([1e8, 1e8 + 8.0, 1e8 + 16.0, 1e8 + 32.0, 1e8 + 64.0], np.float32),
        np.array([10000.0, 10001.0, 9998.0, -10000.0], np.float32),
        np.array([-1e30, 1e30, 0.0, 5e29, -5e29], np.float32),
        np.array([-F32_MAX, F32_MAX, 0.0], np.float32),
        np.array(near, np.float32),
        -np.array(near, np.float32),
    ]


# Tolerances of close() (conformance/statistics.rs:321-341, 357-379).
STATS_TOL = {"softmax": 4e-5, "log_softmax": 5e-5, "norm": 2e-4, "logsumexp": 5e-5, "mean": 2e-5, "variance": 2e-4}


def close(label: str, actual: np.ndarray, expected: np.ndarray, tol: float) -> None:
    actual = np.asarray(actual, np.float32).reshape(-1)
    expected = np.asarray(expected, np.float32).reshape(-1)
    assert actual.shape == expected.shape, f"{label} length"
    fmin = np.finfo(np.float32).tiny
    for i, (a, e) in enumerate(zip(actual, expected)):
        if np.isinf(e):
            assert a == e, f"{label}[{i}] infinity: {a} != {e}"
            continue
        if label in ("softmax", "variance"):
            scale = max(abs(float(e)), fmin / tol)
        else:
            scale = max(abs(float(e)), 1.0)
        assert np.isfinite(a) and abs(float(a) - float(e)) <= tol * scale, f"{label}[{i}]: {a!r} != {e!r}"


def check(actual, expected, tol=3e-5) -> None:
    """check() of conformance.rs:38-46: |a-b| <= tol * max(|b|, 1)."""
    a = np.asarray(actual, np.float64).reshape(-1)
    b = np.asarray(expected, np.float64).reshape(-1)
    assert a.shape == b.shape
    bad = ~(np.isfinite(a) & (np.abs(a - b) <= tol * np.maximum(np.abs(b), 1.0)))
    assert not bad.any(), f"first mismatch at {np.argmax(bad)}: {a[bad][:4]} != {b[bad][:4]}"
