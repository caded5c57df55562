"""numpy front end of the C oracle (``oracle/liboracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
(as the checker) and ``bench.py``'s CPU-baseline leg.  The product path never
imports this module.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc, no CUDA)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = C.CDLL(str(LIB))
        _lib.oracle_attention.restype = C.c_uint64
        _lib.oracle_sum_f64.restype = C.c_double
        _lib.oracle_round_bf16.restype = C.c_uint16
        _lib.oracle_round_f16.restype = C.c_uint16
        _lib.oracle_decode_bf16.restype = C.c_float
        _lib.oracle_decode_f16.restype = C.c_float
        _lib.oracle_conv_dims.restype = C.c_int
    return _lib


def threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _u64(vals) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(vals), dtype=np.uint64).reshape(-1)) if len(vals) else np.zeros(1, np.uint64)


def _u32(vals) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(vals), dtype=np.uint32).reshape(-1)) if len(vals) else np.zeros(1, np.uint32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def data(dims, seed: int) -> np.ndarray:
    """conformance data() generator (conformance/attention.rs:26-35)."""
    n = int(np.prod(dims)) if len(dims) else 1
    out = np.empty(n, np.float32)
    if n:
        lib().oracle_data(C.c_uint64(n), C.c_uint64(seed), _p(out))
    return out.reshape(dims)


def conv_dims(in_dims, w_dims, strides, dilations, pad_before, pad_after) -> list:
    out = np.zeros(8, np.uint64)
    rank = len(in_dims)
    lib().oracle_conv_dims(_p(_u64(in_dims)), _p(_u64(w_dims)), rank, _p(_u64(strides)), _p(_u64(dilations)),
                           _p(_u64(pad_before)), _p(_u64(pad_after)), _p(out))
    return [int(x) for x in out[:rank]]


def _conv_call(fn, x, w, strides, dilations, pad_before, pad_after, groups, out_dtype, nthreads):
    x, w = _f32(x), _f32(w)
    dims = conv_dims(x.shape, w.shape, strides, dilations, pad_before, pad_after)
    out = np.zeros(max(int(np.prod(dims)), 1), out_dtype)
    fn(_p(_u64(x.shape)), _p(x), _p(_u64(w.shape)), _p(w), x.ndim, _p(_u64(strides)), _p(_u64(dilations)),
       _p(_u64(pad_before)), _p(_u64(pad_after)), C.c_uint64(groups), _p(out), nthreads)
    return out[: int(np.prod(dims))].reshape(dims)


def conv(x, w, strides, dilations, pad_before, pad_after, groups=1, nthreads=1) -> np.ndarray:
    """f64 cross-correlation (conformance/convolution.rs:180-231)."""
    return _conv_call(lib().oracle_conv, x, w, strides, dilations, pad_before, pad_after, groups, np.float64, nthreads)


def conv_f32_seq(x, w, strides, dilations, pad_before, pad_after, groups=1, nthreads=1) -> np.ndarray:
    """The reference kernel's f32 order (compute-cuda/src/convolution.cu:41-63)."""
    return _conv_call(lib().oracle_conv_f32_seq, x, w, strides, dilations, pad_before, pad_after, groups, np.float32,
                      nthreads)


def attention(q, k, v, mask=None, scale=None, causal=None, nthreads=1) -> np.ndarray:
    """Dense f64 attention (conformance/attention.rs:118-252).  ``mask`` is an
    additive f64 array (keep masks: 0 / -inf) broadcasting to the scores."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    qc = [1] + list(q.shape) if q.ndim == 2 else list(q.shape)
    kc = [1] + list(k.shape) if k.ndim == 2 else list(k.shape)
    vc = [1] + list(v.shape) if v.ndim == 2 else list(v.shape)
    br = max(len(qc), len(kc), len(vc)) - 3
    batches = [1] * br
    for d in (qc, kc, vc):
        pre = d[:-3]
        for i, x in enumerate(pre):
            if x != 1:
                batches[br - len(pre) + i] = x
    if q.ndim == 2 and k.ndim == 2 and v.ndim == 2:
        out_dims = [qc[-2], vc[-1]]
    else:
        out_dims = batches + [qc[-3], qc[-2], vc[-1]]
    n = int(np.prod(out_dims))
    out = np.zeros(max(n, 1), np.float64)
    m = None
    if mask is not None:
        m = np.ascontiguousarray(np.asarray(mask, dtype=np.float64))
    lib().oracle_attention(
        _p(_u64(q.shape)), q.ndim, _p(q), _p(_u64(k.shape)), k.ndim, _p(k), _p(_u64(v.shape)), v.ndim, _p(v),
        _p(_u64(m.shape)) if m is not None else None, m.ndim if m is not None else 0, _p(m) if m is not None else None,
        1 if scale is not None else 0, C.c_float(scale if scale is not None else 0.0),
        1 if causal is not None else 0, C.c_int32(causal if causal is not None else 0), _p(out), nthreads)
    return out[:n].reshape(out_dims)


def _kept(dims, axes):
    return [d for i, d in enumerate(dims) if i not in axes]


def reduce_f32(x, axes, op: int) -> np.ndarray:
    """expected_f32 (conformance/reduction.rs:24-54); op 0 sum 1 product 2 min 3 max."""
    x = _f32(x)
    kept = _kept(x.shape, axes)
    out = np.zeros(max(int(np.prod(kept)), 1), np.float32)
    lib().oracle_reduce_f32(_p(x), _p(_u64(x.shape)), x.ndim, _p(_u32(axes)), len(axes), op, _p(out))
    return out[: int(np.prod(kept))].reshape(kept)


def reduce_u32(x, axes, op: int) -> np.ndarray:
    x = np.ascontiguousarray(np.asarray(x, dtype=np.uint32))
    kept = _kept(x.shape, axes)
    out = np.zeros(max(int(np.prod(kept)), 1), np.uint32)
    lib().oracle_reduce_u32(_p(x), _p(_u64(x.shape)), x.ndim, _p(_u32(axes)), len(axes), op, _p(out))
    return out[: int(np.prod(kept))].reshape(kept)


def stats(x, axes, eps: float) -> dict:
    """Statistics reference (conformance/statistics.rs:267-319)."""
    x = _f32(x)
    kept = _kept(x.shape, axes)
    rows = int(np.prod(kept))
    r = {k: np.zeros(max(rows, 1), np.float32) for k in ("mean", "variance", "logsumexp")}
    e = {k: np.zeros(max(x.size, 1), np.float32) for k in ("softmax", "log_softmax", "norm")}
    lib().oracle_stats(_p(x), _p(_u64(x.shape)), x.ndim, _p(_u32(axes)), len(axes), C.c_float(eps),
                       _p(r["mean"]), _p(r["variance"]), _p(e["softmax"]), _p(e["log_softmax"]), _p(r["logsumexp"]),
                       _p(e["norm"]))
    out = {k: v[:rows].reshape(kept) for k, v in r.items()}
    out.update({k: v[: x.size].reshape(x.shape) for k, v in e.items()})
    return out


def row_stats(x, eps: float, nthreads=1, which=("mean", "variance", "softmax", "log_softmax", "logsumexp", "norm")):
    x = _f32(x)
    rows, cols = x.shape
    out = {}
    ptr = {}
    for k in ("mean", "variance", "logsumexp"):
        if k in which:
            out[k] = np.zeros(rows, np.float32)
            ptr[k] = _p(out[k])
    for k in ("softmax", "log_softmax", "norm"):
        if k in which:
            out[k] = np.zeros((rows, cols), np.float32)
            ptr[k] = _p(out[k])
    lib().oracle_row_stats(_p(x), C.c_uint64(rows), C.c_uint64(cols), C.c_float(eps), ptr.get("mean"),
                           ptr.get("variance"), ptr.get("softmax"), ptr.get("log_softmax"), ptr.get("logsumexp"),
                           ptr.get("norm"), nthreads)
    return out


def row_reduce(x, op: int, nthreads=1) -> np.ndarray:
    x = _f32(x)
    out = np.zeros(x.shape[0], np.float32)
    lib().oracle_row_reduce(_p(x), C.c_uint64(x.shape[0]), C.c_uint64(x.shape[1]), op, _p(out), nthreads)
    return out


def argmax_rows(x, nthreads=1) -> np.ndarray:
    """total_cmp argmax, lowest index on ties (host_tensor/similarity.rs:82)."""
    x = _f32(x)
    out = np.zeros(x.shape[0], np.uint32)
    lib().oracle_argmax_rows(_p(x), C.c_uint64(x.shape[0]), C.c_uint64(x.shape[1]), _p(out), nthreads)
    return out


def sum_f64(x, nthreads=1) -> float:
    x = _f32(x).reshape(-1)
    return float(lib().oracle_sum_f64(_p(x), C.c_uint64(x.size), nthreads))


def round_bits(x, dtype: str) -> np.ndarray:
    """Nearest-even f32 -> bf16/f16 bits by the conformance codec (conformance/low_ops.rs:20-51)."""
    fn = lib().oracle_round_bf16 if dtype == "bf16" else lib().oracle_round_f16
    flat = _f32(x).reshape(-1)
    return np.array([fn(C.c_float(float(v))) for v in flat], np.uint16).reshape(np.shape(x))


def decode_bits(b, dtype: str) -> np.ndarray:
    fn = lib().oracle_decode_bf16 if dtype == "bf16" else lib().oracle_decode_f16
    flat = np.asarray(b, np.uint16).reshape(-1)
    return np.array([fn(C.c_uint16(int(v))) for v in flat], np.float32).reshape(np.shape(b))
