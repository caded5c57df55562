"""Operator API of the B200 dense-op backend, mirroring Forma's tensor-core traits.

Each function corresponds to one trait method of the reference and keeps its
name, argument meaning, output shape and error behaviour:

==========================  =====================================================
this module                 reference (crates/tensor-core/src/...)
==========================  =====================================================
``conv``                    ``TensorConvBackend::conv`` (convolution.rs:125-132)
``conv_low_f32``/``conv_low``  ``TensorLowConvBackend`` (low_convolution.rs:16-44)
``attention``               ``TensorAttentionBackend::attention`` (attention.rs:49-58)
``attention_low_f32``       ``TensorLowAttentionBackend`` (low_attention.rs:28-49)
``reduce_f32``/``reduce_u32``/``mean_axes``  ``TensorReduceBackend`` (reduction.rs:20-41)
``softmax`` ... ``layer_norm``  ``TensorStatsBackend`` (statistics.rs:100-129), and the
                            ``*_low_f32`` methods of ``TensorLowStatsBackend`` for
                            f16/bf16 inputs (low_statistics.rs:25-57)
``argmax``                  new: ``Tensor::topk``'s ordering (host_tensor/similarity.rs:82)
``global_sum``              ``reduce_f32(Sum, all axes)`` with rows sharded over ranks
==========================  =====================================================

Tensors are torch CUDA tensors used purely as device memory: any strided view
(permuted, broadcast via ``expand``, offset) is passed through as a layout
descriptor, like the reference's ``CudaTensor`` = storage + ``Layout``.  F16 and
BF16 tensors are the reference's low storage (the same 16-bit patterns).
Outputs are freshly allocated and contiguous, like ``CudaRuntime::zeros``.
Errors raise :class:`TensorError` with the reference's error kind.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import FbAttentionOptions, FbConvOptions, FbTensor

_DTYPES = {torch.float32: _lib.F32, torch.int32: _lib.U32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
# u32 tensors are held as torch.int32 storage (same bits; torch has no uint32 arithmetic on CUDA).
_TORCH = {_lib.F32: torch.float32, _lib.U32: torch.int32, _lib.F16: torch.float16, _lib.BF16: torch.bfloat16}


class TensorError(RuntimeError):
    """A non-zero status from the C ABI; ``kind`` is the reference's variant name."""

    def __init__(self, status: int, detail: str):
        self.status = status
        self.kind = _lib.STATUS_NAMES.get(status, f"Status{status}")
        super().__init__(f"{self.kind}: {detail}")


class ReduceOp(IntEnum):
    """tensor_core::ReduceOp (reduction.rs:6-13)."""

    Sum = 0
    Product = 1
    Min = 2
    Max = 3


@dataclass
class ConvOptions:
    """tensor_core::ConvOptions (convolution.rs:7-26)."""

    strides: list = field(default_factory=list)
    dilations: list = field(default_factory=list)
    padding_before: list = field(default_factory=list)
    padding_after: list = field(default_factory=list)
    groups: int = 1

    @classmethod
    def new(cls, spatial_rank: int) -> "ConvOptions":
        return cls([1] * spatial_rank, [1] * spatial_rank, [0] * spatial_rank, [0] * spatial_rank, 1)


@dataclass
class AttentionOptions:
    """tensor_core::AttentionOptions (attention.rs:3-13)."""

    scale: Optional[float] = None
    causal: Optional[int] = None


@dataclass
class Mask:
    """tensor_core::AttentionMask: ``kind`` is "keep" (u32/int32 tensor) or "additive" (f32)."""

    kind: str
    tensor: torch.Tensor


@dataclass
class Moments:
    mean: torch.Tensor
    variance: torch.Tensor


def lib() -> C.CDLL:
    return _lib.load()


def _check(status: int) -> None:
    if status != 0:
        raise TensorError(status, lib().fb_last_error().decode(errors="replace"))


def describe(t: torch.Tensor) -> FbTensor:
    """Layout descriptor of a torch tensor view (storage + strides + offset, in elements)."""
    if t.dtype not in _DTYPES:
        raise TensorError(33, f"unsupported dtype {t.dtype}")
    if t.dim() > _lib.MAX_RANK:
        raise TensorError(32, f"rank {t.dim()} exceeds {_lib.MAX_RANK}")
    if any(s < 0 for s in t.stride()):
        raise TensorError(32, "negative strides require materialization")
    d = FbTensor()
    st = t.untyped_storage()
    d.data = st.data_ptr() if st.nbytes() else None
    d.storage_len = st.nbytes() // t.element_size()
    d.dtype = _DTYPES[t.dtype]
    d.rank = t.dim()
    for i, (n, s) in enumerate(zip(t.shape, t.stride())):
        d.dims[i] = n
        d.strides[i] = s
    d.offset = t.storage_offset()
    return d


def _stream(device: torch.device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _on:
    """Makes `device` current around one C call (every entry point runs on the
    current device, which must own its operands and stream) and restores the
    previous device afterwards; a no-op when it is current already."""

    __slots__ = ("device", "prev")

    def __init__(self, device: torch.device):
        self.device = device
        self.prev = None

    def __enter__(self) -> torch.device:
        cur = torch.cuda.current_device()
        if cur != self.device.index:
            self.prev = cur
            torch.cuda.set_device(self.device)
        return self.device

    def __exit__(self, *exc) -> None:
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _device(*ts: torch.Tensor) -> torch.device:
    """The one CUDA device that holds every given tensor."""
    dev = None
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise TensorError(32, "tensors must be CUDA device memory (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise TensorError(36, f"operands on {dev} and {t.device}: one call runs on one device")
    if dev is None:
        raise TensorError(32, "no tensor")
    return dev


def _conv_options(o: ConvOptions):
    keep = [_lib.u64_array(o.strides), _lib.u64_array(o.dilations), _lib.u64_array(o.padding_before),
            _lib.u64_array(o.padding_after)]
    opts = FbConvOptions(
        C.cast(keep[0], _lib.U64P), len(o.strides),
        C.cast(keep[1], _lib.U64P), len(o.dilations),
        C.cast(keep[2], _lib.U64P), len(o.padding_before),
        C.cast(keep[3], _lib.U64P), len(o.padding_after),
        o.groups,
    )
    return opts, keep


def _attn_options(o: AttentionOptions) -> FbAttentionOptions:
    return FbAttentionOptions(
        1 if o.scale is not None else 0,
        float(o.scale) if o.scale is not None else 0.0,
        1 if o.causal is not None else 0,
        int(o.causal) if o.causal is not None else 0,
    )


# ----------------------------------------------------------------- plans

def conv_plan(input_shape: Sequence[int], weight_shape: Sequence[int], options: ConvOptions) -> list:
    """ConvPlan::new output dims (host only)."""
    opts, _keep = _conv_options(options)
    out = (C.c_uint64 * _lib.MAX_RANK)()
    rank = C.c_uint32()
    _check(lib().fb_conv_plan(_lib.u64_array(input_shape), len(input_shape), _lib.u64_array(weight_shape),
                              len(weight_shape), C.byref(opts), out, C.byref(rank)))
    return [out[i] for i in range(rank.value)]


def attention_plan(q: Sequence[int], k: Sequence[int], v: Sequence[int], mask: Optional[Sequence[int]],
                   options: AttentionOptions) -> list:
    """AttentionPlan::new output dims (host only)."""
    out = (C.c_uint64 * _lib.MAX_RANK)()
    rank = C.c_uint32()
    m = _lib.u64_array(mask) if mask is not None else None
    _check(lib().fb_attention_plan(_lib.u64_array(q), len(q), _lib.u64_array(k), len(k), _lib.u64_array(v), len(v),
                                   C.cast(m, _lib.U64P) if m is not None else None, len(mask) if mask is not None else 0,
                                   _attn_options(options), out, C.byref(rank)))
    return [out[i] for i in range(rank.value)]


def reduce_shape(op: int, shape: Sequence[int], axes: Sequence[int], keep_dims: bool, mean: bool = False) -> list:
    """reduction_shape / mean_shape (host only)."""
    out = (C.c_uint64 * _lib.MAX_RANK)()
    rank = C.c_uint32()
    _check(lib().fb_reduce_shape(int(op), _lib.u64_array(shape), len(shape), _lib.u32_array(axes), len(axes),
                                 int(keep_dims), int(mean), out, C.byref(rank)))
    return [out[i] for i in range(rank.value)]


# ----------------------------------------------------------- convolution

def _conv(fn, input, weight, options, out_dtype):
    dev = _device(input, weight)
    opts, _keep = _conv_options(options)
    dims = conv_plan(list(input.shape), list(weight.shape), options)
    out = torch.empty(dims, dtype=out_dtype, device=dev)
    di, dw, do = describe(input), describe(weight), describe(out)
    with _on(dev) as dev_:
        _check(fn(C.byref(di), C.byref(dw), C.byref(opts), C.byref(do), _stream(dev_)))
    return out


def conv(input: torch.Tensor, weight: torch.Tensor, options: ConvOptions) -> torch.Tensor:
    """f32 cross-correlation, bit-identical to the reference kernel's f32 arithmetic."""
    return _conv(lib().fb_conv, input, weight, options, torch.float32)


def conv_low_f32(input: torch.Tensor, weight: torch.Tensor, options: ConvOptions) -> torch.Tensor:
    """f16/bf16 operands, f32 accumulation and output."""
    return _conv(lib().fb_conv_low_f32, input, weight, options, torch.float32)


def conv_low(input: torch.Tensor, weight: torch.Tensor, options: ConvOptions) -> torch.Tensor:
    """conv_low_f32 rounded once (nearest-even) to the input dtype."""
    return _conv(lib().fb_conv_low, input, weight, options, input.dtype)


def conv_low_f32_into(input, weight, options, out):
    """conv_low_f32 into a caller-provided output view (e.g. a channels-last permuted view)."""
    dev = _device(input, weight, out)
    opts, _keep = _conv_options(options)
    di, dw, do = describe(input), describe(weight), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_conv_low_f32(C.byref(di), C.byref(dw), C.byref(opts), C.byref(do), _stream(dev_)))
    return out


def conv_low_into(input, weight, options, out):
    """conv_low into a caller-provided 16-bit output view (e.g. channels-last)."""
    dev = _device(input, weight, out)
    opts, _keep = _conv_options(options)
    di, dw, do = describe(input), describe(weight), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_conv_low(C.byref(di), C.byref(dw), C.byref(opts), C.byref(do), _stream(dev_)))
    return out


def conv_low_gelu_into(input, weight, options, out):
    """gelu_to_low(conv_low_f32(input, weight)) into a 16-bit output view, the
    GELU applied in the tensor-core GEMM's epilogue (bit-identical)."""
    dev = _device(input, weight, out)
    opts, _keep = _conv_options(options)
    di, dw, do = describe(input), describe(weight), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_conv_low_gelu(C.byref(di), C.byref(dw), C.byref(opts), C.byref(do), _stream(dev_)))
    return out


def conv_low_f32_accumulate(input, weight, options, out):
    """out += conv_low_f32(input, weight) in place (f32 output view): a
    residual connection folded into the GEMM epilogue (bit-identical to add)."""
    dev = _device(input, weight, out)
    opts, _keep = _conv_options(options)
    di, dw, do = describe(input), describe(weight), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_conv_low_f32_accumulate(C.byref(di), C.byref(dw), C.byref(opts), C.byref(do), _stream(dev_)))
    return out


# ------------------------------------------------------- low-precision GEMM

def matmul_plan(left_shape: Sequence[int], right_shape: Sequence[int]) -> list:
    """MatmulPlan::new output dims (host only)."""
    out = (C.c_uint64 * _lib.MAX_RANK)()
    rank = C.c_uint32()
    _check(lib().fb_matmul_plan(_lib.u64_array(left_shape), len(left_shape), _lib.u64_array(right_shape),
                                len(right_shape), out, C.byref(rank)))
    return [out[i] for i in range(rank.value)]


def _matmul(fn, left, right, out_dtype, out=None):
    dev = _device(left, right, out)
    if out is None:
        out = torch.empty(matmul_plan(list(left.shape), list(right.shape)), dtype=out_dtype, device=dev)
    dl, dr, do = describe(left), describe(right), describe(out)
    with _on(dev) as dev_:
        _check(fn(C.byref(dl), C.byref(dr), C.byref(do), _stream(dev_)))
    return out


def matmul_low_f32(left: torch.Tensor, right: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """f16/bf16 operands (one dtype), f32 accumulation and output; vectors and batches broadcast."""
    return _matmul(lib().fb_matmul_low_f32, left, right, torch.float32, out)


def matmul_low(left: torch.Tensor, right: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """matmul_low_f32 rounded once (nearest even) to the operands' dtype."""
    return _matmul(lib().fb_matmul_low, left, right, left.dtype, out)


# ------------------------------------------------------------- attention

def _attention(fn, query, key, value, mask: Optional[Mask], options: AttentionOptions, out=None,
               out_dtype=torch.float32):
    dev = _device(query, key, value, out, mask.tensor if mask is not None else None)
    kind = 0
    dm = None
    if mask is not None:
        kind = {"keep": 1, "additive": 2}[mask.kind]
    if out is None:
        dims = attention_plan(list(query.shape), list(key.shape), list(value.shape),
                              list(mask.tensor.shape) if mask is not None else None, options)
        out = torch.empty(dims, dtype=out_dtype, device=dev)
    dq, dk, dv, do = describe(query), describe(key), describe(value), describe(out)
    if mask is not None:
        dm = describe(mask.tensor)
        if mask.kind == "keep":
            dm.dtype = _lib.U32
    with _on(dev) as dev_:
        _check(fn(C.byref(dq), C.byref(dk), C.byref(dv), kind, C.byref(dm) if dm is not None else None,
                  _attn_options(options), C.byref(do), _stream(dev_)))
    return out


def attention(query, key, value, mask: Optional[Mask] = None, options: AttentionOptions = AttentionOptions()):
    """softmax(scale * Q K^T + mask) V for f32 operands."""
    return _attention(lib().fb_attention, query, key, value, mask, options)


def attention_low_f32_into(query, key, value, mask: Optional[Mask], options: AttentionOptions, out):
    """attention_low_f32 into a caller-provided f32 output view (any row strides)."""
    return _attention(lib().fb_attention_low_f32, query, key, value, mask, options, out)


def attention_low_f32(query, key, value, mask: Optional[Mask] = None, options: AttentionOptions = AttentionOptions()):
    """Attention from f16/bf16 operands with f32 output."""
    return _attention(lib().fb_attention_low_f32, query, key, value, mask, options)


def attention_low_into(query, key, value, mask: Optional[Mask], options: AttentionOptions, out):
    """attention_low into a caller-provided 16-bit output view (a dense block in any axis order)."""
    return _attention(lib().fb_attention_low, query, key, value, mask, options, out)


def attention_low(query, key, value, mask: Optional[Mask] = None, options: AttentionOptions = AttentionOptions()):
    """attention_low_f32 rounded once (nearest even) to the operands' dtype
    (tensor-core/src/low_attention.rs:38-47)."""
    return _attention(lib().fb_attention_low, query, key, value, mask, options, out_dtype=query.dtype)


# ------------------------------------------------------------- reductions

def _reduce(fn, op, input, axes, keep_dims, mean, out_dtype):
    dev = _device(input)
    dims = reduce_shape(op, list(input.shape), axes, keep_dims, mean)
    out = torch.empty(dims, dtype=out_dtype, device=dev)
    di, do = describe(input), describe(out)
    if out_dtype == torch.int32:
        do.dtype = _lib.U32
        if input.dtype == torch.int32:
            di.dtype = _lib.U32
    ax = _lib.u32_array(axes)
    if mean:
        with _on(dev) as dev_:
            _check(fn(C.byref(di), ax, len(axes), int(keep_dims), C.byref(do), _stream(dev_)))
    else:
        with _on(dev) as dev_:
            _check(fn(int(op), C.byref(di), ax, len(axes), int(keep_dims), C.byref(do), _stream(dev_)))
    return out


def reduce_f32(op: ReduceOp, input: torch.Tensor, axes: Sequence[int], keep_dims: bool = False) -> torch.Tensor:
    return _reduce(lib().fb_reduce_f32, op, input, list(axes), keep_dims, False, torch.float32)


def reduce_u32(op: ReduceOp, input: torch.Tensor, axes: Sequence[int], keep_dims: bool = False) -> torch.Tensor:
    """u32 reduction; u32 data is carried in int32 tensors (same bits)."""
    return _reduce(lib().fb_reduce_u32, op, input, list(axes), keep_dims, False, torch.int32)


def mean_axes(input: torch.Tensor, axes: Sequence[int], keep_dims: bool = False) -> torch.Tensor:
    return _reduce(lib().fb_mean_axes, ReduceOp.Sum, input, list(axes), keep_dims, True, torch.float32)


def argmax(input: torch.Tensor, axis: int, keep_dims: bool = False) -> torch.Tensor:
    """Index of the maximum along ``axis`` (total order, lowest index on ties), as int32 holding u32."""
    dev = _device(input)
    dims = reduce_shape(ReduceOp.Max, list(input.shape), [axis], keep_dims)
    out = torch.empty(dims, dtype=torch.int32, device=dev)
    di, do = describe(input), describe(out)
    do.dtype = _lib.U32
    with _on(dev) as dev_:
        _check(lib().fb_argmax(C.byref(di), axis, int(keep_dims), C.byref(do), _stream(dev_)))
    return out


def sum_partial_f64(input: torch.Tensor, partial: Optional[torch.Tensor] = None) -> torch.Tensor:
    """f64 sum of every element, left on the device (one-element float64 tensor)."""
    dev = _device(input)
    if partial is None:
        partial = torch.empty((), dtype=torch.float64, device=dev)
    di = describe(input)
    with _on(dev) as dev_:
        _check(lib().fb_sum_partial_f64(C.byref(di), C.c_void_p(partial.data_ptr()), _stream(dev_)))
    return partial


def finish_sum(partial: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    dev = _device(partial, out)
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=dev)
    do = describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_finish_sum_f64(C.c_void_p(partial.data_ptr()), C.byref(do), _stream(dev_)))
    return out


class NcclCommunicator:
    """An NCCL communicator of one device, created and used through the C ABI
    (``fb_nccl_*``), for :func:`global_sum` across GPUs."""

    def __init__(self, handle: C.c_void_p, device: torch.device):
        self.handle, self.device = handle, device

    @staticmethod
    def unique_id() -> bytes:
        """A fresh NCCL unique id (rank 0 makes it and hands it to the others)."""
        buf = (C.c_char * _lib.NCCL_UNIQUE_ID_BYTES)()
        _check(lib().fb_nccl_unique_id(buf))
        return bytes(buf)

    @classmethod
    def init_rank(cls, nranks: int, unique_id: bytes, rank: int, device) -> "NcclCommunicator":
        """Joins rank `rank` of `nranks` on `device` (every rank calls this)."""
        device = torch.device(device)
        if len(unique_id) != _lib.NCCL_UNIQUE_ID_BYTES:
            raise TensorError(32, "an NCCL unique id has 128 bytes")
        uid = (C.c_char * _lib.NCCL_UNIQUE_ID_BYTES).from_buffer_copy(unique_id)
        h = C.c_void_p()
        with _on(device):
            _check(lib().fb_nccl_comm_init_rank(C.byref(h), nranks, uid, rank))
        return cls(h, device)

    def destroy(self) -> None:
        if self.handle is not None and self.handle.value:
            with _on(self.device):
                _check(lib().fb_nccl_comm_destroy(self.handle))
        self.handle = None


def global_sum(shard: torch.Tensor, comm: Optional[NcclCommunicator] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Sum over all elements of every rank's shard, rounded to f32 (a 0-d
    tensor).  With a communicator: ``fb_global_sum_nccl`` - this shard's f64
    partial, one 8-byte NCCL all-reduce and the rounding, all on the C side
    and the current stream (every rank of the communicator makes the call).
    Without one: this shard alone."""
    dev = _device(shard, out)
    if out is None:
        out = torch.empty((), dtype=torch.float32, device=dev)
    if comm is None:
        return finish_sum(sum_partial_f64(shard), out)
    if comm.device != dev:
        raise TensorError(36, f"communicator of {comm.device}, shard on {dev}")
    di, do = describe(shard), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_global_sum_nccl(C.byref(di), comm.handle, C.byref(do), _stream(dev_)))
    return out


# ------------------------------------------------------------- statistics

def _normalize(fn, input, axes, eps=None):
    dev = _device(input)
    out = torch.empty(list(input.shape), dtype=torch.float32, device=dev)
    di, do = describe(input), describe(out)
    ax = _lib.u32_array(axes)
    if eps is None:
        with _on(dev) as dev_:
            _check(fn(C.byref(di), ax, len(axes), C.byref(do), _stream(dev_)))
    else:
        with _on(dev) as dev_:
            _check(fn(C.byref(di), ax, len(axes), C.c_float(eps), C.byref(do), _stream(dev_)))
    return out


def softmax(input: torch.Tensor, axes: Sequence[int]) -> torch.Tensor:
    return _normalize(lib().fb_softmax, input, list(axes))


def log_softmax(input: torch.Tensor, axes: Sequence[int]) -> torch.Tensor:
    return _normalize(lib().fb_log_softmax, input, list(axes))


def layer_norm(input: torch.Tensor, axes: Sequence[int], epsilon: float) -> torch.Tensor:
    return _normalize(lib().fb_layer_norm, input, list(axes), float(epsilon))


def _normalize_low(fn, input, axes, dtype, eps=None, out=None):
    dev = _device(input, out)
    if out is None:
        out = torch.empty(list(input.shape), dtype=dtype, device=dev)
    ax = _lib.u32_array(axes)
    di, do = describe(input), describe(out)
    if eps is None:
        with _on(dev) as dev_:
            _check(fn(C.byref(di), ax, len(axes), C.byref(do), _stream(dev_)))
    else:
        with _on(dev) as dev_:
            _check(fn(C.byref(di), ax, len(axes), C.c_float(eps), C.byref(do), _stream(dev_)))
    return out


def softmax_low(input: torch.Tensor, axes: Sequence[int]) -> torch.Tensor:
    """softmax_low: f16/bf16 input, result rounded once to the input dtype."""
    return _normalize_low(lib().fb_softmax, input, axes, input.dtype)


def log_softmax_low(input: torch.Tensor, axes: Sequence[int]) -> torch.Tensor:
    """log_softmax_low: f16/bf16 input, result rounded once to the input dtype."""
    return _normalize_low(lib().fb_log_softmax, input, axes, input.dtype)


def layer_norm_low(input: torch.Tensor, axes: Sequence[int], epsilon: float, dtype: Optional[torch.dtype] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """layer_norm_low: result rounded once to ``dtype`` (the input's 16-bit dtype
    for the trait method; an f32 input may name bf16/f16 explicitly)."""
    return _normalize_low(lib().fb_layer_norm, input, axes, dtype or input.dtype, epsilon, out)


def logsumexp(input: torch.Tensor, axes: Sequence[int], keep_dims: bool = False) -> torch.Tensor:
    dev = _device(input)
    dims = reduce_shape(ReduceOp.Sum, list(input.shape), list(axes), keep_dims, True)
    out = torch.empty(dims, dtype=torch.float32, device=dev)
    di, do = describe(input), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_logsumexp(C.byref(di), _lib.u32_array(axes), len(axes), int(keep_dims), C.byref(do), _stream(dev_)))
    return out


def moments(input: torch.Tensor, axes: Sequence[int], keep_dims: bool = False) -> Moments:
    dev = _device(input)
    dims = reduce_shape(ReduceOp.Sum, list(input.shape), list(axes), keep_dims, True)
    mean = torch.empty(dims, dtype=torch.float32, device=dev)
    var = torch.empty(dims, dtype=torch.float32, device=dev)
    di, dm, dv = describe(input), describe(mean), describe(var)
    with _on(dev) as dev_:
        _check(lib().fb_moments(C.byref(di), _lib.u32_array(axes), len(axes), int(keep_dims), C.byref(dm), C.byref(dv),
                                _stream(dev_)))
    return Moments(mean, var)


# low-storage statistics are the same calls with f16/bf16 inputs
softmax_low_f32 = softmax
log_softmax_low_f32 = log_softmax
layer_norm_low_f32 = layer_norm
logsumexp_low_f32 = logsumexp
moments_low_f32 = moments


def cast_to_low(input: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    dev = _device(input)
    out = torch.empty(list(input.shape), dtype=dtype, device=dev)
    di, do = describe(input), describe(out)
    with _on(dev) as dev_:
        _check(lib().fb_cast_to_low(C.byref(di), C.byref(do), _stream(dev_)))
    return out


def cast_to_low_into(input: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """cast_to_low into a caller-owned contiguous tensor (chains reuse buffers)."""
    di, do = describe(input), describe(out)
    with _on(_device(input, out)) as dev_:
        _check(lib().fb_cast_to_low(C.byref(di), C.byref(do), _stream(dev_)))
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = a + b (f32), operands of out's shape with any strides (expand() broadcasts).

    Elementwise glue for chained workloads (residual additions); ``out`` may
    be ``a`` or ``b`` itself when that operand is contiguous."""
    if out is None:
        out = torch.empty(list(a.shape), dtype=torch.float32, device=_device(a, b))
    da, db, do = describe(a), describe(b), describe(out)
    with _on(_device(a, b, out)) as dev_:
        _check(lib().fb_add(C.byref(da), C.byref(db), C.byref(do), _stream(dev_)))
    return out


def gelu_to_low(input: torch.Tensor, dtype: torch.dtype, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """tanh-form GELU of an f32 tensor, rounded once to f16/bf16 (contiguous result)."""
    if out is None:
        out = torch.empty(list(input.shape), dtype=dtype, device=_device(input))
    di, do = describe(input), describe(out)
    with _on(_device(input, out)) as dev_:
        _check(lib().fb_gelu_to_low(C.byref(di), C.byref(do), _stream(dev_)))
    return out


def device_status() -> int:
    """Synchronises and returns (and clears) the mask of timed-out bounded waits."""
    return int(lib().fb_device_status())


def selftest_bounded_wait(limit_ns: int, device=None) -> None:
    """Enqueues a kernel whose bounded wait on an mbarrier nothing arrives at
    gives up after `limit_ns`; the timeout then shows in device_status()."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with _on(dev) as dev_:
        _check(lib().fb_selftest_bounded_wait(int(limit_ns), _stream(dev_)))


def launch_count() -> int:
    """Kernel launches this library has enqueued."""
    return int(lib().fb_launch_count())


def last_route() -> list:
    """Kernels the most recent call on this thread enqueued, in launch order
    (e.g. ``["conv_gemm_pair_kernel<192,12>"]``)."""
    r = lib().fb_last_route().decode()
    return r.split(";") if r else []
