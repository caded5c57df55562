"""The reference's own CUDA kernels as a second oracle (test infrastructure only).

``oracle/ref_build.sh`` compiles the reference's kernel sources, as the
reference's runtime hands them to NVRTC (compute-cuda/src/runtime.rs:15-29,
160-168), into ``oracle/_ref/reference_kernels.cubin``.  This module loads that
cubin through the CUDA driver API and launches its kernels with the argument
lists and metadata layouts the reference's Rust side builds, restated here:

* ``conv_f32`` / ``conv_low``: metadata of compute-cuda/src/convolution.rs:20-103
  (header: spatial rank, C/group, O/group, kernel volume, input/weight offsets,
  input N/C strides, weight O/C strides, O; then input/output/kernel dims,
  input/weight spatial strides, stride, dilation, padding before), launch as
  convolution.rs:110-140 (one thread per output, grid-stride);
* ``reduce_axes``: metadata of compute-cuda/src/reduction/dispatch.rs:52-103
  (kept dims, kept strides, reduced dims, reduced strides), 256 threads,
  min(outputs, 8 x SMs) blocks (dispatch.rs:41-49, 136-185);
* ``attention_f32`` / ``attention_low``: metadata of compute-cuda/src/
  attention_dispatch.rs:20-71 for dense or head-broadcast [batch, heads, L, D]
  operands, flags and launch of attention_dispatch.rs:107-230.

Outputs are torch CUDA tensors.  Nothing in the product imports this module.
"""

from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

import torch

CUBIN = Path(__file__).resolve().parent / "_ref" / "reference_kernels.cubin"

_cuda = None
_module = None
_functions: dict = {}


def available() -> bool:
    return CUBIN.exists()


def _driver():
    global _cuda
    if _cuda is None:
        _cuda = C.CDLL("libcuda.so.1")
        _cuda.cuModuleLoad.argtypes = [C.POINTER(C.c_void_p), C.c_char_p]
        _cuda.cuModuleGetFunction.argtypes = [C.POINTER(C.c_void_p), C.c_void_p, C.c_char_p]
        _cuda.cuLaunchKernel.argtypes = [C.c_void_p, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                         C.c_uint, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]
    return _cuda


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with CUDA driver error {rc}")


def _function(name: str):
    global _module
    if name in _functions:
        return _functions[name]
    drv = _driver()
    torch.cuda.init()
    torch.empty(1, device="cuda")  # the primary context is current on this thread
    if _module is None:
        mod = C.c_void_p()
        _check(drv.cuModuleLoad(C.byref(mod), str(CUBIN).encode()), "cuModuleLoad")
        _module = mod
    fn = C.c_void_p()
    _check(drv.cuModuleGetFunction(C.byref(fn), _module, name.encode()), f"cuModuleGetFunction({name})")
    _functions[name] = fn
    return fn


def _launch(name: str, grid: int, block: int, args: list) -> None:
    """args: ctypes scalars (c_void_p for pointers, c_uint64, c_uint32, c_float, c_int32)."""
    fn = _function(name)
    params = (C.c_void_p * len(args))(*[C.cast(C.pointer(a), C.c_void_p) for a in args])
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _check(_driver().cuLaunchKernel(fn, grid, 1, 1, block, 1, 1, 0, stream, params, None), f"launch {name}")


def _ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.untyped_storage().data_ptr())


def _u64(values) -> torch.Tensor:
    return torch.tensor([int(v) for v in values] or [0], dtype=torch.int64, device="cuda")


def _sms() -> int:
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def _low_code(dtype: torch.dtype) -> int:
    return {torch.float16: 0, torch.bfloat16: 1}[dtype]


# ------------------------------------------------------------------ conv

def conv_metadata(x_shape, x_strides, x_offset, w_shape, w_strides, w_offset, strides, dilations, pad_before,
                  pad_after, groups: int = 1):
    """(metadata, output spatial dims) of compute-cuda/src/convolution.rs:20-103."""
    rank = len(x_shape) - 2
    out_sp = []
    for d in range(rank):
        eff = (w_shape[d + 2] - 1) * dilations[d] + 1
        out_sp.append((x_shape[d + 2] + pad_before[d] + pad_after[d] - eff) // strides[d] + 1)
    meta = [rank, w_shape[1], w_shape[0] // groups, math.prod(w_shape[2:]), x_offset, w_offset,
            x_strides[0], x_strides[1], w_strides[0], w_strides[1], w_shape[0]]
    meta += list(x_shape[2:]) + out_sp + list(w_shape[2:]) + list(x_strides[2:]) + list(w_strides[2:])
    meta += list(strides) + list(dilations) + list(pad_before)
    return meta, out_sp


def conv(x: torch.Tensor, w: torch.Tensor, strides, dilations, pad_before, pad_after, groups: int = 1) -> torch.Tensor:
    """The reference's conv_f32 (f32 operands) or conv_low (f16/bf16 operands)
    kernel on any strided views; returns the contiguous f32 [N, O, *spatial]."""
    meta, out_sp = conv_metadata(list(x.shape), list(x.stride()), x.storage_offset(), list(w.shape), list(w.stride()),
                                 w.storage_offset(), strides, dilations, pad_before, pad_after, groups)
    out = torch.zeros(x.shape[0], w.shape[0], *out_sp, dtype=torch.float32, device=x.device)
    if out.numel() == 0 or x.numel() == 0:
        return out
    m = _u64(meta)
    count = out.numel()
    grid = max(1, min((count + 255) // 256, 65535 * 64))
    args = [_ptr(x), _ptr(w), _ptr(out), _ptr(m), C.c_uint64(count)]
    if x.dtype == torch.float32:
        _launch("conv_f32", grid, 256, args)
    else:
        _launch("conv_low", grid, 256, args + [C.c_uint32(_low_code(x.dtype))])
    torch.cuda.synchronize()
    return out


# ------------------------------------------------------------- reduction

def reduce_metadata(shape, strides, axes) -> list:
    """compute-cuda/src/reduction/dispatch.rs:52-103: kept dims and strides
    (in axis order), then the reduced axes' dims and strides in the order the
    caller lists them."""
    kept = [a for a in range(len(shape)) if a not in axes]
    return [shape[a] for a in kept] + [strides[a] for a in kept] + [shape[a] for a in axes] + [strides[a] for a in axes]


def reduce_axes(op: int, x: torch.Tensor, axes) -> torch.Tensor:
    """The reference's reduce_axes (f32) kernel: op 0 sum, 1 product, 2 min,
    3 max over `axes`; returns the contiguous f32 result without kept axes."""
    axes = list(axes)
    kept = [a for a in range(x.dim()) if a not in axes]
    out = torch.zeros([x.shape[a] for a in kept], dtype=torch.float32, device=x.device)
    out_count = out.numel()
    red_count = math.prod(x.shape[a] for a in axes)
    m = _u64(reduce_metadata(list(x.shape), list(x.stride()), axes))
    grid = max(1, min(out_count, 8 * _sms()))
    _launch("reduce_axes", grid, 256, [_ptr(x), _ptr(out), _ptr(m), C.c_uint64(out_count), C.c_uint64(red_count),
                                       C.c_uint32(len(kept)), C.c_uint32(len(axes)),
                                       C.c_uint64(x.storage_offset()), C.c_uint32(op)])
    torch.cuda.synchronize()
    return out


# ------------------------------------------------------------- attention

def attention_metadata(q_shape, q_strides, q_offset, k_strides, k_offset, v_strides, v_offset, group) -> list:
    """compute-cuda/src/attention_dispatch.rs:20-71 for [B, H, L, D] queries and
    [B, Hkv, Lk, D] keys/values without a mask: row dims, the Q/K/V/mask row
    strides (K/V query strides 0, no mask), then offsets, depth and key
    strides and the query heads per key/value head."""
    B, H, L, _ = q_shape
    return ([B, H, L] + list(q_strides[:3]) + [k_strides[0], k_strides[1], 0] + [v_strides[0], v_strides[1], 0] +
            [0, 0, 0] + [q_offset, k_offset, v_offset, 0, q_strides[3], k_strides[2], k_strides[3], v_strides[2],
                         v_strides[3], 0, group])


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale=None, causal=None) -> torch.Tensor:
    """The reference's attention_f32 (f32 operands) or attention_low (f16/bf16)
    kernel for [B, H, L, D] query and [B, Hkv, Lk, D] key/value views (Hkv
    dividing H; any strides), no mask; returns the contiguous f32 output."""
    B, H, L, D = q.shape
    Hkv, Lk, Dv = k.shape[1], k.shape[2], v.shape[3]
    group = H // Hkv
    out = torch.zeros(B, H, L, Dv, dtype=torch.float32, device=q.device)
    acc = torch.zeros(B * H * L * Dv, dtype=torch.float64, device=q.device)
    rows = B * H * L
    if rows == 0 or Lk == 0:
        return out
    m = _u64(attention_metadata(list(q.shape), list(q.stride()), q.storage_offset(), list(k.stride()),
                                k.storage_offset(), list(v.stride()), v.storage_offset(), group))
    sc = float(scale) if scale is not None else float(torch.tensor(1.0) / torch.tensor(float(D)).sqrt())
    flags = 4 if causal is not None else 0
    grid = max(1, min(rows, 8 * _sms()))
    args = [_ptr(q), _ptr(k), _ptr(v), _ptr(q), _ptr(q), _ptr(out), _ptr(acc), _ptr(m), C.c_uint64(rows),
            C.c_uint64(Lk), C.c_uint64(D), C.c_uint64(Dv), C.c_uint32(3), C.c_float(sc), C.c_uint32(flags),
            C.c_int32(causal or 0)]
    if q.dtype == torch.float32:
        _launch("attention_f32", grid, 256, args)
    else:
        _launch("attention_low", grid, 256, args + [C.c_uint32(_low_code(q.dtype))])
    torch.cuda.synchronize()
    return out
