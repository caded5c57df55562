"""ctypes binding of ``libforma_b200.so`` (the C ABI in ``include/forma_b200.h``).

The library is built in-tree by ``forma_b200.build``.  There is no fallback:
if the shared library is missing, importing the operator API raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libforma_b200.so"
MAX_RANK = 8

F32, U32, F16, BF16 = 0, 1, 2, 3

# Status codes (mirror tensor_core::TensorError and compute_cuda::CudaError).
STATUS_NAMES = {
    0: "Ok",
    1: "ShapeOverflow",
    2: "LayoutOverflow",
    3: "RankMismatch",
    4: "AxisOutOfBounds",
    5: "DuplicateAxis",
    6: "IncompatibleBroadcast",
    7: "StorageOutOfBounds",
    8: "EmptyReduction",
    9: "InvalidEpsilon",
    10: "InvalidAttention",
    11: "InvalidAttentionScale",
    12: "InvalidConvolution",
    13: "LowDtypeMismatch",
    14: "MatmulRank",
    15: "MatmulInnerDimension",
    32: "InvalidInput",
    33: "Dtype",
    34: "Driver",
    35: "Unsupported",
    36: "ForeignRuntime",
    37: "MissingSymbol",
    38: "Graph",
    39: "ProgramPoisoned",
}


class FbTensor(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("storage_len", C.c_uint64),
        ("dtype", C.c_uint32),
        ("rank", C.c_uint32),
        ("dims", C.c_uint64 * MAX_RANK),
        ("strides", C.c_uint64 * MAX_RANK),
        ("offset", C.c_uint64),
    ]


class FbConvOptions(C.Structure):
    _fields_ = [
        ("strides", C.POINTER(C.c_uint64)),
        ("strides_len", C.c_uint32),
        ("dilations", C.POINTER(C.c_uint64)),
        ("dilations_len", C.c_uint32),
        ("padding_before", C.POINTER(C.c_uint64)),
        ("padding_before_len", C.c_uint32),
        ("padding_after", C.POINTER(C.c_uint64)),
        ("padding_after_len", C.c_uint32),
        ("groups", C.c_uint64),
    ]


class FbAttentionOptions(C.Structure):
    _fields_ = [
        ("has_scale", C.c_int32),
        ("scale", C.c_float),
        ("has_causal", C.c_int32),
        ("causal", C.c_int32),
    ]


T = C.POINTER(FbTensor)
U64P = C.POINTER(C.c_uint64)
U32P = C.POINTER(C.c_uint32)
VP = C.c_void_p

# name -> (restype, argtypes)
SIGNATURES = {
    "fb_abi_version": (C.c_int, []),
    "fb_status_string": (C.c_char_p, [C.c_int]),
    "fb_last_error": (C.c_char_p, []),
    "fb_launch_count": (C.c_uint64, []),
    "fb_last_route": (C.c_char_p, []),
    "fb_device_status": (C.c_uint32, []),
    "fb_conv_plan": (C.c_int, [U64P, C.c_uint32, U64P, C.c_uint32, C.POINTER(FbConvOptions), U64P, U32P]),
    "fb_conv": (C.c_int, [T, T, C.POINTER(FbConvOptions), T, VP]),
    "fb_conv_low_f32": (C.c_int, [T, T, C.POINTER(FbConvOptions), T, VP]),
    "fb_conv_low": (C.c_int, [T, T, C.POINTER(FbConvOptions), T, VP]),
    "fb_conv_low_gelu": (C.c_int, [T, T, C.POINTER(FbConvOptions), T, VP]),
    "fb_conv_low_f32_accumulate": (C.c_int, [T, T, C.POINTER(FbConvOptions), T, VP]),
    "fb_attention_plan": (
        C.c_int,
        [U64P, C.c_uint32, U64P, C.c_uint32, U64P, C.c_uint32, U64P, C.c_uint32, FbAttentionOptions, U64P, U32P],
    ),
    "fb_attention": (C.c_int, [T, T, T, C.c_uint32, T, FbAttentionOptions, T, VP]),
    "fb_attention_low_f32": (C.c_int, [T, T, T, C.c_uint32, T, FbAttentionOptions, T, VP]),
    "fb_attention_low": (C.c_int, [T, T, T, C.c_uint32, T, FbAttentionOptions, T, VP]),
    "fb_reduce_shape": (C.c_int, [C.c_uint32, U64P, C.c_uint32, U32P, C.c_uint32, C.c_int32, C.c_int32, U64P, U32P]),
    "fb_reduce_f32": (C.c_int, [C.c_uint32, T, U32P, C.c_uint32, C.c_int32, T, VP]),
    "fb_reduce_u32": (C.c_int, [C.c_uint32, T, U32P, C.c_uint32, C.c_int32, T, VP]),
    "fb_mean_axes": (C.c_int, [T, U32P, C.c_uint32, C.c_int32, T, VP]),
    "fb_argmax": (C.c_int, [T, C.c_uint32, C.c_int32, T, VP]),
    "fb_sum_partial_f64": (C.c_int, [T, VP, VP]),
    "fb_finish_sum_f64": (C.c_int, [VP, T, VP]),
    "fb_sum_partial_f64_static": (C.c_int, [T, VP, VP]),
    "fb_sum_static_max_elements": (C.c_uint64, []),
    "fb_softmax": (C.c_int, [T, U32P, C.c_uint32, T, VP]),
    "fb_log_softmax": (C.c_int, [T, U32P, C.c_uint32, T, VP]),
    "fb_logsumexp": (C.c_int, [T, U32P, C.c_uint32, C.c_int32, T, VP]),
    "fb_moments": (C.c_int, [T, U32P, C.c_uint32, C.c_int32, T, T, VP]),
    "fb_layer_norm": (C.c_int, [T, U32P, C.c_uint32, C.c_float, T, VP]),
    "fb_cast_to_low": (C.c_int, [T, T, VP]),
    "fb_matmul_plan": (C.c_int, [U64P, C.c_uint32, U64P, C.c_uint32, U64P, U32P]),
    "fb_matmul_low_f32": (C.c_int, [T, T, T, VP]),
    "fb_matmul_low": (C.c_int, [T, T, T, VP]),
    "fb_add": (C.c_int, [T, T, T, VP]),
    "fb_gelu_to_low": (C.c_int, [T, T, VP]),
    "fb_global_sum_nccl": (C.c_int, [T, VP, T, VP]),
    "fb_nccl_unique_id": (C.c_int, [VP]),
    "fb_nccl_comm_init_rank": (C.c_int, [C.POINTER(VP), C.c_int, VP, C.c_int]),
    "fb_nccl_comm_init_all": (C.c_int, [C.POINTER(VP), C.c_int, C.POINTER(C.c_int)]),
    "fb_nccl_comm_destroy": (C.c_int, [VP]),
    "fb_program_begin": (C.c_int, [VP]),
    "fb_program_end": (C.c_int, [VP, C.POINTER(VP)]),
    "fb_program_launch": (C.c_int, [VP, VP]),
    "fb_program_stats": (C.c_int, [VP, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_int32)]),
    "fb_program_destroy": (C.c_int, [VP]),
    "fb_selftest_bounded_wait": (C.c_int, [C.c_uint64, VP]),
}

NCCL_UNIQUE_ID_BYTES = 128

_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads the library once and declares every exported signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `python -m forma_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def u64_array(values) -> C.Array:
    values = list(values)
    return (C.c_uint64 * max(len(values), 1))(*values)


def u32_array(values) -> C.Array:
    values = list(values)
    return (C.c_uint32 * max(len(values), 1))(*values)
