"""C ABI checks that need no GPU: the library loads, exports every declared
symbol, and its host-side planners and validation match the reference's own
unit tests (all of which run before any device work)."""

import ctypes as C
import re
from pathlib import Path

import pytest

from forma_b200 import _lib, api
from forma_b200.api import AttentionOptions, ConvOptions, ReduceOp, TensorError

HEADER = Path(__file__).resolve().parent.parent / "include" / "forma_b200.h"


def declared_symbols():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(fb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"
    assert lib.fb_abi_version() == 1


def opts(strides, dilations, before, after, groups=1):
    return ConvOptions(list(strides), list(dilations), list(before), list(after), groups)


def test_conv_plan_geometry():
    # tensor-core/src/convolution.rs:141-172
    o = opts([2, 1], [1, 2], [1, 2], [0, 1], 4)
    assert api.conv_plan([2, 4, 5, 7], [8, 1, 3, 2], o) == [2, 8, 2, 8]
    assert api.conv_plan([1, 2, 5, 6, 7], [4, 2, 2, 3, 4], ConvOptions.new(3)) == [1, 4, 4, 4, 4]
    # zeros_have_geometry_even_without_a_contraction (convolution.rs:174-202)
    for i, w, out in (([0, 2, 5], [4, 2, 3], [0, 4, 3]), ([3, 0, 5], [4, 0, 3], [3, 4, 3]),
                      ([3, 2, 5], [0, 2, 3], [3, 0, 3]), ([3, 2, 1], [4, 2, 3], [3, 4, 0])):
        assert api.conv_plan(i, w, ConvOptions.new(1)) == out
    o = ConvOptions.new(1)
    o.padding_before[0] = 2
    o.padding_after[0] = 3
    assert api.conv_plan([2, 3, 0], [6, 3, 3], o) == [2, 6, 3]
    o.groups = 7
    assert api.conv_plan([2, 0, 1], [0, 0, 1], o) == [2, 0, 6]


def test_conv_plan_rejections():
    # invalid_geometry_is_not_bypassed_by_empty_inputs (convolution.rs:204-249)
    inp, w = [0, 4, 5], [6, 2, 3]
    o = ConvOptions.new(1)
    o.groups = 2
    assert api.conv_plan(inp, w, o) == [0, 6, 3]
    for rank in (0, 1, 2, 6):
        with pytest.raises(TensorError) as e:
            api.conv_plan([1] * rank, [1] * rank, ConvOptions.new(max(rank - 2, 0)))
        assert e.value.kind == "InvalidConvolution"
    with pytest.raises(TensorError):
        api.conv_plan(inp, [0, 2, 3, 1], o)
    for g in (0, 3, 4):
        bad = ConvOptions.new(1)
        bad.groups = g
        with pytest.raises(TensorError):
            api.conv_plan(inp, w, bad)
    with pytest.raises(TensorError):
        api.conv_plan(inp, [6, 1, 3], o)
    with pytest.raises(TensorError):
        api.conv_plan(inp, [6, 2, 0], o)
    for field in ("strides", "dilations", "padding_before", "padding_after"):
        bad = ConvOptions.new(1)
        bad.groups = 2
        getattr(bad, field).append(0)
        with pytest.raises(TensorError):
            api.conv_plan(inp, w, bad)
    for field in ("strides", "dilations"):
        bad = ConvOptions.new(1)
        bad.groups = 2
        getattr(bad, field)[0] = 0
        with pytest.raises(TensorError):
            api.conv_plan(inp, w, bad)
    # arithmetic_overflow_is_checked_including_empty_shapes (convolution.rs:251-283)
    umax = 2**64 - 1
    o = ConvOptions.new(1)
    o.padding_after[0] = 1
    with pytest.raises(TensorError) as e:
        api.conv_plan([0, 0, umax], [1, 0, 1], o)
    assert e.value.kind == "ShapeOverflow"
    o = ConvOptions.new(1)
    o.dilations[0] = 2
    with pytest.raises(TensorError) as e:
        api.conv_plan([0, 0, 1], [0, 0, umax], o)
    assert e.value.kind == "ShapeOverflow"
    assert api.conv_plan([0, 0, umax, umax], [0, 0, 1, 1], ConvOptions.new(2)) == [0, 0, umax, umax]


def test_attention_plan():
    o = AttentionOptions()
    assert api.attention_plan([3, 7], [5, 7], [5, 9], None, o) == [3, 9]
    assert api.attention_plan([2, 1, 6, 3, 5], [1, 3, 2, 7, 5], [3, 2, 7, 9], None, o) == [2, 3, 6, 3, 9]
    assert api.attention_plan([8, 32, 4096, 128], [8, 32, 4096, 128], [8, 32, 4096, 128], None,
                              AttentionOptions(causal=0)) == [8, 32, 4096, 128]
    # invalid cases of conformance/attention.rs:444-471
    with pytest.raises(TensorError) as e:
        api.attention_plan([3, 4], [7, 4], [7, 5], [2, 3, 7], o)
    assert e.value.kind == "IncompatibleBroadcast"
    for s in (float("nan"), float("inf"), float("-inf")):
        with pytest.raises(TensorError) as e:
            api.attention_plan([3, 4], [7, 4], [7, 5], None, AttentionOptions(scale=s))
        assert e.value.kind == "InvalidAttentionScale"
    with pytest.raises(TensorError) as e:
        api.attention_plan([], [7, 4], [7, 5], None, o)
    assert e.value.kind == "InvalidAttention"
    for q, k, v in (([3, 0], [7, 0], [7, 5]), ([3, 4], [7, 3], [7, 5]), ([3, 3, 4], [2, 7, 4], [2, 7, 5]),
                    ([3, 4], [7, 4], [6, 5]), ([4, 3, 4], [2, 7, 4], [3, 7, 5])):
        with pytest.raises(TensorError) as e:
            api.attention_plan(q, k, v, None, o)
        assert e.value.kind == "InvalidAttention"
    # empty geometry is valid (conformance/attention.rs:426-443)
    assert api.attention_plan([0, 4], [3, 4], [3, 5], None, o) == [0, 5]
    assert api.attention_plan([0, 4, 3, 5], [1, 2, 7, 5], [2, 7, 3], None, o) == [0, 4, 3, 3]


def test_reduce_shapes_and_rejections():
    assert api.reduce_shape(ReduceOp.Sum, [65536, 4096], [1], False) == [65536]
    assert api.reduce_shape(ReduceOp.Sum, [3, 2, 5], [2, 0], True) == [1, 2, 1]
    assert api.reduce_shape(ReduceOp.Sum, [2, 0, 3], [1], False) == [2, 3]
    with pytest.raises(TensorError) as e:
        api.reduce_shape(ReduceOp.Min, [2, 0, 3], [1], False)
    assert e.value.kind == "EmptyReduction"
    assert api.reduce_shape(ReduceOp.Min, [0, 0, 3], [1], True) == [0, 1, 3]
    with pytest.raises(TensorError) as e:
        api.reduce_shape(ReduceOp.Sum, [2, 3, 5], [0, 0], False)
    assert e.value.kind == "DuplicateAxis"
    with pytest.raises(TensorError) as e:
        api.reduce_shape(ReduceOp.Min, [2, 3, 5], [3], True)
    assert e.value.kind == "AxisOutOfBounds"
    with pytest.raises(TensorError) as e:
        api.reduce_shape(ReduceOp.Sum, [2, 0, 3], [1], False, mean=True)
    assert e.value.kind == "EmptyReduction"


def _desc(dims, dtype, strides=None, storage=None, ptr=0x10000):
    d = _lib.FbTensor()
    d.data = ptr
    d.dtype = dtype
    d.rank = len(dims)
    st = strides
    if st is None:
        st, s = [0] * len(dims), 1
        for i in range(len(dims) - 1, -1, -1):
            st[i] = s
            s *= dims[i]
    n = 1
    for x in dims:
        n *= x
    for i, (x, s) in enumerate(zip(dims, st)):
        d.dims[i] = x
        d.strides[i] = s
    d.storage_len = storage if storage is not None else n
    return d


def test_validation_precedes_any_launch():
    """Errors that the reference raises before touching the device; the
    descriptors point at no real memory, so reaching a launch would fail
    differently (Driver), which the assertions exclude."""
    lib = _lib.load()
    o, keep = api._conv_options(ConvOptions.new(1))
    # dtype mismatch precedes empty shortcuts and geometry (low_convolution.rs:345-365)
    a = _desc([0, 0, 3], _lib.F16)
    b = _desc([0, 0, 1], _lib.BF16)
    out = _desc([0, 0, 3], _lib.F32)
    assert lib.fb_conv_low_f32(C.byref(a), C.byref(b), C.byref(o), C.byref(out), None) == 13
    o3, keep3 = api._conv_options(ConvOptions.new(3))
    assert lib.fb_conv_low_f32(C.byref(a), C.byref(b), C.byref(o3), C.byref(out), None) == 13
    # storage bounds (Layout::validate_storage_len) before planning
    x = _desc([2, 3, 5], _lib.F32, storage=29)
    w = _desc([4, 3, 1], _lib.F32)
    y = _desc([2, 4, 5], _lib.F32)
    assert lib.fb_conv(C.byref(x), C.byref(w), C.byref(o), C.byref(y), None) == 7
    # f32 conv rejects low operands
    xl = _desc([2, 3, 5], _lib.BF16)
    assert lib.fb_conv(C.byref(xl), C.byref(w), C.byref(o), C.byref(y), None) == 33
    # planned output dims must match
    x = _desc([2, 3, 5], _lib.F32)
    bad = _desc([2, 4, 4], _lib.F32)
    assert lib.fb_conv(C.byref(x), C.byref(w), C.byref(o), C.byref(bad), None) == 32
    # layer norm epsilon (conformance/statistics.rs:479-482), also for empty inputs
    e = _desc([2, 0, 3], _lib.F32)
    ax = _lib.u32_array([1])
    for eps in (0.0, -0.0, -1.0, float("inf"), float("nan")):
        assert lib.fb_layer_norm(C.byref(e), ax, 1, C.c_float(eps), C.byref(e), None) == 9
    # statistics axes (conformance/statistics.rs:472-478)
    x = _desc([2, 3, 5], _lib.F32)
    for axes in ([3], [1, 1]):
        arr = _lib.u32_array(axes)
        assert lib.fb_softmax(C.byref(x), arr, len(axes), C.byref(x), None) in (4, 5)
    # reduce_u32 on an f32 tensor
    assert lib.fb_reduce_u32(0, C.byref(x), ax, 1, 0, C.byref(x), None) == 33
    # output aliasing a non-dense layout is rejected
    y = _desc([2, 5], _lib.F32, strides=[5, 0])
    assert lib.fb_reduce_f32(0, C.byref(x), ax, 1, 0, C.byref(y), None) == 32
    # fused projection entry points validate like conv_low / conv_low_f32
    xl = _desc([2, 3, 5], _lib.BF16)
    wl = _desc([4, 3, 1], _lib.BF16)
    y16 = _desc([2, 4, 5], _lib.BF16)
    y32 = _desc([2, 4, 5], _lib.F32)
    assert lib.fb_conv_low_gelu(C.byref(x), C.byref(w), C.byref(o), C.byref(y16), None) == 33  # f32 operands
    assert lib.fb_conv_low_gelu(C.byref(xl), C.byref(wl), C.byref(o), C.byref(y32), None) == 33  # output dtype
    assert lib.fb_conv_low_f32_accumulate(C.byref(xl), C.byref(wl), C.byref(o), C.byref(y16), None) == 33
    assert lib.fb_conv_low_f32_accumulate(C.byref(xl), C.byref(wl), C.byref(o), C.byref(_desc([2, 4, 4], _lib.F32)),
                                          None) == 32  # planned dims
    # an accumulated output may not overlap the input or the weight
    buf = (C.c_uint16 * 4096)()
    base = C.addressof(buf)
    xin = _desc([1, 4, 2, 2], _lib.BF16)
    xin.data = base
    wk = _desc([4, 4, 1, 1], _lib.BF16)
    wk.data = base + 1024
    acc = _desc([1, 4, 2, 2], _lib.F32)
    acc.data = base + 8  # inside the input's bytes
    o1, keep1 = api._conv_options(ConvOptions([1, 1], [1, 1], [0, 0], [0, 0]))
    assert lib.fb_conv_low_f32_accumulate(C.byref(xin), C.byref(wk), C.byref(o1), C.byref(acc), None) == 32
    assert b"overlaps" in lib.fb_last_error()
    # low GEMM: operands of one 16-bit dtype, planned output dims
    ml = _desc([3, 4], _lib.BF16)
    mr = _desc([4, 5], _lib.F16)
    mo = _desc([3, 5], _lib.F32)
    assert lib.fb_matmul_low_f32(C.byref(ml), C.byref(mr), C.byref(mo), None) == 32
    mr = _desc([4, 5], _lib.BF16)
    assert lib.fb_matmul_low_f32(C.byref(ml), C.byref(mr), C.byref(_desc([3, 4], _lib.F32)), None) == 32
    assert lib.fb_matmul_low(C.byref(ml), C.byref(mr), C.byref(mo), None) == 33  # matmul_low writes the operands' dtype
    assert lib.fb_matmul_low_f32(C.byref(ml), C.byref(_desc([5, 5], _lib.BF16)), C.byref(mo), None) == 15
    # attention_low: one 16-bit operand dtype, output in that dtype, a dense output block
    ao = api._attn_options(AttentionOptions())
    aq, ak = _desc([2, 3, 4], _lib.BF16), _desc([2, 7, 4], _lib.BF16)
    a16 = _desc([2, 3, 4], _lib.BF16)
    args = lambda q, k, v, out: (C.byref(q), C.byref(k), C.byref(v), 0, None, ao, C.byref(out), None)
    af = _desc([2, 3, 4], _lib.F32)
    assert lib.fb_attention_low(*args(af, af, af, a16)) == 33  # f32 operands
    assert lib.fb_attention_low(*args(aq, _desc([2, 7, 4], _lib.F16), ak, a16)) == 13
    assert lib.fb_attention_low(*args(aq, ak, ak, _desc([2, 3, 4], _lib.F32))) == 33  # output dtype
    assert lib.fb_attention_low(*args(aq, ak, ak, _desc([2, 3, 4], _lib.F16))) == 33
    gap = _desc([2, 3, 4], _lib.BF16, strides=[16, 5, 1], storage=32)  # rows with gaps: not a dense block
    assert lib.fb_attention_low(*args(aq, ak, ak, gap)) == 32
    assert b"address each element once" in lib.fb_last_error()
    # status strings
    assert lib.fb_status_string(8).decode().startswith("min, max and mean")


def test_matmul_plan_follows_reference_shapes():
    # MatmulPlan::new (tensor-core/src/shape.rs:148-192): promotion and broadcast
    assert api.matmul_plan([3], [3]) == []
    assert api.matmul_plan([2, 3], [3]) == [2]
    assert api.matmul_plan([3], [3, 4]) == [4]
    assert api.matmul_plan([5, 1, 2, 3], [4, 3, 6]) == [5, 4, 2, 6]
    with pytest.raises(api.TensorError) as e:
        api.matmul_plan([], [3])
    assert e.value.kind == "MatmulRank"
    with pytest.raises(api.TensorError) as e:
        api.matmul_plan([2, 3], [4, 5])
    assert e.value.kind == "MatmulInnerDimension"
    with pytest.raises(api.TensorError) as e:
        api.matmul_plan([2, 2, 3], [3, 3, 4])
    assert e.value.kind == "IncompatibleBroadcast"
