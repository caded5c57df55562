"""This backend against the reference's own CUDA kernels, run on the same GPU
on the same inputs (the second oracle: oracle/ref_kernels.py launches the
kernels oracle/ref_build.sh compiled from the reference's sources).

* f32 convolution: bit-identical to the reference's conv_f32 (the same per-
  output f32 order with separately rounded multiply and add), on the C1
  geometry, on the reference's own grouped / strided / dilated / offset unit-
  test geometry (compute-cuda/src/convolution.rs:171-189), in 1-D and 3-D and
  on channels-last views;
* low convolution: the CUDA-core route bit-identical to the reference's
  conv_low, the tensor-core route within 1e-4 after normalisation;
* reductions: min / max bit-identical to reduce_axes, sum / product within
  the 1e-5 relative gate (scale max(|e|, 1));
* attention: the f32 path within 1e-5 of the reference's attention_f32 (both
  keep f64 state), the tensor-core path within the bf16 gate of attention_low.
"""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions, ConvOptions, ReduceOp
from oracle import ref_kernels as ref

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref.available(), reason="the reference kernels are built only where the "
                                                             "reference sources exist (oracle/ref_build.sh)")]


def bits(t):
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def rel(got, want):
    g = got.double().cpu().numpy()
    w = want.double().cpu().numpy()
    return float(np.abs(g - w).max() / max(float(np.abs(w).max()), 1.0))


def conv_pair(x, w, s, d, pb, pa, groups=1):
    mine = api.conv(x, w, ConvOptions(list(s), list(d), list(pb), list(pa), groups))
    theirs = ref.conv(x, w, s, d, pb, pa, groups)
    return mine, theirs


def test_f32_conv_bit_identical_at_c1_geometry(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.rand(2, 64, 56, 56, device=cuda, generator=g) * 2 - 1
    w = torch.randn(64, 64, 3, 3, device=cuda, generator=g) * (2 / 576) ** 0.5
    mine, theirs = conv_pair(x, w, [1, 1], [1, 1], [1, 1], [1, 1])
    assert api.last_route() == ["conv2d_f32_tiled_kernel<3,3>"]
    assert np.array_equal(bits(mine), bits(theirs))


def test_f32_conv_bit_identical_on_reference_unit_geometry(cuda):
    # convolution.rs:171-189: groups 2, strides [2, 1], dilations [1, 2], padding
    # [1, 2] / [0, 1], input offset 11 and weight offset 3 inside larger storage
    g = torch.Generator(device=cuda).manual_seed(1)
    xs = torch.randn(11 + 2 * 140, device=cuda, generator=g)
    ws = torch.randn(3 + 6 * 12, device=cuda, generator=g)
    x = xs[11:].view(2, 4, 5, 7)
    w = ws[3:].view(6, 2, 2, 3)
    mine, theirs = conv_pair(x, w, [2, 1], [1, 2], [1, 2], [0, 1], groups=2)
    assert list(mine.shape) == [2, 6, 3, 6]
    assert np.array_equal(bits(mine), bits(theirs))


@pytest.mark.parametrize("case", ["1d", "3d", "channels_last", "5x5_stride2"])
def test_f32_conv_bit_identical_other_ranks_and_layouts(cuda, case):
    g = torch.Generator(device=cuda).manual_seed(2)
    if case == "1d":
        x, w = torch.randn(3, 5, 40, device=cuda, generator=g), torch.randn(7, 5, 4, device=cuda, generator=g)
        args = ([1], [2], [3], [1])
    elif case == "3d":
        x, w = torch.randn(2, 3, 6, 7, 5, device=cuda, generator=g), torch.randn(4, 3, 2, 3, 2, device=cuda, generator=g)
        args = ([1, 2, 1], [1, 1, 2], [1, 0, 1], [0, 1, 1])
    elif case == "channels_last":
        x = torch.randn(2, 9, 11, 64, device=cuda, generator=g).permute(0, 3, 1, 2)
        w = torch.randn(32, 3, 3, 64, device=cuda, generator=g).permute(0, 3, 1, 2) * 0.1
        args = ([1, 1], [1, 1], [1, 1], [1, 1])
    else:
        x, w = torch.randn(2, 8, 17, 19, device=cuda, generator=g), torch.randn(32, 8, 5, 5, device=cuda, generator=g)
        args = ([2, 2], [1, 1], [2, 2], [2, 2])
    mine, theirs = conv_pair(x, w, *args)
    assert np.array_equal(bits(mine), bits(theirs))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_conv_against_reference_conv_low(cuda, dtype):
    g = torch.Generator(device=cuda).manual_seed(3)
    o = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])
    # NCHW storage: the CUDA-core route, the reference's own order
    x = torch.randn(2, 24, 10, 12, device=cuda, generator=g).to(dtype)
    w = (torch.randn(16, 24, 3, 3, device=cuda, generator=g) * 0.2).to(dtype)
    mine = api.conv_low_f32(x, w, o)
    assert api.last_route() == ["conv_direct_kernel"]
    assert np.array_equal(bits(mine), bits(ref.conv(x, w, [1, 1], [1, 1], [1, 1], [1, 1])))
    # channels-last at a tensor-core shape: f32 accumulation in another order
    xl = torch.randn(4, 14, 14, 256, device=cuda, generator=g).to(dtype).permute(0, 3, 1, 2)
    wl = (torch.randn(128, 3, 3, 256, device=cuda, generator=g) * 0.03).to(dtype).permute(0, 3, 1, 2)
    mine = api.conv_low_f32(xl, wl, o)
    assert api.last_route()[-1].startswith("conv_gemm")
    assert rel(mine, ref.conv(xl, wl, [1, 1], [1, 1], [1, 1], [1, 1])) <= 1e-4


@pytest.mark.parametrize("view", ["rows", "columns", "transposed"])
def test_reductions_against_reference_reduce_axes(cuda, view):
    g = torch.Generator(device=cuda).manual_seed(4)
    base = torch.randn(300, 1000, device=cuda, generator=g)
    x, axes = {"rows": (base, [1]), "columns": (base, [0]), "transposed": (base.t()[:, 1:], [0])}[view]
    for op in (ReduceOp.Min, ReduceOp.Max):
        assert np.array_equal(bits(api.reduce_f32(op, x, axes)), bits(ref.reduce_axes(int(op), x, axes)))
    assert rel(api.reduce_f32(ReduceOp.Sum, x, axes), ref.reduce_axes(0, x, axes)) <= 1e-5
    small = (x[:, :40] if view != "columns" else x[:40]) * 0.05 + 1.0  # products that stay in range
    assert rel(api.reduce_f32(ReduceOp.Product, small, axes), ref.reduce_axes(1, small, axes)) <= 1e-5


@pytest.mark.parametrize("causal", [None, 0, -3])
def test_f32_attention_against_reference_attention(cuda, causal):
    g = torch.Generator(device=cuda).manual_seed(5)
    q = torch.randn(2, 4, 70, 48, device=cuda, generator=g)
    k = torch.randn(2, 2, 90, 48, device=cuda, generator=g)
    v = torch.randn(2, 2, 90, 33, device=cuda, generator=g)
    mine = api.attention(q, k, v, None, AttentionOptions(None, causal))
    assert rel(mine, ref.attention(q, k, v, None, causal)) <= 1e-5


def test_tensor_core_attention_against_reference_attention_low(cuda):
    g = torch.Generator(device=cuda).manual_seed(6)
    q, k, v = (torch.randn(1, 4, 512, 128, device=cuda, generator=g).bfloat16() for _ in range(3))
    mine = api.attention_low_f32(q, k, v, None, AttentionOptions(None, 0))
    assert api.last_route()[0] == "attn_fwd_kernel<128,0,2>"  # 8 CTAs: key ranges split, then merged
    theirs = ref.attention(q, k, v, None, 0)
    err = float((mine - theirs).abs().max() / theirs.abs().max())
    assert err <= 5e-3, err
    assert api.device_status() == 0
