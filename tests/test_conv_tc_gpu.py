"""The tcgen05 implicit-GEMM convolution (bf16/f16 channels-last) versus the
f64 oracle.  Shapes are chosen to take the tensor-core path: channels a
multiple of 64, input >= 128 KiB for the im2col map, one group."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ConvOptions
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def run_case(cuda, n, h, w, c, o, k, stride=1, pad=0, dtype=torch.bfloat16, ohwi=True, nchw_out=True, seed=0,
             expect=None):
    """`expect`: the tensor-core GEMM kernel the call must launch (fb_last_route)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, h, w, c, generator=g).to(dtype)
    wt = (torch.randn(o, k, k, c, generator=g) * (2.0 / (c * k * k)) ** 0.5).to(dtype)
    xv = x.to(cuda).permute(0, 3, 1, 2)  # [N, C, H, W] view of NHWC storage
    if ohwi:
        wv = wt.to(cuda).permute(0, 3, 1, 2)  # [O, C, kh, kw] view of OHWI storage
    else:
        wv = wt.permute(0, 3, 1, 2).contiguous().to(cuda)  # OIHW storage (gathered on device)
    opts = ConvOptions([stride, stride], [1, 1], [pad, pad], [pad, pad])
    before = api.launch_count()
    if nchw_out:
        out = api.conv_low_f32(xv, wv, opts)
    else:
        dims = api.conv_plan(list(xv.shape), list(wv.shape), opts)
        store = torch.empty(dims[0], dims[2], dims[3], dims[1], device=cuda)
        out = api.conv_low_f32_into(xv, wv, opts, store.permute(0, 3, 1, 2))
    route = api.last_route()
    assert expect in route, route  # the tensor cores served the call, not a CUDA-core fallback
    if not ohwi:
        assert route[0] == "weights_to_ohwi_kernel", route
    got = out.cpu().numpy()
    assert api.device_status() == 0, "a bounded wait timed out"
    assert api.launch_count() > before
    ref = orc.conv(xv.float().cpu().numpy(), wv.float().cpu().numpy(), [stride] * 2, [1, 1], [pad] * 2, [pad] * 2, 1,
                   nthreads=orc.threads())
    assert got.shape == ref.shape
    scale = max(float(np.abs(ref).max()), 1e-30)
    err = float(np.abs(got.astype(np.float64) - ref).max()) / scale
    # Parity gate: 2e-2 after normalisation by max|e|; f32 accumulation of
    # exact bf16 products is far tighter, so a layout bug cannot hide.
    assert err <= 2e-2, err
    assert err <= 1e-4, err
    return err


def test_tc_conv_1x1(cuda):
    # 4 CTA-pair tiles would leave most clusters idle: single-CTA tiles 128 wide
    run_case(cuda, 4, 14, 14, 1024, 256, 1, expect="conv_gemm_kernel<128>")


def test_tc_conv_3x3_pad1(cuda):
    run_case(cuda, 2, 14, 14, 256, 256, 3, pad=1, expect="conv_gemm_kernel<128>")


def test_tc_conv_3x3_stride2(cuda):
    run_case(cuda, 2, 28, 28, 128, 128, 3, stride=2, pad=1, expect="conv_gemm_kernel<128>")


def test_tc_conv_partial_tile_and_small_n(cuda):
    run_case(cuda, 3, 7, 7, 512, 64, 3, pad=1, expect="conv_gemm_kernel<64>")  # M = 147, BN = 64


def test_tc_conv_oihw_weights_and_nhwc_output(cuda):
    run_case(cuda, 2, 14, 14, 256, 128, 3, pad=1, ohwi=False, nchw_out=False, expect="conv_gemm_kernel<128>")


def test_tc_conv_nhwc_output_partial_tile(cuda):
    # channels-last f32 result through the staged float4 epilogue; M = 189
    # leaves a partial last tile whose missing rows must not be stored
    run_case(cuda, 3, 7, 9, 64, 64, 1, nchw_out=False, expect="conv_gemm_kernel<64>")
    run_case(cuda, 3, 7, 7, 512, 64, 3, pad=1, nchw_out=False, expect="conv_gemm_kernel<64>")


def test_tc_conv_f16(cuda):
    run_case(cuda, 2, 14, 14, 256, 256, 3, pad=1, dtype=torch.float16, expect="conv_gemm_kernel<128>")


def test_tc_conv_c3_shapes_sampled(cuda):
    """The ResNet-50 stage shapes at batch 256: full-size run, outputs of a
    few images compared against the oracle."""
    g = torch.Generator(device=cuda).manual_seed(3)
    for c, k, pad in ((256, 3, 1), (1024, 1, 0)):
        x = torch.randn(256, 14, 14, c, device=cuda, generator=g).bfloat16()
        w = (torch.randn(256, k, k, c, device=cuda, generator=g) * (2.0 / (c * k * k)) ** 0.5).bfloat16()
        opts = ConvOptions([1, 1], [1, 1], [pad, pad], [pad, pad])
        out = api.conv_low_f32(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2), opts)
        assert api.last_route() == ["conv_gemm_pair_kernel<256,4>"], api.last_route()
        assert api.device_status() == 0
        for img in (0, 37, 131, 200, 255):
            ref = orc.conv(x[img:img + 1].permute(0, 3, 1, 2).float().cpu().numpy(),
                           w.permute(0, 3, 1, 2).float().cpu().numpy(), [1, 1], [1, 1], [pad] * 2, [pad] * 2, 1,
                           nthreads=orc.threads())
            got = out[img:img + 1].cpu().numpy()
            err = float(np.abs(got - ref).max()) / float(np.abs(ref).max())
            assert err <= 1e-4, (c, img, err)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("channels_last_out", [False, True])
def test_tc_conv_low_rounds_in_the_epilogue(cuda, dtype, channels_last_out):
    """conv_low on the tensor-core path rounds the f32 accumulator once in the
    GEMM epilogue: bit-identical to rounding conv_low_f32's result."""
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(2, 14, 14, 256, generator=g).to(dtype).to(cuda).permute(0, 3, 1, 2)
    w = (torch.randn(128, 3, 3, 256, generator=g) * 0.03).to(dtype).to(cuda).permute(0, 3, 1, 2)
    o = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])
    ref = api.cast_to_low(api.conv_low_f32(x, w, o), dtype)
    if channels_last_out:
        store = torch.empty(2, 14, 14, 128, dtype=dtype, device=cuda)
        got = api.conv_low_into(x, w, o, store.permute(0, 3, 1, 2))
    else:
        got = api.conv_low(x, w, o)
    assert api.last_route() == ["conv_gemm_kernel<128>"], api.last_route()  # rounded in the epilogue
    assert api.device_status() == 0
    assert torch.equal(got.contiguous().view(torch.int16).cpu(), ref.contiguous().view(torch.int16).cpu())


def test_patch_conv_low_rounds_in_the_epilogue(cuda):
    g = torch.Generator(device="cpu").manual_seed(12)
    x = torch.randn(2, 3, 32, 32, generator=g).bfloat16().to(cuda)
    w = (torch.randn(128, 3, 16, 16, generator=g) * 0.03).bfloat16().to(cuda)
    o = ConvOptions([16, 16], [1, 1], [0, 0], [0, 0])
    ref = api.cast_to_low(api.conv_low_f32(x, w, o), torch.bfloat16)
    got = api.conv_low(x, w, o)
    assert api.last_route() == ["patches_vec8_kernel", "conv_gemm_kernel<128>"], api.last_route()
    assert torch.equal(got.view(torch.int16).cpu(), ref.view(torch.int16).cpu())
