"""Low-precision GEMM (matmul_low_f32 / matmul_low) against f64 products of
the same 16-bit operands: tensor-core layouts (right row-major or transposed),
broadcast batches, vector promotion, odd shapes on the CUDA-core kernel, and
the one-rounding contract of matmul_low."""

import numpy as np
import pytest
import torch

from forma_b200 import api

pytestmark = pytest.mark.gpu


def f64(t):
    return t.float().cpu().numpy().astype(np.float64)


def check(left, right, tol=2e-2, expect=None):
    """`expect`: the GEMM kernel the call must launch (fb_last_route)."""
    got = api.matmul_low_f32(left, right)
    if expect is not None:
        assert expect in api.last_route(), api.last_route()
    assert api.device_status() == 0
    ref = np.matmul(f64(left), f64(right))
    g = got.cpu().numpy().astype(np.float64)
    assert g.shape == ref.shape
    err = float(np.abs(g - ref).max()) / max(float(np.abs(ref).max()), 1e-30)
    assert err <= tol, err
    # f32 accumulation of exact products: far inside the gate
    assert err <= 1e-4, err
    return got


def rnd(*shape, seed=0, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_matmul_tensor_core_row_major_right(cuda, dtype):
    # N = 192 with a row-major (MN-major) right operand: single-CTA tiles of 64 columns
    check(rnd(300, 256, seed=1, dtype=dtype).to(cuda), rnd(256, 192, seed=2, dtype=dtype).to(cuda),
          expect="conv_gemm_kernel<64>")


def test_matmul_tensor_core_transposed_right(cuda):
    w = rnd(512, 128, seed=3).to(cuda)  # [N, K] storage
    check(rnd(200, 128, seed=4).to(cuda), w.t(), expect="conv_gemm_kernel<128>")


def test_matmul_broadcast_batches(cuda):
    check(rnd(2, 3, 130, 64, seed=5).to(cuda), rnd(3, 64, 128, seed=6).to(cuda), expect="conv_gemm_kernel<128>")
    check(rnd(4, 1, 70, 64, seed=7).to(cuda), rnd(1, 2, 64, 256, seed=8).to(cuda))


def test_matmul_vectors_and_odd_shapes(cuda):
    k = rnd(37, 50, seed=9).to(cuda)
    check(k, rnd(50, 23, seed=10).to(cuda), expect="gemm_simt_kernel")  # CUDA-core kernel
    check(rnd(50, seed=11).to(cuda), rnd(50, 23, seed=12).to(cuda))    # [K] x [K, N] -> [N]
    check(k, rnd(50, seed=13).to(cuda))                # [M, K] x [K] -> [M]
    got = api.matmul_low_f32(rnd(64, seed=14).to(cuda), rnd(64, seed=15).to(cuda))
    assert got.shape == ()
    assert abs(float(got) - float(np.dot(f64(rnd(64, seed=14)), f64(rnd(64, seed=15))))) < 1e-4


def test_matmul_low_rounds_once(cuda):
    for left, right in ((rnd(256, 128, seed=16), rnd(128, 256, seed=17)), (rnd(37, 50, seed=18), rnd(50, 23, seed=19))):
        l, r = left.to(cuda), right.to(cuda)
        got = api.matmul_low(l, r)
        ref = api.cast_to_low(api.matmul_low_f32(l, r), torch.bfloat16)
        assert got.dtype == torch.bfloat16
        assert torch.equal(got.view(torch.int16).cpu(), ref.view(torch.int16).cpu())


def test_matmul_empty_contraction_and_errors(cuda):
    z = api.matmul_low_f32(rnd(3, 0).to(cuda), rnd(0, 4).to(cuda))
    assert z.shape == (3, 4) and float(z.abs().max()) == 0.0
    with pytest.raises(api.TensorError) as e:
        api.matmul_low_f32(rnd(3, 5).to(cuda), rnd(4, 2).to(cuda))
    assert e.value.kind == "MatmulInnerDimension"
    with pytest.raises(api.TensorError) as e:
        api.matmul_low_f32(rnd(3, 4).to(cuda), rnd(4, 2, dtype=torch.float16).to(cuda))
    assert e.value.kind == "InvalidInput"


@pytest.mark.parametrize("M,K,N", [(19200, 512, 256), (19200, 2048, 512), (12608, 768, 768)])
def test_matmul_many_tiles(cuda, M, K, N):
    """More output tiles than persistent CTAs (several per CTA, a partial
    last wave, both TMEM accumulators in turn): results against an f32
    product on the GPU with TF32 off, bit-identical across repeated calls."""
    g = torch.Generator(device=cuda).manual_seed(M + K + N)
    a = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    b = torch.randn(K, N, device=cuda, generator=g).bfloat16()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = a.float() @ b.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    first = api.matmul_low_f32(a, b)
    assert api.last_route()[0].startswith("conv_gemm_pair_kernel<"), api.last_route()  # CTA pairs, many tiles
    assert api.device_status() == 0
    err = float((first - ref).abs().max()) / float(ref.abs().max())
    assert err <= 1e-4, err
    for _ in range(2):
        again = api.matmul_low_f32(a, b)
        assert torch.equal(again, first)
    assert api.device_status() == 0


@pytest.mark.parametrize("offset", [0, 4])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_matmul_low_into_offset_output(cuda, dtype, offset):
    """matmul_low into a dense output starting `offset` elements into its
    buffer: at 4 every row is 8- but not 16-byte aligned, so the CTA-pair
    epilogue takes its 8-byte row stores; the bits equal the fresh result
    and the elements around the view stay untouched."""
    g = torch.Generator(device="cpu").manual_seed(17)
    a = torch.randn(512, 256, generator=g).to(dtype).to(cuda)
    b = torch.randn(256, 768, generator=g).to(dtype).to(cuda)
    want = api.matmul_low(a, b)
    flat = torch.full((512 * 768 + 16,), 7.0, dtype=dtype, device=cuda)
    out = flat[offset:offset + 512 * 768].view(512, 768)
    api.matmul_low(a, b, out=out)
    assert api.device_status() == 0
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    assert bool((flat[:offset] == 7.0).all()) and bool((flat[offset + 512 * 768:] == 7.0).all())
