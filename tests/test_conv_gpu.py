"""Convolution on the GPU versus the oracle: the reference's conformance
cases (exact), bit-identity with the reference kernel's f32 order at the
fp32 workload geometry, and the low-storage cases."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ConvOptions, TensorError
from oracle import oracle as orc
from tests import conformance as cf

pytestmark = pytest.mark.gpu


def options(case):
    return ConvOptions(case.strides, case.dilations, case.padding_before, case.padding_after, case.groups)


def test_conv_conformance_cases_exact(cuda):
    """check_conv_backend (conformance/convolution.rs:246-258): exact equality."""
    for case in cf.conv_cases():
        x = case.input.to_device(torch, cuda)
        w = case.weight.to_device(torch, cuda)
        exp = cf.conv_expected(case)
        out = api.conv(x, w, options(case))
        assert list(out.shape) == list(exp.shape)
        assert np.array_equal(out.cpu().numpy().astype(np.float64), exp)
        # sources unchanged
        assert np.array_equal(x.cpu().numpy(), case.input.logical())


def test_conv_inexact_and_invalid(cuda):
    xs = np.array([(i - 30.0) / 37.0 for i in range(65)], np.float32)
    ws = np.array([((i * 17) % 31) / 23.0 - 0.7 for i in range(65)], np.float32)
    out = api.conv(torch.from_numpy(xs).reshape(1, 1, 65).to(cuda), torch.from_numpy(ws).reshape(1, 1, 65).to(cuda),
                   ConvOptions.new(1)).item()
    exp, absolute = 0.0, 0.0
    for a, b in zip(xs.tolist(), ws.tolist()):
        exp += a * b
        absolute += abs(a * b)
    assert abs(out - exp) <= 2e-5 * absolute
    a = torch.empty(0, 2, 5, device=cuda)
    w = torch.ones(4, 2, 3, device=cuda)
    bad = [ConvOptions.new(0), ConvOptions.new(2), ConvOptions([1], [1], [0], [0], 0), ConvOptions([0], [1], [0], [0]),
           ConvOptions([1], [0], [0], [0]), ConvOptions([1], [1], [0], [0], 3)]
    for o in bad:
        with pytest.raises(TensorError):
            api.conv(a, w, o)
    with pytest.raises(TensorError):
        api.conv(torch.empty(0, 2, device=cuda), w, ConvOptions.new(1))
    with pytest.raises(TensorError):
        api.conv(a, torch.ones(4, 1, 3, device=cuda), ConvOptions.new(1))
    with pytest.raises(TensorError):
        api.conv(a, torch.empty(4, 2, 0, device=cuda), ConvOptions.new(1))


@pytest.mark.parametrize("batch", [1, 2])
def test_conv_f32_bit_identical_to_reference_order(cuda, batch):
    """The fp32 workload's geometry ([N,64,56,56] x [64,64,3,3], stride 1,
    pad 1) with U(-1,1) inputs and N(0, sqrt(2/576)) weights: every output
    bit equals the reference kernel's sequential f32 order."""
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (batch, 64, 56, 56)).astype(np.float32)
    w = (rng.standard_normal((64, 64, 3, 3)) * np.sqrt(2 / 576)).astype(np.float32)
    o = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])
    out = api.conv(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), o).cpu().numpy()
    exp = orc.conv_f32_seq(x, w, [1, 1], [1, 1], [1, 1], [1, 1], 1, nthreads=orc.threads())
    assert out.shape == exp.shape
    assert np.array_equal(out.view(np.uint32), exp.view(np.uint32))
    f64 = orc.conv(x[:1, :, :8], w, [1, 1], [1, 1], [1, 1], [1, 1], 1)
    cf.check(out[:1, :, :6], f64[:, :, :6], tol=1e-5)


def test_conv_f32_strided_and_grouped_bit_identical(cuda):
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (2, 8, 13, 11)).astype(np.float32)
    w = rng.uniform(-1, 1, (12, 4, 3, 2)).astype(np.float32)
    o = ConvOptions([2, 1], [1, 2], [1, 0], [2, 1], 2)
    xt = torch.from_numpy(x).to(cuda).permute(0, 2, 3, 1).contiguous().permute(0, 3, 1, 2)  # channels-last view
    out = api.conv(xt, torch.from_numpy(w).to(cuda), o).cpu().numpy()
    exp = orc.conv_f32_seq(x, w, [2, 1], [1, 2], [1, 0], [2, 1], 2)
    assert np.array_equal(out.view(np.uint32), exp.view(np.uint32))


LOW = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.mark.parametrize("name", ["f16", "bf16"])
def test_low_conv_conformance_cases(cuda, name):
    """check_low_conv_backend (conformance/convolution/low.rs:44-73)."""
    dt = LOW[name]

    def narrow(a):
        return orc.decode_bits(orc.round_bits(a, name), name)

    for case in cf.conv_cases():
        x = case.input.to_device(torch, cuda, dt)
        w = case.weight.to_device(torch, cuda, dt)
        exp = cf.conv_expected(case, narrow)
        out = api.conv_low_f32(x, w, options(case))
        assert list(out.shape) == list(exp.shape)
        assert np.array_equal(out.cpu().numpy().astype(np.float64), exp)
        low = api.conv_low(x, w, options(case))
        assert low.dtype == dt
        want = orc.round_bits(exp.astype(np.float32), name)
        got = low.cpu().view(torch.int16).numpy().view(np.uint16)
        ok = (got == want) | (((got & 0x7FFF) == 0) & ((want & 0x7FFF) == 0))
        assert ok.all()


@pytest.mark.parametrize("name", ["f16", "bf16"])
def test_low_conv_final_rounding_and_tiny_products(cuda, name):
    """final_rounding and tiny_products (conformance/convolution/low.rs:75-160)."""
    dt = LOW[name]
    half = 2.0**-11 if name == "f16" else 2.0**-8
    x = torch.tensor([1.0, half, half, half], dtype=dt, device=cuda).reshape(1, 4, 1)
    w = torch.ones(1, 4, 1, dtype=dt, device=cuda)
    out = api.conv_low_f32(x, w, ConvOptions.new(1)).item()
    assert out == 1.0 + 3 * half
    large = 2048.0 if name == "f16" else 256.0
    x = torch.tensor([large, 1.0, -large], dtype=dt, device=cuda).reshape(1, 1, 3)
    w = torch.ones(1, 1, 3, dtype=dt, device=cuda)
    assert api.conv_low_f32(x, w, ConvOptions.new(1)).item() == 1.0
    last_sub, big, one = (0x03FF, 0x7BFF, 0x3C00) if name == "f16" else (0x007F, 0x7F7F, 0x3F80)
    tiny = np.array([1, last_sub, 0x8001, last_sub | 0x8000, 0, one], np.uint16)
    xt = torch.from_numpy(tiny.view(np.int16)).view(dt).reshape(1, 1, 6).to(cuda)
    wt = torch.from_numpy(np.array([big], np.uint16).view(np.int16)).view(dt).reshape(1, 1, 1).to(cuda)
    exp = orc.decode_bits(tiny, name).astype(np.float64) * float(orc.decode_bits(np.array([big], np.uint16), name)[0])
    assert np.array_equal(api.conv_low_f32(xt, wt, ConvOptions.new(1)).cpu().numpy().reshape(-1).astype(np.float64), exp)
    assert np.array_equal(api.conv_low_f32(wt.expand(1, 1, 1), xt[..., :1], ConvOptions.new(1)).cpu().numpy().reshape(-1),
                          exp[:1].astype(np.float32))


def test_low_conv_dtype_mismatch(cuda):
    a = torch.empty(0, 0, 3, dtype=torch.float16, device=cuda)
    b = torch.empty(0, 0, 1, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(TensorError) as e:
        api.conv_low_f32(a, b, ConvOptions.new(1))
    assert e.value.kind == "LowDtypeMismatch"
