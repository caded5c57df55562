"""The encoder chain (patch conv -> layer norm -> attention -> projections ->
GELU MLP, residual additions) against the oracle composed in the same order
with the same low-precision rounding points, plus the pieces the chain adds:
the space-to-depth patch convolution route and the elementwise glue."""

import math

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ConvOptions
from forma_b200.vit import ViTConfig, ViTEncoder
from oracle import oracle as orc
from oracle import vit as ovit
from oracle.vit import f32, gelu_tanh, low  # noqa: F401  (the chain's rounding points; other tests import them here)

pytestmark = pytest.mark.gpu


def oracle_forward(enc: ViTEncoder, img: torch.Tensor) -> np.ndarray:
    """The oracle composition (oracle/vit.py) on the encoder's weights."""
    cfg = enc.cfg
    w = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    blocks = [{k: w(blk[k]) for k in ("qkv", "proj", "fc1", "fc2")} for blk in enc.blocks]
    return ovit.forward(w(img), w(enc.w_patch), w(enc.pos), w(enc.cls), blocks, cfg.heads, cfg.patch, cfg.eps,
                        nthreads=orc.threads())


def test_vit_chain_small_matches_oracle(cuda):
    cfg = ViTConfig(batch=8, image=64, channels=3, patch=16, embed=128, heads=2, layers=2, mlp=256)
    enc = ViTEncoder(cfg, cuda, seed=3)
    g = torch.Generator(device="cpu").manual_seed(4)
    img = torch.randn(cfg.batch, cfg.channels, cfg.image, cfg.image, generator=g).bfloat16()
    before = api.launch_count()
    out = enc.forward(img.to(cuda)).cpu().numpy()
    assert api.device_status() == 0
    assert api.launch_count() > before
    ref = oracle_forward(enc, img)
    assert out.shape == ref.shape == (cfg.batch, cfg.tokens, cfg.embed)
    assert np.isfinite(out).all()
    err = float(np.abs(out - ref).max() / np.abs(ref).max())
    assert err <= 2e-2, err  # bf16 tensor-core gate, applied to the chain's output


def test_vit_flop_count_matches_configuration():
    f = ViTConfig().flops()
    assert f["patch"] == 14_797_504_512                  # 2 * 64 * 196 * 768 * 768
    assert f["attention"] == 12 * 7_630_159_872          # 4 * B * H * L^2 * D per layer


@pytest.mark.parametrize("contiguous_weights", [True, False])
def test_patch_convolution_route(cuda, contiguous_weights):
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(4, 3, 64, 64, generator=g).bfloat16()
    w = (torch.randn(256, 3, 16, 16, generator=g) / math.sqrt(768)).bfloat16()
    wd = w.to(cuda)
    if not contiguous_weights:
        wd = wd.permute(0, 2, 3, 1).contiguous().permute(0, 3, 1, 2)  # OHWI storage, OIHW view
    out = api.conv_low_f32(x.to(cuda), wd, ConvOptions([16, 16], [1, 1], [0, 0], [0, 0])).cpu().numpy()
    ref = orc.conv(x.float().numpy(), w.float().numpy(), [16, 16], [1, 1], [0, 0], [0, 0])
    err = float(np.abs(out - ref).max() / np.abs(ref).max())
    assert err <= 2e-2, err
    # f32 accumulation of exactly representable products: far tighter than the gate
    assert err <= 1e-4, err
    # channels-last storage (width stride 3): the element-wise gather, same GEMM, same bits
    xl = x.to(cuda).permute(0, 2, 3, 1).contiguous().permute(0, 3, 1, 2)
    out_l = api.conv_low_f32(xl, wd, ConvOptions([16, 16], [1, 1], [0, 0], [0, 0])).cpu().numpy()
    assert np.array_equal(out_l.view(np.uint32), out.view(np.uint32))


def test_add_broadcast_and_strided_output(cuda):
    g = torch.Generator(device="cpu").manual_seed(6)
    a = torch.randn(3, 5, 7, generator=g)
    bias = torch.randn(1, 5, 7, generator=g)
    big = torch.zeros(3, 6, 7, device=cuda)
    api.add(a.to(cuda), bias.to(cuda).expand(3, 5, 7), out=big[:, 1:])
    got = big.cpu().numpy()
    exp = (a.numpy() + bias.numpy()).astype(np.float32)
    assert np.array_equal(got[:, 1:].view(np.uint32), exp.view(np.uint32))  # one f32 add, bit-exact
    assert (got[:, 0] == 0).all()
    # in place on the identical view
    x = a.to(cuda).contiguous()
    api.add(x, x, out=x)
    assert np.array_equal(x.cpu().numpy(), (a.numpy() * 2).astype(np.float32))
    with pytest.raises(api.TensorError):
        api.add(big[:, :5], big[:, 1:], out=big[:, 1:])  # overlapping, not identical


@pytest.mark.parametrize("inner", [16, 768])
def test_add_four_wide_runs_over_strided_views(cuda, inner):
    """Views whose innermost axis is contiguous (a multiple of four): the
    encoder's [cls; patches] + pos (offset output rows, a batch-broadcast
    operand) and a permuted operand; one f32 add, bit-exact."""
    g = torch.Generator(device="cpu").manual_seed(inner)
    a = torch.randn(9, 4, inner, generator=g)
    pos = torch.randn(1, 10, inner, generator=g)
    big = torch.zeros(4, 10, inner, device=cuda)
    api.add(a.to(cuda).permute(1, 0, 2), pos.to(cuda)[:, 1:].expand(4, 9, inner), out=big[:, 1:])
    got = big.cpu().numpy()
    exp = (a.permute(1, 0, 2).numpy() + pos[:, 1:].numpy()).astype(np.float32)
    assert np.array_equal(got[:, 1:].view(np.uint32), exp.view(np.uint32))
    assert (got[:, 0] == 0).all()


def test_gelu_to_low_matches_tanh_form(cuda):
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(4096, generator=g) * 4
    got = api.gelu_to_low(x.to(cuda), torch.bfloat16).float().cpu().numpy().astype(np.float64)
    exp = low(gelu_tanh(x.numpy().astype(np.float64)))
    # f32 evaluation can move a value across a BF16 rounding boundary: one BF16
    # step at most; below 1e-6 in magnitude the f64 form itself has no
    # relative accuracy left (1 + tanh cancels), so compare absolutely there.
    tol = np.abs(exp) * 2.0 ** -7 + 1e-6  # a BF16 step is at most 2^-7 of the value
    assert (np.abs(got - exp) <= tol).all()
    # where the f64 form keeps its precision (|GELU| above 1e-4), the BF16
    # results agree bit for bit except for rare rounding-boundary cases
    m = np.abs(exp) > 1e-4
    assert (got[m] == exp[m]).mean() > 0.99


@pytest.mark.parametrize("inner", [64, 13])
def test_cast_to_low_strided_views(cuda, inner):
    """Head-split views (innermost axis contiguous: 8-element vector path when
    its length allows, element path otherwise), nearest-even BF16."""
    g = torch.Generator(device="cpu").manual_seed(8)
    x = torch.randn(2, 5, 3, 4, inner, generator=g)
    view = x.to(cuda)[:, :, 1].permute(0, 2, 1, 3)  # [2, 4, 5, inner], strides not dense
    got = api.cast_to_low(view, torch.bfloat16).float().cpu().numpy()
    exp = low(x[:, :, 1].permute(0, 2, 1, 3).numpy())
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("cout,cin,tokens", [(768, 768, 197 * 4), (128, 256, 300), (40, 24, 50)])
def test_fused_projection_epilogues_match_the_unfused_chain(cuda, cout, cin, tokens):
    """conv_low_gelu == gelu_to_low(conv_low_f32) and conv_low_f32_accumulate
    == add(x, conv_low_f32), bit for bit: CTA-pair tiles (768), single-CTA
    tiles (128) and the scratch route the tensor cores refuse (40 x 24)."""
    g = torch.Generator(device="cpu").manual_seed(cout + cin)
    tok = torch.randn(2, tokens, cin, generator=g).bfloat16().to(cuda)
    w = (torch.randn(cout, cin, 1, 1, generator=g) * cin ** -0.5).bfloat16().to(cuda)
    xin = tok.view(2, 1, tokens, cin).permute(0, 3, 1, 2)
    one = ConvOptions([1, 1], [1, 1], [0, 0], [0, 0])
    ref32 = torch.empty(2, 1, tokens, cout, device=cuda)
    api.conv_low_f32_into(xin, w, one, ref32.permute(0, 3, 1, 2))
    # GELU + rounding in the epilogue
    ref_low = api.gelu_to_low(ref32, torch.bfloat16)
    got_low = torch.empty(2, 1, tokens, cout, dtype=torch.bfloat16, device=cuda)
    api.conv_low_gelu_into(xin, w, one, got_low.permute(0, 3, 1, 2))
    assert api.device_status() == 0
    assert torch.equal(got_low.view(torch.int16), ref_low.view(torch.int16))
    # residual accumulation in the epilogue
    x0 = torch.randn(2, tokens, cout, generator=g).to(cuda)
    want = api.add(x0, ref32.view(2, tokens, cout))
    x = x0.clone()
    api.conv_low_f32_accumulate(xin, w, one, x.view(2, 1, tokens, cout).permute(0, 3, 1, 2))
    assert api.device_status() == 0
    assert torch.equal(x, want)
