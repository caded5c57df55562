"""The encoder workload at its configured size (E 768, 12 heads of depth 64,
197 tokens, MLP 3072, 12 layers, batch 64) against the f64 oracle.

Images of a batch never interact, so the GPU runs the whole 64-image batch -
the exact launches the benchmark times - and the oracle recomputes a few of
its images in the same order with the same rounding points.  The four
projection GEMMs are also checked on their own at the full token count, with
the tensor-core instantiation they run asserted through fb_last_route."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ConvOptions
from forma_b200.vit import ViTConfig, ViTEncoder
from oracle import oracle as orc
from tests.test_vit_gpu import gelu_tanh, low, oracle_forward

pytestmark = pytest.mark.gpu

_ONE = ConvOptions([1, 1], [1, 1], [0, 0], [0, 0])
TOKENS = 64 * 197  # GEMM rows of one C5 projection


def _rows(m, count, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(m, size=count, replace=False))


@pytest.mark.parametrize("name,cout,cin", [("qkv", 2304, 768), ("fc1", 3072, 768), ("proj", 768, 768),
                                           ("fc2", 768, 3072)])
def test_c5_projection_gemms_match_oracle(cuda, name, cout, cin):
    """QKV (16-bit output rounded in the epilogue), fc1 (GELU + rounding in the
    epilogue) and the residual projections (f32 read-modify-write epilogue) at
    M = 12608 tokens, on the CTA-pair kernel with twelve epilogue warps and
    192-column tiles; 512 sampled rows against f64 products."""
    g = torch.Generator(device="cpu").manual_seed(cout + cin)
    tok = torch.randn(64, 197, cin, generator=g).bfloat16()
    w = (torch.randn(cout, cin, 1, 1, generator=g) * cin ** -0.5).bfloat16()
    x_in = tok.to(cuda).view(64, 1, 197, cin).permute(0, 3, 1, 2)
    wd = w.to(cuda)
    rows = _rows(TOKENS, 512, cout)
    prod = tok.view(-1, cin).double().numpy()[rows] @ w[:, :, 0, 0].double().numpy().T  # f64 sums, [512, cout]
    if name in ("qkv", "fc1"):
        out = torch.empty(64, 1, 197, cout, dtype=torch.bfloat16, device=cuda)
        fn = api.conv_low_into if name == "qkv" else api.conv_low_gelu_into
        fn(x_in, wd, _ONE, out.permute(0, 3, 1, 2))
        assert api.last_route() == ["conv_gemm_pair_kernel<192,12>"], api.last_route()
        got = out.view(-1, cout).float().cpu().numpy().astype(np.float64)[rows]
        # the oracle rounds the f64 sum (and GELU) once to BF16; the kernel's
        # f32 sum may sit on the other side of a rounding boundary: one BF16
        # step (2^-8 relative) at most
        want = low(prod) if name == "qkv" else low(gelu_tanh(prod))
        tol = np.abs(want) * 2.0 ** -7 + 1e-3 * np.abs(want).max()
        assert (np.abs(got - want) <= tol).all(), float(np.abs(got - want).max())
        assert (got == want).mean() > 0.95
    else:
        base = torch.randn(64, 197, cout, generator=g)
        x = base.to(cuda)
        api.conv_low_f32_accumulate(x_in, wd, _ONE, x.view(64, 1, 197, cout).permute(0, 3, 1, 2))
        assert api.last_route() == ["conv_gemm_pair_kernel<192,12>"], api.last_route()
        got = x.view(-1, cout).cpu().numpy().astype(np.float64)[rows]
        want = base.view(-1, cout).double().numpy()[rows] + prod
        err = float(np.abs(got - want).max()) / float(np.abs(want).max())
        assert err <= 2e-2, err  # parity gate
        assert err <= 1e-5, err  # f32 accumulation of exact bf16 products, one f32 add
    assert api.device_status() == 0


def test_c5_forward_at_configured_size_matches_oracle(cuda):
    """The 64-image, 12-layer forward; images 0 and 63 through the oracle."""
    cfg = ViTConfig()
    assert (cfg.batch, cfg.embed, cfg.heads, cfg.layers, cfg.mlp, cfg.tokens) == (64, 768, 12, 12, 3072, 197)
    enc = ViTEncoder(cfg, cuda, seed=0)
    g = torch.Generator(device="cpu").manual_seed(2)
    img = torch.randn(cfg.batch, cfg.channels, cfg.image, cfg.image, generator=g).bfloat16()
    out = enc.forward(img.to(cuda)).cpu().numpy()
    assert api.device_status() == 0
    assert np.isfinite(out).all()
    picks = [0, cfg.batch - 1]
    ref = oracle_forward(enc, img[picks])
    got = out[picks]
    assert got.shape == ref.shape == (2, cfg.tokens, cfg.embed)
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err <= 2e-2, err  # bf16 tensor-core gate, applied to the chain's output


def test_c5_layer_kernels_are_the_tensor_core_ones(cuda):
    """Every contraction of one encoder forward at batch 64 runs on tcgen05:
    the route of each call (patch gather + GEMM, QKV / fc1 / residual pair
    GEMMs, the short-range attention kernel) recorded through fb_last_route."""
    cfg = ViTConfig()
    enc = ViTEncoder(cfg, cuda, seed=1)
    img = torch.randn(cfg.batch, 3, 224, 224, generator=torch.Generator(device="cpu").manual_seed(3)).bfloat16()
    seen = []
    orig = api._check

    def spy(status):
        orig(status)
        seen.append(tuple(api.last_route()))

    api._check = spy
    try:
        enc.forward(img.to(cuda))
    finally:
        api._check = orig
    assert api.device_status() == 0
    kinds = {r for route in seen for r in route}
    assert "conv_gemm_pair_kernel<192,12>" in kinds  # QKV, fc1, proj, fc2
    assert "attn_short_kernel<2>" in kinds  # 197 keys: two softmax warps per query row
    assert "patches_vec8_kernel" in kinds and "rows_warp_kernel" in kinds
    simt = {"conv_direct_kernel", "attention_simt_kernel", "attention_part_kernel", "gemm_simt_kernel"}
    assert not (kinds & simt), kinds & simt
    assert sum(1 for route in seen if "attn_short_kernel<2>" in route) == cfg.layers
