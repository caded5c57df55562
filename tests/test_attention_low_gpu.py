"""attention_low (tensor-core/src/low_attention.rs:38-47): attention_low_f32
rounded once, nearest even, to the operands' 16-bit dtype.  The tensor-core
kernel rounds in its epilogue (and in the key-split merge); the CUDA-core
routes compute f32 rows into scratch and cast them.  Every case must equal
cast_to_low(attention_low_f32(...)) bit for bit, and the f64 oracle at the
16-bit gate."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions, Mask
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def operands(shapes, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [torch.randn(*s, generator=g).to(dtype) for s in shapes]


def check(cuda, q, k, v, mask=None, opts=AttentionOptions(), out_view=None, oracle_mask=None):
    tq, tk, tv = (t.to(cuda) for t in (q, k, v))
    want = api.cast_to_low(api.attention_low_f32(tq, tk, tv, mask, opts), q.dtype)
    if out_view is None:
        got = api.attention_low(tq, tk, tv, mask, opts)
    else:
        got = out_view(tq.shape, q.dtype)
        api.attention_low_into(tq, tk, tv, mask, opts, got)
    assert api.device_status() == 0
    assert got.dtype == q.dtype and got.shape == want.shape
    assert torch.equal(got.contiguous().view(torch.int16), want.view(torch.int16))
    exp = orc.attention(*(t.float().numpy() for t in (q, k, v)), causal=opts.causal, mask=oracle_mask)
    a = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(a - exp).max() / max(np.abs(exp).max(), 1e-30)
    assert err <= 2e-2, err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("depth,causal", [(64, None), (128, 0)])
def test_tensor_core_epilogue_rounding(cuda, dtype, depth, causal):
    q, k, v = operands([(2, 4, 300, depth)] * 3, dtype, depth)
    check(cuda, q, k, v, opts=AttentionOptions(causal=causal))


def test_head_interleaved_output_view(cuda):
    """[B, L, H, D] storage written through a [B, H, L, D] view (the encoder's layout)."""
    q, k, v = operands([(2, 12, 197, 64)] * 3, torch.bfloat16, 3)

    def view(shape, dtype):
        B, H, L, D = shape
        return torch.empty(B, L, H, D, dtype=dtype, device=cuda).permute(0, 2, 1, 3)

    check(cuda, q, k, v, out_view=view)


def test_masks_on_the_tensor_cores(cuda):
    q, k, v = operands([(2, 2, 130, 64)] * 3, torch.bfloat16, 5)
    keep = (np.random.default_rng(6).random((2, 1, 130, 256)) < 0.5).astype(np.int32)
    keep[0, 0, 7] = 0  # a fully masked row: zeros
    k2, v2 = operands([(2, 2, 256, 64)] * 2, torch.bfloat16, 7)
    check(cuda, q, k2, v2, mask=Mask("keep", torch.from_numpy(keep).to(cuda)),
          oracle_mask=np.where(keep > 0, 0.0, -np.inf))


@pytest.mark.parametrize("lq,lk", [(1, 8192), (4, 2048)])
def test_grouped_decode_packed_and_key_split(cuda, lq, lk):
    """GQA 8 query heads over 2 packed into one tile's rows; the key range
    split across CTAs, the merge kernel rounding."""
    q, = operands([(2, 8, lq, 128)], torch.bfloat16, 8)
    k, v = operands([(2, 2, lk, 128)] * 2, torch.bfloat16, 9)
    check(cuda, q, k, v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cuda_core_routes_cast_from_scratch(cuda, dtype):
    """Depth 48 (no tensor-core tiling): split-key decode and the warp-per-row
    kernel write f32 into scratch in the output's memory order, then cast."""
    q, k, v = operands([(1, 4, 3, 48), (1, 2, 1500, 48), (1, 2, 1500, 48)], dtype, 10)
    check(cuda, q, k, v)
    q, k, v = operands([(2, 3, 70, 40), (2, 3, 90, 40), (2, 3, 90, 24)], dtype, 11)

    def view(shape, dt):
        B, H, L, _ = shape
        return torch.empty(B, L, H, 24, dtype=dt, device=cuda).permute(0, 2, 1, 3)

    check(cuda, q, k, v, opts=AttentionOptions(causal=5), out_view=view)


def test_no_keys_gives_zeros(cuda):
    q = torch.randn(1, 2, 3, 64).bfloat16().to(cuda)
    kv = torch.empty(1, 2, 0, 64, dtype=torch.bfloat16, device=cuda)
    got = api.attention_low(q, kv, kv)
    assert api.device_status() == 0
    assert got.dtype == torch.bfloat16 and not got.view(torch.int16).any()
