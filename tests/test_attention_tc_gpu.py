"""The tcgen05 flash-attention path versus the f64 oracle.  Shapes are dense
[B, H, L, D] with D in {64, 128} and no mask tensor, which route to the
tensor-core kernel."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def check(cuda, qs, ks, vs, causal=None, scale=None, dtype=torch.bfloat16, seed=0, vconst=None, expect=None):
    """`expect`: the kernels the call must launch (fb_last_route), tcgen05 first."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(*qs, generator=g).to(dtype)
    k = torch.randn(*ks, generator=g).to(dtype)
    v = torch.randn(*vs, generator=g).to(dtype) if vconst is None else torch.full(vs, vconst).to(dtype)
    before = api.launch_count()
    out = api.attention_low_f32(q.to(cuda), k.to(cuda), v.to(cuda), None, AttentionOptions(scale, causal))
    assert api.last_route() == expect, api.last_route()  # the tensor-core kernel, not a CUDA-core fallback
    out = out.cpu().numpy()
    assert api.device_status() == 0, "a bounded wait timed out"
    assert api.launch_count() > before
    ref = orc.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), None, scale, causal,
                        nthreads=orc.threads())
    assert out.shape == ref.shape
    assert np.isfinite(out).all()
    scale_e = max(float(np.abs(ref).max()), 1e-30)
    err = float(np.abs(out.astype(np.float64) - ref).max()) / scale_e
    assert err <= 2e-2, err  # parity gate for bf16 tensor-core ops
    assert err <= 5e-3, err  # the kernel's own accuracy (bf16 P, f32 accumulate)
    return out, ref


def test_tc_attention_causal_d128(cuda):
    check(cuda, (1, 2, 256, 128), (1, 2, 256, 128), (1, 2, 256, 128), causal=0, expect=["attn_fwd_kernel<128,0,2>"])


def test_tc_attention_ragged_noncausal_d128(cuda):
    check(cuda, (1, 2, 300, 128), (1, 2, 300, 128), (1, 2, 300, 128), expect=["attn_fwd_kernel<128,0,2>"])


def test_tc_attention_vit_shape_d64(cuda):
    # keys fit one TMEM row: one S group over all of them, a single exact-maximum softmax pass
    # (197 keys: two softmax warps per query row, keys 0-127 and 128-196)
    check(cuda, (2, 3, 197, 64), (2, 3, 197, 64), (2, 3, 197, 64), expect=["attn_short_kernel<2>"])


def test_tc_attention_gqa_and_offsets(cuda):
    for causal in (-5, 100, -300):
        out, ref = check(cuda, (1, 4, 256, 64), (1, 2, 256, 64), (1, 2, 256, 64), causal=causal, seed=7,
                         expect=["attn_short_kernel"])
        if causal == -300:
            assert (out == 0).all()  # every row fully masked


def test_tc_attention_f16_and_scale(cuda):
    check(cuda, (1, 2, 256, 128), (1, 2, 384, 128), (1, 2, 384, 128), causal=128, scale=0.05, dtype=torch.float16,
          expect=["attn_fwd_kernel<128,0,2>"])


def test_tc_attention_large_values_do_not_overflow(cuda):
    big = 3.3e38  # near the bf16 maximum: the unnormalised numerator must stay finite
    # one CTA's worth of queries over 32 key tiles: the key range is split across CTAs and merged
    out, ref = check(cuda, (1, 1, 128, 64), (1, 1, 4096, 64), (1, 1, 4096, 64), vconst=big,
                     expect=["attn_fwd_kernel<64,0,2>", "attn_merge_kernel<64>"])
    assert np.isfinite(out).all()


def test_tc_attention_c4_size_sampled(cuda):
    """Causal attention at the workload size [8, 32, 4096, 128]: the full
    tensor is computed, two (batch, head) pairs are compared to the oracle."""
    g = torch.Generator(device=cuda).manual_seed(2)
    q = torch.randn(8, 32, 4096, 128, device=cuda, generator=g).bfloat16()
    k = torch.randn(8, 32, 4096, 128, device=cuda, generator=g).bfloat16()
    v = torch.randn(8, 32, 4096, 128, device=cuda, generator=g).bfloat16()
    out = api.attention_low_f32(q, k, v, None, AttentionOptions(causal=0))
    assert api.last_route() == ["attn_fwd_kernel<128,0,2>"], api.last_route()
    assert api.device_status() == 0
    for b, h in ((0, 0), (7, 31)):
        ref = orc.attention(q[b, h].float().cpu().numpy(), k[b, h].float().cpu().numpy(),
                            v[b, h].float().cpu().numpy(), None, None, 0, nthreads=orc.threads())
        got = out[b, h].cpu().numpy()
        err = float(np.abs(got - ref).max()) / float(np.abs(ref).max())
        assert err <= 5e-3, (b, h, err)


def _check_views(cuda, q, k, v, out=None, causal=None, tol=2e-2):
    """q/k/v (and out) are strided device views; the oracle sees dense copies."""
    before = api.launch_count()
    if out is None:
        got = api.attention_low_f32(q, k, v, None, AttentionOptions(None, causal))
    else:
        got = api.attention_low_f32_into(q, k, v, None, AttentionOptions(None, causal), out)
    route = api.last_route()
    assert len(route) == 1 and (route[0].startswith(f"attn_fwd_kernel<{q.shape[-1]},0,") or
                                route[0].startswith("attn_short_kernel")), route
    assert api.device_status() == 0
    assert api.launch_count() > before
    ref = orc.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), None, None,
                        causal, nthreads=orc.threads())
    g = got.cpu().numpy()
    err = float(np.abs(g.astype(np.float64) - ref).max()) / max(float(np.abs(ref).max()), 1e-30)
    assert err <= tol, err


def test_tc_attention_blhd_views_and_strided_output(cuda):
    # [B, L, H, D] storage viewed as [B, H, L, D], output written in [B, L, H, D] order
    g = torch.Generator(device="cpu").manual_seed(21)
    B, L, H, D = 2, 300, 4, 64
    q, k, v = (torch.randn(B, L, H, D, generator=g).bfloat16().to(cuda).permute(0, 2, 1, 3) for _ in range(3))
    store = torch.empty(B, L, H, D, device=cuda)
    _check_views(cuda, q, k, v, store.permute(0, 2, 1, 3), causal=0)


def test_tc_attention_interleaved_qkv_buffer(cuda):
    # one [B, L, 3, H, D] buffer (a fused QKV projection's output); D = 128
    g = torch.Generator(device="cpu").manual_seed(22)
    B, L, H, D = 2, 256, 2, 128
    qkv = torch.randn(B, L, 3, H, D, generator=g).bfloat16().to(cuda)
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    _check_views(cuda, q, k, v)


def test_tc_attention_broadcast_kv_batch(cuda):
    # K/V shared by every batch index (stride 0), GQA with 2 query heads per K/V head
    g = torch.Generator(device="cpu").manual_seed(23)
    q = torch.randn(3, 4, 192, 64, generator=g).bfloat16().to(cuda)
    k = torch.randn(1, 2, 192, 64, generator=g).bfloat16().to(cuda).expand(3, 2, 192, 64)
    v = torch.randn(1, 2, 192, 64, generator=g).bfloat16().to(cuda).expand(3, 2, 192, 64)
    _check_views(cuda, q, k, v, causal=0)


def _masked_case(cuda, kind, qs, ks, mshape, causal=None, seed=41):
    from forma_b200.api import Mask

    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(*qs, generator=g).bfloat16()
    k = torch.randn(*ks, generator=g).bfloat16()
    v = torch.randn(*ks, generator=g).bfloat16()
    if kind == "keep":
        keep = (torch.rand(*mshape, generator=g) > 0.3).to(torch.int32)
        keep[..., 0, :] = 0  # a fully masked query row -> zeros
        mask = Mask("keep", keep.to(cuda))
        additive = np.where(keep.numpy() != 0, 0.0, -np.inf)
    else:
        add = torch.randn(*mshape, generator=g) * 2
        add[torch.rand(*mshape, generator=g) < 0.2] = float("-inf")
        mask = Mask("additive", add.to(cuda))
        additive = add.numpy().astype(np.float64)
    before = api.launch_count()
    got = api.attention_low_f32(q.to(cuda), k.to(cuda), v.to(cuda), mask, AttentionOptions(None, causal))
    mk = 1 if kind == "keep" else 2
    route = api.last_route()
    assert len(route) == 1 and route[0].startswith(f"attn_fwd_kernel<{qs[-1]},{mk},"), route  # masks on the tensor cores
    got = got.cpu().numpy()
    assert api.device_status() == 0
    assert api.launch_count() > before
    ref = orc.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), additive, None, causal,
                        nthreads=orc.threads())
    assert np.isfinite(got).all()
    err = float(np.abs(got.astype(np.float64) - ref).max()) / max(float(np.abs(ref).max()), 1e-30)
    assert err <= 2e-2, err
    return got, ref


def test_tc_attention_keep_mask_broadcast(cuda):
    # [L, Lk] keep mask broadcast over batch and heads; a fully masked row
    got, ref = _masked_case(cuda, "keep", (2, 3, 256, 64), (2, 3, 320, 64), (256, 320))
    assert np.abs(got[:, :, 0]).max() == 0.0


def test_tc_attention_additive_mask_per_head_causal(cuda):
    # additive mask with -inf entries, per head (broadcast over batch), causal, D = 128
    _masked_case(cuda, "additive", (2, 2, 256, 128), (2, 2, 256, 128), (1, 2, 256, 256), causal=0)


@pytest.mark.parametrize("case", ["ragged_129", "one_key", "full_256", "causal_masked_rows", "f16_negative_scale",
                                  "gqa_packed_decode", "large_values", "split_f16_negative_scale",
                                  "split_177_causal"])
def test_short_key_range_kernel(cuda, case):
    """Key ranges of at most 256 at depth 64 (attn_short_kernel): key counts
    that are not multiples of the MMA step, a single key, a full 256-key row,
    causal offsets that mask whole rows, f16 with a negative scale, grouped
    decode rows packed into one tile (query index = row mod L), and values
    near the BF16 maximum (the numerator's pre-scale).  180 and 200 keys (192 and
    208 score columns) take the two-softmax-warps-per-row instantiation."""
    kw = dict(expect=["attn_short_kernel"])
    if case == "ragged_129":
        check(cuda, (2, 2, 150, 64), (2, 2, 129, 64), (2, 2, 129, 64), **kw)
    elif case == "one_key":
        check(cuda, (1, 2, 70, 64), (1, 2, 1, 64), (1, 2, 1, 64), **kw)
    elif case == "full_256":
        check(cuda, (1, 2, 256, 64), (1, 2, 256, 64), (1, 2, 256, 64), causal=0, **kw)
    elif case == "causal_masked_rows":
        out, ref = check(cuda, (1, 2, 200, 64), (1, 2, 180, 64), (1, 2, 180, 64), causal=-40,
                         expect=["attn_short_kernel<2>"])  # 192 score columns: two warps per row
        assert (out[:, :, :40] == 0).all()  # rows whose visible keys start past the range
    elif case == "f16_negative_scale":
        check(cuda, (1, 3, 100, 64), (1, 3, 222, 64), (1, 3, 222, 64), scale=-0.09, dtype=torch.float16, **kw)
    elif case == "gqa_packed_decode":
        check(cuda, (2, 8, 3, 64), (2, 2, 200, 64), (2, 2, 200, 64), causal=150, expect=["attn_short_kernel<2>"])
    elif case == "split_f16_negative_scale":
        # two softmax warps per row with the row minimum as the logit maximum
        check(cuda, (1, 3, 150, 64), (1, 3, 197, 64), (1, 3, 197, 64), scale=-0.09, dtype=torch.float16,
              expect=["attn_short_kernel<2>"])
    elif case == "split_177_causal":
        # 177 keys: the second warp's last chunk holds one visible key of 16 columns
        check(cuda, (2, 2, 200, 64), (2, 2, 177, 64), (2, 2, 177, 64), causal=-10, expect=["attn_short_kernel<2>"])
    else:
        out, ref = check(cuda, (1, 1, 128, 64), (1, 1, 250, 64), (1, 1, 250, 64), vconst=3.3e38, **kw)
        assert np.isfinite(out).all()
