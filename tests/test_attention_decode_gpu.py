"""Decode-shaped attention (at most 64 query rows per head over at least
512 keys) against the f64 oracle.  f32 operands (and 16-bit ones whose
layout the tensor cores refuse) take the split-key kernels: key ranges of
about 256 computed by separate warps, merged by their maxima and
denominators.  Cases: the decode shape of the reference's attention
benchmark (4 query heads over 2 key/value heads, one query, 4097 keys,
depth 64), causal offsets that leave whole key ranges masked, keep and
additive masks, a fully masked row, 16-bit operands at depth 48 (split) and
64 (tensor cores), and the 64-row boundary of the split."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions, Mask
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def rnd(shape, seed):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def close(got, exp, tol=1e-5):
    a = got.cpu().numpy().astype(np.float64)
    assert a.shape == exp.shape
    err = np.abs(a - exp) / np.maximum(np.abs(exp), 1.0)
    assert err.max() <= tol, err.max()


def low_round(x, name="bf16"):
    return orc.decode_bits(orc.round_bits(x, name), name).astype(np.float32)


def test_decode_benchmark_shape_f32(cuda):
    q, k, v = rnd((1, 4, 1, 64), 1), rnd((1, 2, 4097, 64), 2), rnd((1, 2, 4097, 64), 3)
    got = api.attention(*(torch.from_numpy(t).to(cuda) for t in (q, k, v)), None, AttentionOptions())
    assert api.device_status() == 0
    close(got, orc.attention(q, k, v))


@pytest.mark.parametrize("name,dtype", [("bf16", torch.bfloat16), ("f16", torch.float16)])
@pytest.mark.parametrize("depth", [48, 64])
def test_decode_benchmark_shape_low(cuda, name, dtype, depth):
    shapes = ((2, 4, 3, depth), (2, 2, 4097, depth), (2, 2, 4097, depth))
    q, k, v = (low_round(rnd(s, i), name) for i, s in enumerate(shapes))
    got = api.attention_low_f32(*(torch.from_numpy(t).to(dtype).to(cuda) for t in (q, k, v)), None, AttentionOptions())
    # depth 48: split-key (f64 throughout); depth 64: tensor cores (BF16 P)
    close(got, orc.attention(q, k, v), 1e-5 if depth == 48 else 2e-2)


@pytest.mark.parametrize("offset", [996, 100, -3])
def test_decode_causal_offsets(cuda, offset):
    """Queries at key positions offset..offset+3: with offset 100 most key
    ranges are fully masked (zero weight in the merge); with -3 the first
    three rows see no key at all (zeros)."""
    q, k, v = rnd((1, 2, 4, 32), 4), rnd((1, 2, 1000, 32), 5), rnd((1, 2, 1000, 48), 6)
    got = api.attention(*(torch.from_numpy(t).to(cuda) for t in (q, k, v)), None, AttentionOptions(causal=offset))
    close(got, orc.attention(q, k, v, causal=offset))


def test_decode_masks(cuda):
    q, k, v = rnd((2, 4, 2, 64), 7), rnd((2, 4, 2048, 64), 8), rnd((2, 4, 2048, 64), 9)
    keep = (np.random.default_rng(10).random((2, 1, 2, 2048)) < 0.3).astype(np.int32)
    keep[1, 0, 0, :] = 0  # a fully masked row: zeros
    add = np.where(keep > 0, 0.0, -np.inf)
    tq, tk, tv = (torch.from_numpy(t).to(cuda) for t in (q, k, v))
    got = api.attention(tq, tk, tv, Mask("keep", torch.from_numpy(keep).to(cuda)), AttentionOptions())
    close(got, orc.attention(q, k, v, mask=add))
    assert float(got[1, :, 0].abs().max()) == 0.0
    bias = (rnd((1, 4, 2, 2048), 11) * 3.0).astype(np.float32)
    bias[0, 1, 1, 500:1500] = -np.inf
    got = api.attention(tq, tk, tv, Mask("additive", torch.from_numpy(bias).to(cuda)), AttentionOptions())
    close(got, orc.attention(q, k, v, mask=bias.astype(np.float64)))


@pytest.mark.parametrize("lq", [64, 65])
def test_decode_row_boundary(cuda, lq):
    """64 query rows per head still split; 65 take the one-warp-per-row
    kernel; both f64 throughout."""
    q, k, v = rnd((1, 8, lq, 40), 20), rnd((1, 2, 512, 40), 21), rnd((1, 2, 512, 40), 22)
    got = api.attention(*(torch.from_numpy(t).to(cuda) for t in (q, k, v)), None, AttentionOptions())
    close(got, orc.attention(q, k, v))


@pytest.mark.parametrize("lq,lk,causal,depth", [(1, 8192, None, 128), (4, 4100, 4096, 128), (3, 2048, None, 64),
                                                (16, 3000, 2990, 64)])
def test_decode_tensor_core_key_split(cuda, lq, lk, causal, depth):
    """16-bit decode on the tensor cores with the key range split across CTAs
    (few query blocks over many key tiles) and the ranges merged on the
    device: GQA 8 query heads over 2, causal offsets that leave the last
    ranges partly or wholly masked; against the f64 oracle at the BF16 gate
    and at the kernel's own accuracy."""
    shapes = ((2, 8, lq, depth), (2, 2, lk, depth), (2, 2, lk, depth))
    q, k, v = (low_round(rnd(s, 30 + i)) for i, s in enumerate(shapes))
    opts = AttentionOptions(causal=causal)
    got = api.attention_low_f32(*(torch.from_numpy(t).to(torch.bfloat16).to(cuda) for t in (q, k, v)), None, opts)
    assert api.device_status() == 0
    exp = orc.attention(q, k, v, causal=causal)
    a = got.cpu().numpy().astype(np.float64)
    err = np.abs(a - exp).max() / max(np.abs(exp).max(), 1e-30)
    assert err <= 2e-2, err
    assert err <= 3e-3, err  # BF16 P, f32 accumulation and merge


def _decode16(cuda, qs, ks, causal=None, dtype=torch.bfloat16, seed=40, out_low=False):
    # 16-bit inputs (nearest-even conversion); the oracle sees their exact values
    lows = [torch.from_numpy(rnd(s, seed + i)).to(dtype) for i, s in enumerate((qs, ks, ks))]
    q, k, v = (t.float().numpy() for t in lows)
    tq, tk, tv = (t.to(cuda) for t in lows)
    opts = AttentionOptions(causal=causal)
    got = api.attention_low(tq, tk, tv, None, opts) if out_low else api.attention_low_f32(tq, tk, tv, None, opts)
    route = api.last_route()
    assert api.device_status() == 0
    exp = orc.attention(q, k, v, causal=causal, nthreads=orc.threads())
    a = got.float().cpu().numpy().astype(np.float64)
    err = np.abs(a - exp).max() / max(np.abs(exp).max(), 1e-30)
    assert err <= 2e-2, err  # bf16 tensor-core gate
    assert err <= (8e-3 if out_low else 3e-3), err  # the kernel's own accuracy (16-bit P, f32 accumulation)
    return route


@pytest.mark.parametrize("case", ["bench_gqa", "bench_gqa_one_batch", "rows16_causal", "d64_mha_f16", "low_out"])
def test_decode16_kernel_routes(cuda, case):
    """16-bit decode with at most 16 query rows per key/value head runs on
    attn_decode16_kernel: 40 (batch, key/value head) units of the bench's
    GQA group (each unit's seven key ranges one cluster merging in shared
    memory: one launch), a single batch (more than eight ranges: records
    merged by attn_merge_kernel), 16 rows per head with causal offsets,
    depth 64 with f16 and one head per group, and a 16-bit output rounded
    in the cluster merge."""
    dec128 = ["attn_decode16_kernel<128,1>"]
    if case == "bench_gqa":
        assert _decode16(cuda, (5, 32, 1, 128), (5, 8, 4096, 128)) == dec128
    elif case == "bench_gqa_one_batch":
        route = _decode16(cuda, (1, 32, 1, 128), (1, 8, 8192, 128))
        assert route == dec128 + ["attn_merge_kernel<128>"], route
    elif case == "rows16_causal":
        assert _decode16(cuda, (2, 8, 4, 128), (2, 2, 4100, 128), causal=4096)[0] == dec128[0]
    elif case == "d64_mha_f16":
        assert _decode16(cuda, (2, 4, 2, 64), (2, 4, 3000, 64), dtype=torch.float16)[0] == "attn_decode16_kernel<64,0>"
    else:
        assert _decode16(cuda, (5, 32, 1, 128), (5, 8, 4096, 128), out_low=True) == dec128
