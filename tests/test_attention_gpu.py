"""Attention on the GPU versus the f64 oracle: every case of the reference's
conformance suite for f32 and low (f16/bf16) operands."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions, Mask, TensorError
from oracle import oracle as orc
from tests import conformance as cf

pytestmark = pytest.mark.gpu


def run(case, cuda, dtype=None):
    q = case.q.to_device(torch, cuda, dtype)
    k = case.k.to_device(torch, cuda, dtype)
    v = case.v.to_device(torch, cuda, dtype)
    mask = None
    if case.mask is not None:
        if case.mask_kind == "keep":
            m = cf.Host(case.mask.dims, np.asarray(case.mask.values, np.uint32).view(np.int32), case.mask.permutation)
            mask = Mask("keep", m.to_device(torch, cuda))
        else:
            mask = Mask("additive", case.mask.to_device(torch, cuda))
    opts = AttentionOptions(case.scale, case.causal)
    fn = api.attention if dtype is None else api.attention_low_f32
    return fn(q, k, v, mask, opts)


def test_attention_conformance_suite_f32(cuda):
    """check_attention_backend; tolerance 1e-5 relative with scale
    max(|e|, 1) (tighter than the suite's 3e-4)."""
    for i, case in enumerate(cf.attention_cases()):
        out = run(case, cuda)
        exp = cf.attention_expected(case)
        assert list(out.shape) == list(exp.shape), i
        a = out.cpu().numpy().astype(np.float64)
        assert np.isfinite(a).all(), i
        err = np.abs(a - exp) / np.maximum(np.abs(exp), 1.0)
        assert err.size == 0 or err.max() <= 1e-5, (i, err.max())


@pytest.mark.parametrize("name", ["f16", "bf16"])
def test_attention_conformance_suite_low(cuda, name):
    dt = {"f16": torch.float16, "bf16": torch.bfloat16}[name]

    def narrow(a):
        return orc.decode_bits(orc.round_bits(a, name), name)

    for i, case in enumerate(cf.attention_cases()):
        vals = [case.q.logical(), case.k.logical(), case.v.logical()]
        if any(np.isinf(narrow(x)).any() for x in vals):
            continue  # f32::MAX does not fit the low format (not a low-suite case)
        out = run(case, cuda, dt)
        exp = cf.attention_expected(case, narrow)
        assert list(out.shape) == list(exp.shape), i
        a = out.cpu().numpy().astype(np.float64)
        err = np.abs(a - exp) / np.maximum(np.abs(exp), 1.0)
        assert err.size == 0 or err.max() <= 1e-5, (i, err.max())


def test_attention_invalid(cuda):
    q = torch.ones(3, 4, device=cuda)
    k = torch.ones(7, 4, device=cuda)
    v = torch.ones(7, 5, device=cuda)
    bad = torch.ones(2, 3, 7, dtype=torch.int32, device=cuda)
    with pytest.raises(TensorError):
        api.attention(q, k, v, Mask("keep", bad))
    for s in (float("nan"), float("inf"), float("-inf")):
        with pytest.raises(TensorError):
            api.attention(q, k, v, None, AttentionOptions(scale=s))
    with pytest.raises(TensorError):
        api.attention(torch.tensor(1.0, device=cuda), k, v)
    with pytest.raises(TensorError) as e:
        api.attention_low_f32(q.half(), k.bfloat16(), v.half())
    assert e.value.kind == "LowDtypeMismatch"


def test_attention_cuda_edges(cuda):
    """compute-cuda/tests/cuda_tensor.rs:774-800: 67 keys, depth 35, value depth 263."""
    q = cf.data([2, 5, 35], 1)
    k = cf.data([2, 67, 35], 2)
    v = cf.data([2, 67, 263], 3)
    case = cf.AttnCase(q, k, v, causal=30)
    out = run(case, cuda).cpu().numpy()
    exp = cf.attention_expected(case)
    assert np.abs(out - exp).max() <= 1e-5 * max(1.0, np.abs(exp).max())
