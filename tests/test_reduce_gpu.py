"""Reductions, argmax, statistics and the global sum on the GPU versus the
oracle (the reference's conformance suites, restated), plus size-independent
checks at the row-reduction workload's full size."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import ReduceOp, TensorError
from oracle import oracle as orc
from tests import conformance as cf

pytestmark = pytest.mark.gpu
OPS = [ReduceOp.Sum, ReduceOp.Product, ReduceOp.Min, ReduceOp.Max]


def u32(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint32)


def test_reduce_conformance_suite(cuda):
    """check_reduce_backend (conformance/reduction.rs:83-143)."""
    floats = cf.reduce_float_values()
    ints = cf.reduce_uint_values()
    inp = torch.from_numpy(floats).reshape(2, 3, 5).to(cuda).permute(1, 0, 2)
    uint = torch.from_numpy(ints.view(np.int32)).reshape(2, 3, 5).to(cuda).permute(1, 0, 2)
    fl = np.transpose(floats.reshape(2, 3, 5), (1, 0, 2))
    ul = np.transpose(ints.reshape(2, 3, 5), (1, 0, 2))
    for axes in cf.axis_masks():
        for keep in (False, True):
            out_dims = [1 if a in axes else d for a, d in enumerate([3, 2, 5]) if keep or a not in axes]
            for op in OPS:
                out = api.reduce_f32(op, inp, axes, keep)
                assert list(out.shape) == out_dims
                cf.check(out.cpu().numpy(), cf_reduce(fl, axes, op))
                out = api.reduce_u32(op, uint, axes, keep)
                assert list(out.shape) == out_dims
                assert (u32(out).reshape(-1) == orc.reduce_u32(ul, axes, int(op)).reshape(-1)).all()
            count = int(np.prod([[3, 2, 5][a] for a in axes])) if axes else 1
            mean = api.mean_axes(inp, axes, keep)
            assert list(mean.shape) == out_dims
            cf.check(mean.cpu().numpy(), orc.reduce_f32(fl, axes, 0) / np.float32(count))


def cf_reduce(x, axes, op):
    return orc.reduce_f32(x, axes, int(op))


def test_reduce_edge_cases(cuda):
    """conformance/reduction.rs:145-253."""
    fmax = cf.F32_MAX
    for op, values, want in ((ReduceOp.Min, [fmax, fmax / 2], fmax / 2), (ReduceOp.Max, [-fmax, -fmax / 2], -fmax / 2)):
        v = torch.tensor(values, dtype=torch.float32, device=cuda)
        cf.check(api.reduce_f32(op, v, [0]).cpu().numpy(), [np.float32(want)])
    for dims in ([2, 0, 3], [0, 0, 3]):
        f = torch.empty(dims, dtype=torch.float32, device=cuda)
        u = torch.empty(dims, dtype=torch.int32, device=cuda)
        for keep in (False, True):
            for op in OPS:
                if dims[0] != 0 and op in (ReduceOp.Min, ReduceOp.Max):
                    with pytest.raises(TensorError):
                        api.reduce_f32(op, f, [1], keep)
                    with pytest.raises(TensorError):
                        api.reduce_u32(op, u, [1], keep)
                else:
                    rf = api.reduce_f32(op, f, [1], keep)
                    ru = api.reduce_u32(op, u, [1], keep)
                    out = [dims[0], 1, 3] if keep else [dims[0], 3]
                    assert list(rf.shape) == out and list(ru.shape) == out
                    ident = 1 if op == ReduceOp.Product else 0
                    assert (rf.cpu().numpy() == ident).all() and (u32(ru) == ident).all()
            if dims[0] != 0:
                with pytest.raises(TensorError):
                    api.mean_axes(f, [1], keep)
            else:
                assert api.mean_axes(f, [1], keep).numel() == 0
        for op in OPS:
            assert api.reduce_f32(op, f, []).numel() == 0
            assert api.reduce_u32(op, u, []).numel() == 0
    scalar = torch.tensor(1.25, device=cuda)
    uscalar = torch.tensor(np.array(0xFFFFFFFF, np.uint32).view(np.int32), device=cuda)
    for op in OPS:
        r = api.reduce_f32(op, scalar, [])
        assert r.shape == () and r.item() == 1.25
        assert u32(api.reduce_u32(op, uscalar, [], True)).tolist() == 0xFFFFFFFF
    exp = scalar.expand(3, 2, 5)
    cf.check(api.mean_axes(exp, [0, 2], True).cpu().numpy(), [1.25, 1.25])
    cf.check(api.reduce_f32(ReduceOp.Product, exp, [1]).cpu().numpy(), [1.5625] * 15)
    uexp = uscalar.expand(2, 3)
    assert u32(api.reduce_u32(ReduceOp.Sum, uexp, [1])).tolist() == [0xFFFFFFFD] * 2
    n = 131077
    values = np.ones(n, np.float32)
    values[17] = -1.0
    values[n - 1] = 2.0
    uints = np.ones(n, np.uint32)
    uints[0] = 0xFFFFFFFF
    uints[n - 1] = 3
    f = torch.from_numpy(values).to(cuda)
    u = torch.from_numpy(uints.view(np.int32)).to(cuda)
    for op in OPS:
        cf.check(api.reduce_f32(op, f, [0]).cpu().numpy(), orc.reduce_f32(values, [0], int(op)))
        assert u32(api.reduce_u32(op, u, [0])).reshape(-1).tolist() == orc.reduce_u32(uints, [0], int(op)).reshape(-1).tolist()
    cf.check(api.mean_axes(f, [0]).cpu().numpy(), [np.float32(n - 1) / np.float32(n)])
    floats = cf.reduce_float_values()
    inp = torch.from_numpy(floats).reshape(2, 3, 5).to(cuda).permute(1, 0, 2)
    first = api.reduce_f32(ReduceOp.Product, inp, [2])
    last = api.mean_axes(first, [1, 0])
    prods = orc.reduce_f32(np.transpose(floats.reshape(2, 3, 5), (1, 0, 2)), [2], 1)
    cf.check(last.cpu().numpy(), [np.float32(prods.astype(np.float64).sum()) / np.float32(6)])
    with pytest.raises(TensorError):
        api.reduce_f32(ReduceOp.Sum, inp, [0, 0])
    with pytest.raises(TensorError):
        api.reduce_u32(ReduceOp.Min, u.reshape(1, n), [3], True)


def _rows(n_rows, cols, seed=1):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n_rows, cols)).astype(np.float32)


@pytest.mark.parametrize("cols", [4096, 768, 1000, 131077 // 7, 1])
def test_row_reductions_vs_oracle(cuda, cols):
    """The row-reduction workload's ops (sum, max, argmax, mean) on a slice."""
    x = _rows(384, cols)
    t = torch.from_numpy(x).to(cuda)
    cf.check(api.reduce_f32(ReduceOp.Sum, t, [1]).cpu().numpy(), orc.row_reduce(x, 0), tol=1e-5)
    assert (api.reduce_f32(ReduceOp.Max, t, [1]).cpu().numpy() == orc.row_reduce(x, 3)).all()
    assert (api.reduce_f32(ReduceOp.Min, t, [1]).cpu().numpy() == orc.row_reduce(x, 2)).all()
    assert (u32(api.argmax(t, 1)) == orc.argmax_rows(x)).all()
    cf.check(api.mean_axes(t, [1]).cpu().numpy(), orc.row_reduce(x, 0) / np.float32(cols), tol=1e-5)


def test_argmax_ties_signed_zero_and_strided(cuda):
    x = np.array([[0.0, -0.0, 0.0, 0.0], [-0.0, 0.0, -1.0, 0.0], [3.0, 3.0, 3.0, 3.0], [-np.inf, -5.0, -5.0, -6.0]],
                 np.float32)
    t = torch.from_numpy(x).to(cuda)
    assert u32(api.argmax(t, 1)).tolist() == [0, 1, 0, 1]
    assert u32(api.argmax(t.t(), 0)).tolist() == [0, 1, 0, 1]  # strided rows
    assert u32(api.argmax(t, 1, keep_dims=True)).reshape(-1).tolist() == [0, 1, 0, 1]
    assert u32(api.argmax(t, 0)).tolist() == orc.argmax_rows(x.T.copy()).tolist()
    big = np.zeros((3, 50000), np.float32)
    big[:, 49999] = 1.0
    big[1, 7] = 1.0
    assert u32(api.argmax(torch.from_numpy(big).to(cuda), 1)).tolist() == [49999, 7, 49999]


def _stats_check(cuda, t, values, axes, eps):
    exp = orc.stats(values, axes, eps)
    sm = api.softmax(t, axes)
    lsm = api.log_softmax(t, axes)
    ln = api.layer_norm(t, axes, eps)
    for r in (sm, lsm, ln):
        assert list(r.shape) == list(t.shape)
    cf.close("softmax", sm.cpu().numpy(), exp["softmax"], cf.STATS_TOL["softmax"])
    cf.close("log_softmax", lsm.cpu().numpy(), exp["log_softmax"], cf.STATS_TOL["log_softmax"])
    cf.close("layer_norm", ln.cpu().numpy(), exp["norm"], cf.STATS_TOL["norm"])
    for keep in (False, True):
        lse = api.logsumexp(t, axes, keep)
        m = api.moments(t, axes, keep)
        shape = [1 if a in axes else d for a, d in enumerate(t.shape) if keep or a not in axes]
        assert list(lse.shape) == shape and list(m.mean.shape) == shape and list(m.variance.shape) == shape
        cf.close("logsumexp", lse.cpu().numpy(), exp["logsumexp"], cf.STATS_TOL["logsumexp"])
        cf.close("mean", m.mean.cpu().numpy(), exp["mean"], cf.STATS_TOL["mean"])
        cf.close("population variance", m.variance.cpu().numpy(), exp["variance"], cf.STATS_TOL["variance"])


def test_statistics_conformance_suite(cuda):
    """check_stats_backend (conformance/statistics.rs:387-483)."""
    values = cf.stats_values()
    t = torch.from_numpy(values).reshape(2, 3, 5).to(cuda)
    for axes in ([], [0], [2], [2, 0], [0, 1, 2]):
        _stats_check(cuda, t, values.reshape(2, 3, 5), axes, 1e-5)
    tr = t.permute(2, 0, 1)
    _stats_check(cuda, tr, np.ascontiguousarray(np.transpose(values.reshape(2, 3, 5), (2, 0, 1))), [2, 0], 0.125)
    b = torch.tensor([[2.0], [-3.0]], device=cuda).expand(4, 2, 9)
    _stats_check(cuda, b, np.broadcast_to(np.array([[2.0], [-3.0]], np.float32), (4, 2, 9)).copy(), [0, 2], 1e-5)
    s = torch.tensor(42.0, device=cuda)
    _stats_check(cuda, s, np.array(42.0, np.float32), [], 1e-5)
    for row in cf.huge_offset_rows():
        _stats_check(cuda, torch.from_numpy(row).to(cuda), row, [0], 1e-5)
    for eps in (np.array([1], np.uint32).view(np.float32)[0], 1e-40, 1e-5, cf.F32_MAX):
        vals = np.array([-1e-20, 1e-20, -2e-20, 2e-20], np.float32)
        _stats_check(cuda, torch.from_numpy(vals).to(cuda), vals, [0], float(eps))
    big = np.array([((i * 17) % 127) / 8.0 - 7.0 for i in range(131077)], np.float32)
    _stats_check(cuda, torch.from_numpy(big).to(cuda), big, [0], 0.01)
    empty = torch.empty(2, 0, 3, device=cuda)
    for axes in ([], [0], [1], [0, 1, 2]):
        for r in (api.softmax(empty, axes), api.log_softmax(empty, axes), api.layer_norm(empty, axes, 1e-5)):
            assert list(r.shape) == [2, 0, 3] and r.numel() == 0
    for keep in (False, True):
        for axes in ([], [0]):
            assert api.logsumexp(empty, axes, keep).numel() == 0
            m = api.moments(empty, axes, keep)
            assert m.mean.numel() == 0 and m.variance.numel() == 0
        with pytest.raises(TensorError):
            api.logsumexp(empty, [1], keep)
        with pytest.raises(TensorError):
            api.moments(empty, [1], keep)
    for axes in ([3], [1, 1]):
        for fn in (api.softmax, api.log_softmax):
            with pytest.raises(TensorError):
                fn(t, axes)
        with pytest.raises(TensorError):
            api.logsumexp(t, axes)
        with pytest.raises(TensorError):
            api.moments(t, axes)
        with pytest.raises(TensorError):
            api.layer_norm(t, axes, 1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_statistics(cuda, dtype):
    """TensorLowStatsBackend *_low_f32: low loads, f32 results
    (conformance/low_statistics.rs)."""
    x = _rows(64, 768, seed=3)
    low = torch.from_numpy(x).to(dtype)
    xd = low.float().numpy()
    t = low.to(cuda)
    exp = orc.row_stats(xd, 1e-5)
    cf.close("softmax", api.softmax(t, [1]).cpu().numpy(), exp["softmax"], 4e-5)
    cf.close("layer_norm", api.layer_norm(t, [1], 1e-5).cpu().numpy(), exp["norm"], 2e-4)
    m = api.moments(t, [1])
    cf.close("mean", m.mean.cpu().numpy(), exp["mean"], 2e-5)
    cf.close("population variance", m.variance.cpu().numpy(), exp["variance"], 2e-4)
    cf.close("logsumexp", api.logsumexp(t, [1]).cpu().numpy(), exp["logsumexp"], 5e-5)
    # singleton groups preserve the widened input exactly, including -0
    z = torch.tensor([[-0.0, 1e-40, 3.0]], dtype=dtype, device=cuda)
    assert np.array_equal(api.logsumexp(z, [0]).cpu().numpy().view(np.uint32),
                          z.float().cpu().numpy().reshape(-1).view(np.uint32))


@pytest.mark.parametrize("cols", [4096, 768])
def test_row_statistics_vs_oracle(cuda, cols):
    """Row softmax / log-softmax / layer norm / moments at the workload's
    row length, 1e-5 relative (scale max(|e|, 1) as conformance.rs:38-46)."""
    x = _rows(256, cols, seed=5)
    t = torch.from_numpy(x).to(cuda)
    exp = orc.row_stats(x, 1e-5)
    sm = api.softmax(t, [1]).cpu().numpy()
    rel = np.abs(sm.astype(np.float64) - exp["softmax"]) / np.maximum(np.abs(exp["softmax"]), 1e-30)
    assert rel.max() <= 1e-5
    cf.check(api.log_softmax(t, [1]).cpu().numpy(), exp["log_softmax"], tol=1e-5)
    cf.check(api.layer_norm(t, [1], 1e-5).cpu().numpy(), exp["norm"], tol=1e-5)
    m = api.moments(t, [1])
    cf.check(m.mean.cpu().numpy(), exp["mean"], tol=1e-5)
    cf.check(m.variance.cpu().numpy(), exp["variance"], tol=1e-5)
    cf.check(api.logsumexp(t, [1]).cpu().numpy(), exp["logsumexp"], tol=1e-5)


def test_global_sum(cuda):
    x = _rows(4096, 1000, seed=9)
    t = torch.from_numpy(x).to(cuda)
    want = orc.sum_f64(x)
    assert abs(api.global_sum(t).item() - np.float32(want)) <= 1e-5 * max(abs(want), 1.0)
    assert abs(api.sum_partial_f64(t).item() - want) <= 1e-9 * max(abs(want), 1.0)
    # all-axes reduce_f32 takes the same route
    cf.check(api.reduce_f32(ReduceOp.Sum, t, [0, 1]).cpu().numpy(), [np.float32(want)], tol=1e-5)
    # strided input and repeated calls (the finishing counter re-arms)
    for _ in range(3):
        got = api.sum_partial_f64(t.t()).item()
        assert abs(got - want) <= 1e-9 * max(abs(want), 1.0)
    # streamed chunks with a ragged tail, a 16-byte-misaligned view (plain
    # loads), alternating so that both kernels share the re-armed counter
    flat = _rows(1, 4096 * 300 + 123, seed=10)[0]
    ft = torch.from_numpy(flat).to(cuda)
    for view in (ft, ft[1:], ft, ft[3:], ft):
        want = orc.sum_f64(view.cpu().numpy())
        got = api.sum_partial_f64(view).item()
        assert abs(got - want) <= 1e-9 * max(abs(want), 1.0)
    assert api.device_status() == 0


def test_full_size_row_workload_properties(cuda):
    """X [65536, 4096] ~ N(0,1): size-independent checks at full size."""
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(65536, 4096, device=cuda, generator=g)
    mx = api.reduce_f32(ReduceOp.Max, x, [1])
    idx = api.argmax(x, 1).long()
    rows = torch.arange(65536, device=cuda)
    assert torch.equal(x[rows, idx], mx)
    # no earlier column attains the maximum (lowest index on ties)
    earlier = (x == mx[:, None]) & (torch.arange(4096, device=cuda)[None, :] < idx[:, None])
    assert not earlier.any()
    sm = api.softmax(x, [1])
    assert torch.allclose(sm.double().sum(1), torch.ones(65536, dtype=torch.float64, device=cuda), atol=1e-5)
    m = api.moments(x, [1])
    ln = api.layer_norm(x, [1], 1e-5)
    assert torch.allclose(ln.double().mean(1), torch.zeros(65536, dtype=torch.float64, device=cuda), atol=1e-5)
    s = api.reduce_f32(ReduceOp.Sum, x, [1])
    assert torch.allclose(m.mean.double() * 4096, s.double(), rtol=1e-5, atol=1e-3)
    # a sampled slice against the oracle
    sl = x[::4096].cpu().numpy()
    assert (u32(api.argmax(x[::4096], 1)) == orc.argmax_rows(sl)).all()
    cf.check(s[::4096].cpu().numpy(), orc.row_reduce(sl, 0), tol=1e-5)
    tot = api.global_sum(x).item()
    want = x.double().sum().item()
    assert abs(tot - want) <= 1e-5 * max(abs(want), 1.0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,axes", [((64, 4096), [1]), ((6, 768), [1]), ((33, 17), [0])])
def test_low_statistics_round_once(cuda, dtype, shape, axes):
    """softmax_low / log_softmax_low / layer_norm_low (low_statistics.rs:59-108):
    the f32 result rounded once to the input dtype, whether the row engine
    rounds while storing (contiguous rows) or the result goes through scratch
    (other axes)."""
    g = torch.Generator(device="cpu").manual_seed(31)
    x = (torch.randn(*shape, generator=g) * 3).to(dtype).to(cuda)
    pairs = [
        (api.softmax_low(x, axes), api.softmax(x, axes)),
        (api.log_softmax_low(x, axes), api.log_softmax(x, axes)),
        (api.layer_norm_low(x, axes, 1e-5), api.layer_norm(x, axes, 1e-5)),
    ]
    for got, f32 in pairs:
        assert got.dtype == dtype
        ref = api.cast_to_low(f32, dtype)
        assert torch.equal(got.view(torch.int16).cpu(), ref.view(torch.int16).cpu())


def test_layer_norm_f32_input_low_output(cuda):
    g = torch.Generator(device="cpu").manual_seed(32)
    x = torch.randn(8, 197, 768, generator=g).to(cuda)
    got = api.layer_norm_low(x, [2], 1e-5, torch.bfloat16)
    ref = api.cast_to_low(api.layer_norm(x, [2], 1e-5), torch.bfloat16)
    assert torch.equal(got.view(torch.int16).cpu(), ref.view(torch.int16).cpu())
