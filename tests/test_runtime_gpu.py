"""Runtime services behind the C ABI on one GPU: the bounded-wait self-test,
prepared programs recorded and replayed through fb_program_*, the global sum
over an NCCL communicator made through fb_nccl_*, and the route record."""

import ctypes as C

import numpy as np
import pytest
import torch

from forma_b200 import _lib, api
from forma_b200.api import AttentionOptions, ConvOptions, ReduceOp
from forma_b200.program import Program

pytestmark = pytest.mark.gpu

SELFTEST_BIT = 1 << 6


def test_bounded_wait_gives_up_and_reports(cuda):
    """A wait that nothing completes ends after its limit with a status bit;
    the context stays usable and the bit clears once read."""
    assert api.device_status() == 0
    api.selftest_bounded_wait(1_000_000)  # 1 ms
    assert api.last_route() == ["selftest_wait_kernel"]
    assert api.device_status() == SELFTEST_BIT
    assert api.device_status() == 0
    x = torch.randn(64, 512, device=cuda)
    assert torch.equal(api.reduce_f32(ReduceOp.Max, x, [1]), x.max(dim=1).values)
    with pytest.raises(api.TensorError) as e:
        api.selftest_bounded_wait(0)
    assert e.value.kind == "InvalidInput"


def _c(stream):
    return C.c_void_p(stream.cuda_stream)


def test_program_through_the_c_abi(cuda):
    lib = _lib.load()
    s = torch.cuda.Stream()
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(2, 14, 14, 256, generator=g).bfloat16().to(cuda)
    w = (torch.randn(256, 3, 3, 256, generator=g) * 0.02).bfloat16().to(cuda)
    out = torch.empty(2, 256, 14, 14, device=cuda)
    rows = torch.randn(128, 1024, generator=g).to(cuda)
    sm = torch.empty_like(rows)
    opts = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])

    def step():
        api.conv_low_f32_into(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2), opts, out)
        di, do = api.describe(rows), api.describe(sm)
        api._check(lib.fb_softmax(C.byref(di), _lib.u32_array([1]), 1, C.byref(do), _c(s)))

    with torch.cuda.stream(s):
        step()  # eager: scratch and kernel attributes for this stream
        s.synchronize()
        want_conv, want_sm = out.clone(), sm.clone()
        out.zero_()
        sm.zero_()
        api._check(lib.fb_program_begin(_c(s)))
        step()
        prog = C.c_void_p()
        api._check(lib.fb_program_end(_c(s), C.byref(prog)))
        s.synchronize()
        assert float(out.abs().max()) == 0.0  # recorded, not run
        k, n, p = C.c_uint64(), C.c_uint64(), C.c_int32()
        api._check(lib.fb_program_stats(prog, C.byref(k), C.byref(n), C.byref(p)))
        assert k.value == 2 and n.value >= 2 and p.value == 0
        for _ in range(2):
            api._check(lib.fb_program_launch(prog, _c(s)))
        s.synchronize()
    assert torch.equal(out, want_conv) and torch.equal(sm, want_sm)
    assert lib.fb_program_destroy(prog) == 0
    assert api.device_status() == 0


def test_program_refuses_scratch_growth_while_recording(cuda):
    """A call that would allocate library scratch fails while recording (the
    recording itself stays valid); nothing is allocated under capture."""
    lib = _lib.load()
    s = torch.cuda.Stream()
    # torch hands out pooled stream handles, so this one may have library
    # scratch from an earlier call: ask for a patch gather (100 MB) larger
    # than any earlier call on a pooled stream needed
    x = torch.randn(16, 3, 1024, 1024, device=cuda).bfloat16()
    w = torch.randn(64, 3, 16, 16, device=cuda).bfloat16()
    out = torch.empty(16, 64, 64, 64, dtype=torch.bfloat16, device=cuda)
    opts = ConvOptions([16, 16], [1, 1], [0, 0], [0, 0])
    with torch.cuda.stream(s):
        api._check(lib.fb_program_begin(_c(s)))
        with pytest.raises(api.TensorError) as e:
            api.conv_low_into(x, w, opts, out)  # the patch route needs gather scratch
        assert "graph capture" in str(e.value)
        prog = C.c_void_p()
        api._check(lib.fb_program_end(_c(s), C.byref(prog)))
        assert lib.fb_program_destroy(prog) == 0
    with pytest.raises(api.TensorError) as e:
        api._check(lib.fb_program_begin(None))  # the legacy default stream cannot record
    assert e.value.kind == "InvalidInput"


def test_python_program_replays_and_refuses_temporaries(cuda):
    g = torch.Generator(device="cpu").manual_seed(4)
    q, k, v = (torch.randn(1, 2, 256, 64, generator=g).bfloat16().to(cuda) for _ in range(3))
    prog = Program(lambda: api.attention_low_f32(q, k, v, None, AttentionOptions(None, 0)))
    assert prog.stats()["kernel_launches"] == 1 and not prog.stats()["poisoned"]
    want = api.attention_low_f32(q, k, v, None, AttentionOptions(None, 0))
    got = prog.run()
    torch.cuda.synchronize()
    assert torch.equal(got, want)

    def with_temporary():
        t = api.softmax(torch.ones(8, 8, device=cuda) * 0, [1])  # the input is a freed temporary
        return t

    with pytest.raises(api.TensorError) as e:
        Program(with_temporary)
    assert e.value.kind == "Graph"
    assert api.device_status() == 0


def test_global_sum_over_a_one_rank_communicator(cuda):
    """fb_global_sum_nccl on a one-rank NCCL communicator made through the C
    ABI equals the local partial + rounding bit for bit (an all-reduce over
    one rank is the identity), on contiguous and strided shards."""
    uid = api.NcclCommunicator.unique_id()
    assert len(uid) == 128
    comm = api.NcclCommunicator.init_rank(1, uid, 0, cuda)
    try:
        g = torch.Generator(device=cuda).manual_seed(5)
        x = torch.randn(4096, 1000, device=cuda, generator=g)
        for t in (x, x.t(), x[:, :999], x[:0]):
            got = api.global_sum(t, comm)
            assert api.last_route()[-1] == "finish_sum_kernel"
            want = api.global_sum(t)
            assert torch.equal(got, want), (float(got), float(want))
        assert float(api.global_sum(x[:0], comm)) == 0.0
        ref = float(x.double().sum())
        assert abs(float(api.global_sum(x, comm)) - ref) <= 1e-6 * abs(ref) + 1e-3
    finally:
        comm.destroy()
    assert api.device_status() == 0


def test_comm_init_all_one_device(cuda):
    lib = _lib.load()
    comms = (C.c_void_p * 1)()
    devs = (C.c_int * 1)(0)
    api._check(lib.fb_nccl_comm_init_all(comms, 1, devs))
    try:
        comm = api.NcclCommunicator(C.c_void_p(comms[0]), cuda)
        x = torch.arange(1000, dtype=torch.float32, device=cuda)
        assert float(api.global_sum(x, comm)) == 499500.0
    finally:
        api._check(lib.fb_nccl_comm_destroy(C.c_void_p(comms[0])))


def test_route_names_each_path(cuda):
    x = torch.randn(4, 4096, device=cuda)
    api.softmax(x, [1])
    assert api.last_route() == ["rows_stream_kernel"]
    api.softmax(x[:, :768], [1])
    assert api.last_route() == ["rows_warp_kernel"]
    api.reduce_f32(ReduceOp.Sum, x.t(), [0])
    assert api.last_route() == ["rows_stream_kernel"] or api.last_route() == ["reduce_rows_kernel"]
    api.conv(torch.randn(1, 64, 8, 8, device=cuda), torch.randn(64, 64, 3, 3, device=cuda),
             ConvOptions([1, 1], [1, 1], [1, 1], [1, 1]))
    assert api.last_route() == ["conv2d_f32_tiled_kernel<3,3>"]
    api.conv(torch.randn(1, 3, 8, 8, device=cuda), torch.randn(5, 3, 2, 2, device=cuda),
             ConvOptions([1, 1], [1, 1], [0, 0], [0, 0]))
    assert api.last_route() == ["conv_direct_kernel"]
    api.conv_plan([1, 3, 8, 8], [5, 3, 2, 2], ConvOptions([1, 1], [1, 1], [0, 0], [0, 0]))
    assert api.last_route() == ["conv_direct_kernel"]  # host-only queries leave the record alone
    assert np.isfinite(api.global_sum(x).item())
