"""Benchmark of the dense-op hot path on B200 (one process per GPU).

Headline workload: the row-reduction configuration, X [65536, 4096] f32
~N(0,1) (seed 1 + rank) per GPU.  One step runs, through the C ABI, every
operation the configuration names: per-row sum, max, argmax, softmax,
layer-norm statistics (moments) and a global sum over all ranks' rows (one
8-byte NCCL all-reduce).  The metric is algorithmic HBM bytes per second
summed over all ranks (weak scaling: each rank owns 65536 rows).  X is 1.07 GB
per pass, larger than the 126 MB L2, so no flush is needed between passes.

The JSON line also reports, per convolution / attention / GEMM / encoder
workload at its fixed size (sharded across the ranks: strong scaling),
TFLOP/s against the roofline (key "ops"), the dominant kernel's roofline, the
CPU baseline (the oracle on the host's cores, rows and one unit of each op
workload) and an end-to-end number through host buffers.

``--impl reference`` times the reference's CPU path (the oracle port of its
f64 algorithms, all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 65536, 4096
METRIC = "conv/attn TFLOP/s and reduce HBM GB/s at 1/2/4/8 B200 vs roofline"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "sm_max_mhz": d.get("sm_max_mhz", 1965.0), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "bf16_tflops_sustained": 1400.0,
            "sm_max_mhz": 1965.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a timed region."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str | None, enabled: bool = True):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.file = None
        self.enabled = enabled

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    @staticmethod
    def fallback_index() -> str:
        """nvidia-smi index of this process's GPU when the bus id is unknown."""
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        local = int(os.environ.get("LOCAL_RANK", "0"))
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if ids and local < len(ids) and ids[local].isdigit():
            return ids[local]
        return str(local)

    def lines(self) -> int:
        if self.file is None:
            return 0
        self.file.flush()
        try:
            return len(Path(self.file.name).read_text().splitlines())
        except OSError:
            return 0

    def wait_samples(self, keep_busy, count: int, limit_s: float = 5.0) -> None:
        """Keeps the GPU under the same load until the sampler has written
        `count` more lines (nvidia-smi needs a few hundred ms to start)."""
        if self.proc is None:
            return
        start, t0 = self.lines(), time.time()
        while self.lines() < start + count and time.time() - t0 < limit_s:
            keep_busy()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            bus = parts[1].lower()
            if self.bus_id and not (bus.endswith(self.bus_id[-12:]) or self.bus_id.endswith(bus[-12:])):
                continue
            if not self.bus_id and parts[0] != self.fallback_index():
                continue
            rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, val in zip(names, r[6:10]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def pci_bus_id(torch, dev) -> str | None:
    """nvidia-smi style bus id (DDDDDDDD:BB:DD.F) of a torch device, if known."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = getattr(p, "pci_bus_id", None)
        if isinstance(bus, str):
            return bus
        dom = getattr(p, "pci_domain_id", None)
        dv = getattr(p, "pci_device_id", None)
        if isinstance(bus, int) and isinstance(dom, int) and isinstance(dv, int):
            return f"{dom:08X}:{bus:02X}:{dv:02X}.0"
    except Exception:
        pass
    return None


# ------------------------------------------------------------- distributed

class Dist:
    def __init__(self, gpus: int):
        import torch

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus and gpus != 1:
            print(f"warning: --gpus {gpus} but WORLD_SIZE {self.world}", file=sys.stderr)
        self.torch = torch
        self.pg = None

    def init(self):
        torch = self.torch
        torch.cuda.set_device(self.local)
        self.comm = None
        if self.world > 1:
            from datetime import timedelta

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=60),
                                                 device_id=torch.device("cuda", self.local))
            self.pg = torch.distributed.group.WORLD
            # The global sum's all-reduce runs inside the backend, on an NCCL
            # communicator made through its C ABI: rank 0 creates the id and
            # the process group only carries it to the other ranks.
            from forma_b200.api import NcclCommunicator

            dev = torch.device("cuda", self.local)
            uid = torch.zeros(128, dtype=torch.uint8, device=dev)
            if self.rank == 0:
                uid.copy_(torch.frombuffer(bytearray(NcclCommunicator.unique_id()), dtype=torch.uint8))
            torch.distributed.broadcast(uid, 0)
            self.comm = NcclCommunicator.init_rank(self.world, bytes(uid.cpu().numpy().tobytes()), self.rank, dev)

    def barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier()

    def max(self, value: float) -> float:
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device="cuda")
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device="cuda")
        self.torch.distributed.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.comm is not None:
            self.torch.cuda.synchronize()
            self.comm.destroy()
            self.comm = None
        if self.world > 1:
            self.torch.distributed.destroy_process_group()


# -------------------------------------------------------- row workload

def row_ops(api, x, dist, timers=None):
    """One step of the row workload.  Returns the per-row results."""
    from forma_b200.api import ReduceOp

    out = {}

    def run(name, fn):
        if timers is not None:
            timers[name][0].record()
        out[name] = fn()
        if timers is not None:
            timers[name][1].record()

    run("row_sum", lambda: api.reduce_f32(ReduceOp.Sum, x, [1]))
    run("row_max", lambda: api.reduce_f32(ReduceOp.Max, x, [1]))
    run("row_argmax", lambda: api.argmax(x, 1))
    run("softmax", lambda: api.softmax(x, [1]))
    run("moments", lambda: api.moments(x, [1]))
    run("global_sum", lambda: api.global_sum(x, dist.comm))
    return out


def row_bytes(rows: int, cols: int) -> dict:
    """Algorithmic HBM bytes per launch of each operation."""
    n = rows * cols * 4
    return {"row_sum": n + rows * 4, "row_max": n + rows * 4, "row_argmax": n + rows * 4, "softmax": 2 * n,
            "moments": n + 2 * rows * 4, "global_sum": n + 8}


def cpu_baseline_rows(sample_rows: int, repeats: int = 1) -> dict:
    """The oracle (the reference's f64 algorithms) on the host's cores, on a
    sample of the row workload.  Returns bytes/s with the sample described."""
    import numpy as np

    from oracle import oracle as orc

    threads = orc.threads()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((sample_rows, COLS)).astype(np.float32)
    t0 = time.perf_counter()
    for _ in range(repeats):
        orc.row_reduce(x, 0, threads)
        orc.row_reduce(x, 3, threads)
        orc.argmax_rows(x, threads)
        orc.row_stats(x, 1e-5, threads, which=("softmax",))
        orc.row_stats(x, 1e-5, threads, which=("mean", "variance"))
        orc.sum_f64(x, threads)
    dt = (time.perf_counter() - t0) / repeats
    b = sum(row_bytes(sample_rows, COLS).values())
    return {"value": b / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{sample_rows} of {ROWS} rows x {COLS} f32 through sum, max, argmax, softmax, moments, "
                      f"global sum (oracle, f64 arithmetic, {threads} threads), {dt:.2f} s per pass; GB/s "
                      f"extrapolated per byte to the whole workload"}


# ------------------------------------------------- conv / attention workloads

def _flush_l2(buf):
    buf.add_(1)  # 256 MB written between timed launches: larger than the 126 MB L2


def time_op(torch, fn, iters, flush_buf, stream, flush=True):
    """Average device time of fn over `iters` launches, L2 flushed before each
    (flush=False: the call streams inputs larger than L2 itself).  Calls
    whose host-side issue cost approaches their device time (the decode) are
    preceded by 256 MB writes that need no host work, queued until the host
    can enqueue every timed call ahead of the device, so each event pair
    brackets device work only.  The lead is device work rather than an idle
    sleep: an idle gap lets the next compute-bound kernels run above the
    power-capped clocks they see in a busy stream."""
    import time

    t0 = time.perf_counter()
    fn()  # enqueue cost of one call (nothing here synchronises)
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    # one call from an idle device: its issue cost plus its device time
    a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    fn()
    b0.record(stream)
    torch.cuda.synchronize()
    span_s = a0.elapsed_time(b0) / 1e3
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    if host_s > 0.3 * span_s:  # issue cost above ~40% of the device time
        per_write_s = 60e-6  # one 256 MB read-modify-write, at most
        for _ in range(min(400, int(iters * (host_s + 1e-4) * 2 / per_write_s) + 1)):
            _flush_l2(flush_buf)
    for a, b in evs:
        if flush:
            _flush_l2(flush_buf)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters


def run_ops(api, dev, dist, args, pk) -> dict:
    """TFLOP/s of each convolution / attention / GEMM / encoder workload at
    its FIXED size, sharded across the ranks (strong scaling): images of C1,
    C3 and C5 by batch, (batch, head) pairs of C4 and of the decode case, rows
    of the GEMM.  Each rank builds and runs only its own shard; the time is
    the max over ranks and the FLOPs are those of the whole problem."""
    import torch

    from forma_b200.api import AttentionOptions, ConvOptions
    from forma_b200.shard import shard_range

    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(dist.rank)
    iters = max(3, min(args.steps, 10))
    res = {}
    fp32_peak = 148 * 128 * 2 * pk["sm_max_mhz"] * 1e6 / 1e12  # FMA lanes x 2 FLOP x max clock

    def mine(total):
        """This rank's [begin, end) of `total` units and the unit count."""
        b, e = shard_range(total, dist.world, dist.rank)
        return b, e, e - b

    L2_BYTES = 126 * 1024 * 1024

    def record(name, fn, flops, peak, peak_name, note=None, nbytes=None, shard=None, in_bytes=0):
        """`flops` / `nbytes`: the whole fixed problem's algorithmic FLOPs and
        HBM bytes (inputs read once, outputs written once); the time is the
        slowest rank's, so the rate is the job's.  `in_bytes`: the bytes this
        rank's call streams in; at least twice L2 on every rank and the calls
        are timed back to back (each call evicts its own inputs), otherwise L2
        is flushed by a 256 MB write before each call.  (Given only for calls
        whose outputs are small next to their inputs: a large output leaves
        dirty lines in L2 for the next call to write back, as the flush does.)"""
        for _ in range(2):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        no_flush = dist.max(0.0 if in_bytes >= 2 * L2_BYTES else 1.0) == 0.0  # the same choice on every rank
        ms = dist.max(time_op(torch, fn, iters, flush, stream, flush=not no_flush))
        tf = flops / (ms / 1e3) / 1e12
        res[name] = {"tflops": round(tf, 2), "ms": round(ms, 4), "flop_per_call": flops,
                     "roofline_frac": round(tf / peak / dist.world, 4), "peak_tflops": round(peak, 1),
                     "peak": peak_name + (f" per GPU, x{dist.world} GPUs" if dist.world > 1 else ""),
                     "scaling": "strong", "shard": shard,
                     "l2": (f"inputs larger than L2 ({in_bytes / 2**20:.0f} MiB per call on this rank), no flush"
                            if no_flush else "L2 flushed by a 256 MB write before each call")}
        if nbytes:
            gbs = nbytes / (ms / 1e3) / 1e9
            res[name].update({"bytes_per_call": nbytes, "hbm_gbs": round(gbs, 1),
                              "hbm_frac": round(gbs / pk["hbm_gbs"] / dist.world, 4),
                              "bound": "hbm" if gbs / pk["hbm_gbs"] > tf / peak else "tensor"})
        if note:
            res[name]["note"] = note

    def blank(*shape, dtype=torch.float32):
        return torch.empty(*shape, dtype=dtype, device=dev)

    # C1: conv2d fp32 NCHW [8,64,56,56] x [64,64,3,3], stride 1, pad 1 (bit-faithful f32 path), images sharded
    b0, b1, n = mine(8)
    x = torch.rand(max(n, 1), 64, 56, 56, device=dev, generator=g) * 2 - 1
    w = torch.randn(64, 64, 3, 3, device=dev, generator=g) * math.sqrt(2 / 576)
    o = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])
    record("conv_f32_c1", (lambda: api.conv(x[:n], w, o)) if n else (lambda: None), 2 * 8 * 64 * 56 * 56 * 64 * 9,
           fp32_peak, "fp32 FMA peak (148 SMs x 128 lanes x 2 x max clock)",
           "separate f32 multiply and add (reference order), so half the FMA peak is this kernel's ceiling",
           shard=f"images {b0}:{b1} of 8 on this rank")
    del x, w
    # C3a/C3b: ResNet-50 stage convs, bf16 NHWC, batch 256 sharded by image, f32 output
    b0, b1, n = mine(256)
    for name, cin, k, pad in (("conv_bf16_3x3_c3a", 256, 3, 1), ("conv_bf16_1x1_c3b", 1024, 1, 0)):
        xn = torch.randn(n, 14, 14, cin, device=dev, generator=g).bfloat16()
        wn = (torch.randn(256, k, k, cin, device=dev, generator=g) * math.sqrt(2 / (cin * k * k))).bfloat16()
        xv, wv = xn.permute(0, 3, 1, 2), wn.permute(0, 3, 1, 2)  # NHWC / OHWI storage, logical NCHW / OIHW
        out = blank(n, 256, 14, 14)  # contiguous f32 [N, O, P, Q], as the reference allocates
        oc = ConvOptions([1, 1], [1, 1], [pad, pad], [pad, pad])
        record(name, lambda: api.conv_low_f32_into(xv, wv, oc, out), 2 * 256 * 14 * 14 * 256 * cin * k * k,
               pk["bf16_tflops"], "measured bf16 dense (burst)",
               nbytes=256 * 14 * 14 * cin * 2 + wn.numel() * 2 * dist.world + 256 * 256 * 14 * 14 * 4,
               shard=f"images {b0}:{b1} of 256 on this rank")
        del xn, wn, out
    # C4: causal attention bf16 [8, 32, 4096, 128], scale 1/sqrt(128), f32 output; the 256 (batch, head)
    # pairs sharded as heads of a [pairs, L, D] view
    L = 4096
    p0, p1, n = mine(8 * 32)
    q, k, v = (torch.randn(n, L, 128, device=dev, generator=g).bfloat16() for _ in range(3))
    o4 = blank(n, L, 128)
    record("attention_bf16_causal_c4", lambda: api.attention_low_f32_into(q, k, v, None, AttentionOptions(causal=0), o4),
           4 * 8 * 32 * 128 * L * (L + 1) // 2, pk["bf16_tflops"], "measured bf16 dense (burst)",
           "causal FLOPs count the diagonal: 4*B*H*D*L(L+1)/2", nbytes=8 * 32 * L * 128 * (3 * 2 + 4),
           shard=f"(batch, head) pairs {p0}:{p1} of 256 on this rank", in_bytes=n * L * 128 * 2 * 3)
    del q, k, v, o4
    # decode: one query per head, 32 query heads over 8 key/value heads, 8192 keys, bf16 (HBM-bound:
    # reads K and V once); batches sharded
    b0, b1, n = mine(8)
    q = torch.randn(max(n, 1), 32, 1, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(max(n, 1), 8, 8192, 128, device=dev, generator=g).bfloat16()
    v = torch.randn(max(n, 1), 8, 8192, 128, device=dev, generator=g).bfloat16()
    record("attention_bf16_decode_gqa",
           (lambda: api.attention_low_f32(q[:n], k[:n], v[:n], None, AttentionOptions())) if n else (lambda: None),
           4 * 8 * 32 * 1 * 8192 * 128, pk["bf16_tflops"], "measured bf16 dense (burst)",
           "the 4 query heads of a key/value head as one 16-row block on the warp-level MMA, K/V streamed once "
           "through per-warp cp.async rings, key ranges merged on the device",
           nbytes=2 * 8 * 8 * 8192 * 128 * 2 + 8 * 32 * 128 * 2 + 8 * 32 * 128 * 4, shard=f"batches {b0}:{b1} of 8",
           in_bytes=n * 8 * 8192 * 128 * 2 * 2)
    del q, k, v
    # low-precision GEMM (the reference's cuBLAS matmul_low_f32): [8192, 8192] x [8192, 8192] bf16, f32
    # output, rows of the left operand sharded
    r0, r1, n = mine(8192)
    a = torch.randn(n, 8192, device=dev, generator=g).bfloat16()
    b = torch.randn(8192, 8192, device=dev, generator=g).bfloat16()
    c = blank(n, 8192)
    record("matmul_bf16_8192", lambda: api.matmul_low_f32(a, b, out=c), 2 * 8192 ** 3, pk["bf16_tflops"],
           "measured bf16 dense (burst)", "row-major right operand (MN-major B); f32 output",
           nbytes=8192 * 8192 * (2 + 4) + b.numel() * 2 * dist.world, shard=f"rows {r0}:{r1} of 8192")
    del a, b, c
    # C5: ViT-style encoder forward, [64,3,224,224] bf16, patch 16, 12 layers (E 768, H 12, D 64, L 197,
    # MLP 3072); the 64 images sharded, the same weights on every rank
    from forma_b200.vit import ViTConfig, ViTEncoder

    cfg = ViTConfig()
    b0, b1, n = mine(cfg.batch)
    enc = ViTEncoder(cfg, dev, seed=0)
    img = torch.randn(n, cfg.channels, cfg.image, cfg.image, device=dev, generator=g).bfloat16()
    fl = cfg.flops()
    record("vit_encoder_c5", lambda: enc.forward(img), fl["total"], pk["bf16_tflops"], "measured bf16 dense (burst)",
           "random-init pre-norm encoder, LN eps 1e-5, tanh GELU; FLOPs = patch conv + per layer QKV/out/MLP "
           "projections (1x1 convs) + attention 4*B*H*L^2*D; glue (casts, adds, LN) counted as time only",
           shard=f"images {b0}:{b1} of {cfg.batch}")
    res["vit_encoder_c5"]["flops_by_stage"] = fl
    # the same forward as a prepared program (one CUDA graph launch per forward, fb_program_*)
    from forma_b200.program import Program

    prog = Program(enc.forward, img, device=dev)
    record("vit_encoder_c5_graph", prog.run, fl["total"], pk["bf16_tflops"], "measured bf16 dense (burst)",
           "the C5 forward recorded once and replayed as one CUDA graph (fb_program_*, forma_b200.program.Program)",
           shard=f"images {b0}:{b1} of {cfg.batch}")
    prog.close()
    del prog, enc, img
    return res


def cpu_baseline_ops() -> dict:
    """The oracle (the reference's f64 algorithms) on the host's cores on one
    unit of each fixed problem, extrapolated per unit to the whole problem:
    one image of C1 / C3a / C3b / C5, one (batch, head) pair of C4, one
    (batch, key/value head) unit of the decode."""
    import numpy as np

    from oracle import oracle as orc

    threads = orc.threads()
    rng = np.random.default_rng(0)
    out = {}

    def timed(fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    x = rng.uniform(-1, 1, (1, 64, 56, 56)).astype(np.float32)
    w = (rng.standard_normal((64, 64, 3, 3)) * math.sqrt(2 / 576)).astype(np.float32)
    dt = timed(lambda: orc.conv_f32_seq(x, w, [1, 1], [1, 1], [1, 1], [1, 1], 1, threads))
    out["conv_f32_c1"] = {"tflops": 2 * 64 * 56 * 56 * 64 * 9 / dt / 1e12, "sample": "1 of 8 images, f32 reference order"}
    for name, cin, k, pad in (("conv_bf16_3x3_c3a", 256, 3, 1), ("conv_bf16_1x1_c3b", 1024, 1, 0)):
        x = rng.standard_normal((1, cin, 14, 14)).astype(np.float32)
        w = rng.standard_normal((256, cin, k, k)).astype(np.float32)
        dt = timed(lambda: orc.conv(x, w, [1, 1], [1, 1], [pad, pad], [pad, pad], 1, threads))
        out[name] = {"tflops": 2 * 14 * 14 * 256 * cin * k * k / dt / 1e12, "sample": "1 of 256 images, f64"}
    q, kk, v = (rng.standard_normal((1, 1, 4096, 128)).astype(np.float32) for _ in range(3))
    dt = timed(lambda: orc.attention(q, kk, v, None, None, 0, threads))
    out["attention_bf16_causal_c4"] = {"tflops": 4 * 128 * 4096 * 4097 // 2 / dt / 1e12,
                                       "sample": "1 of 256 (batch, head) pairs, f64 dense attention"}
    # decode: one (batch, key/value head) unit of the 8 x 32/8 heads x 8192 keys problem
    q = rng.standard_normal((1, 4, 1, 128)).astype(np.float32)
    kk, v = (rng.standard_normal((1, 1, 8192, 128)).astype(np.float32) for _ in range(2))
    dt = timed(lambda: orc.attention(q, kk, v, None, None, None, threads))
    out["attention_bf16_decode_gqa"] = {"tflops": 4 * 4 * 8192 * 128 / dt / 1e12,
                                        "gbs": 2 * 8192 * 128 * 2 / dt / 1e9,
                                        "sample": "1 of 64 (batch, key/value head) units, f64 dense attention; "
                                                  "GB/s counts the unit's K/V at 2 bytes per value"}
    # C5: one image through the encoder chain composed from the oracle's operators
    from forma_b200.vit import ViTConfig
    from oracle import vit as ovit

    cfg = ViTConfig()
    E, M, C, P = cfg.embed, cfg.mlp, cfg.channels, cfg.patch
    sd = 1.0 / math.sqrt(E)
    blocks = [{"qkv": rng.standard_normal((3 * E, E, 1, 1)) * sd, "proj": rng.standard_normal((E, E, 1, 1)) * sd,
               "fc1": rng.standard_normal((M, E, 1, 1)) * sd,
               "fc2": rng.standard_normal((E, M, 1, 1)) / math.sqrt(M)}]  # one of the 12 layers
    img = rng.standard_normal((1, C, cfg.image, cfg.image))
    wp = rng.standard_normal((E, C, P, P)) / math.sqrt(C * P * P)
    pos, cls = rng.standard_normal((1, cfg.tokens, E)) * 0.02, rng.standard_normal((1, 1, E)) * 0.02
    dt = timed(lambda: ovit.forward(img, wp, pos, cls, blocks, cfg.heads, P, cfg.eps, nthreads=threads))
    fl = cfg.flops()
    one = (fl["patch"] + (fl["total"] - fl["patch"]) / cfg.layers) / cfg.batch  # patch conv + one layer, one image
    out["vit_encoder_c5"] = {"tflops": one / dt / 1e12,
                             "sample": "1 of 64 images, the patch convolution and 1 of 12 layers, through the encoder "
                                       "composed from the oracle (f64 convolution, attention and layer norm; "
                                       "projections as f64 matrix products)"}
    for v_ in out.values():
        v_["tflops"] = round(v_["tflops"], 5)
        if "gbs" in v_:
            v_["gbs"] = round(v_["gbs"], 3)
        v_.update({"cores": threads, "kind": "port", "extrapolated": True})
    return out


# ------------------------------------------------------------------ main

def run_forma(args) -> int:
    import torch

    dist = Dist(args.gpus)
    dist.init()
    from forma_b200 import api

    dev = torch.device("cuda", dist.local)
    pk = peaks()
    g = torch.Generator(device=dev).manual_seed(1 + dist.rank)
    rows = args.rows
    x = torch.randn(rows, COLS, device=dev, generator=g, dtype=torch.float32)
    bytes_per = row_bytes(rows, COLS)
    step_bytes = sum(bytes_per.values())
    stream = torch.cuda.current_stream(dev)

    for _ in range(args.warmup):
        row_ops(api, x, dist)
    torch.cuda.synchronize(dev)

    # device-resident timed region
    timers = {k: [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(args.steps)]
              for k in bytes_per}
    per_kernel_ms = {k: 0.0 for k in bytes_per}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    class _Local:
        comm = None  # no collective: ranks may run different numbers of busy steps

    def busy():
        row_ops(api, x, _Local)
        torch.cuda.synchronize(dev)

    with ClockSampler(None if args.no_clocks else pci_bus_id(torch, dev), enabled=not args.no_clocks) as clocks:
        # Clocks are sampled under the same load just before, during and just
        # after the timed region (nvidia-smi samples every 200 ms).
        clocks.wait_samples(busy, 2)
        launches0 = api.launch_count()
        dist.barrier()
        torch.cuda.synchronize(dev)
        start.record(stream)
        for i in range(args.steps):
            step_timers = {k: v[i] for k, v in timers.items()}
            row_ops(api, x, dist, step_timers)
        stop.record(stream)
        torch.cuda.synchronize(dev)
        launches = api.launch_count() - launches0
        clocks.wait_samples(busy, 1)
    local_ms = start.elapsed_time(stop)
    for k, evs in timers.items():
        per_kernel_ms[k] = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    total_ms = dist.max(local_ms)
    value = dist.sum(step_bytes * args.steps) / (total_ms / 1e3) / 1e9

    dom = max(per_kernel_ms, key=per_kernel_ms.get)
    achieved = bytes_per[dom] / (per_kernel_ms[dom] / 1e3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / f"{dom}_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("bytes_per_launch")

    # end to end: pinned host input copied in, results read back, every step
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(api, torch, x, dist, dev, stream, step_bytes, args)

    ops = {}
    if not args.no_ops:
        ops = run_ops(api, dev, dist, args, pk)

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = cpu_baseline_rows(args.cpu_rows)
        if not args.no_ops:
            cpu["ops"] = cpu_baseline_ops()
    return emit(args, dist, pk, value, total_ms, step_bytes, dom, achieved, traffic, per_kernel_ms, bytes_per, e2e,
                launches, clocks, cpu, ops, rows)


def run_e2e(api, torch, x, dist, dev, stream, step_bytes, args):
    """The row workload through the public API from pinned host memory: every
    step copies its input X host -> device and reads its per-row results and
    the global sum back.  Two device buffers let the copy of step i + 1 (on its
    own stream) run while step i computes; each step's compute waits for its
    own copy, and the timed region spans every copy and every read-back."""
    ROWS = x.shape[0]
    host_x = torch.empty(ROWS, COLS, dtype=torch.float32, pin_memory=True)
    host_x.copy_(x.cpu())
    outs_host = {k: torch.empty(ROWS, dtype=torch.float32, pin_memory=True) for k in ("row_sum", "row_max", "mean", "var")}
    arg_host = torch.empty(ROWS, dtype=torch.int32, pin_memory=True)
    gs_host = torch.empty((), dtype=torch.float32, pin_memory=True)
    x_dev = [torch.empty_like(x), torch.empty_like(x)]
    copy_stream = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [None, None]  # event after the compute that last read each buffer
    e2e_steps = max(2, min(args.steps, 5))

    def issue_copy(i, after=None):
        buf = i % 2
        if after is not None:
            copy_stream.wait_event(after)
        if consumed[buf] is not None:
            copy_stream.wait_event(consumed[buf])
        with torch.cuda.stream(copy_stream):
            x_dev[buf].copy_(host_x, non_blocking=True)
            copied[buf].record(copy_stream)

    def compute(i):
        buf = i % 2
        stream.wait_event(copied[buf])
        r = row_ops(api, x_dev[buf], dist)
        ev = torch.cuda.Event()
        ev.record(stream)
        consumed[buf] = ev
        outs_host["row_sum"].copy_(r["row_sum"], non_blocking=True)
        outs_host["row_max"].copy_(r["row_max"], non_blocking=True)
        arg_host.copy_(r["row_argmax"], non_blocking=True)
        outs_host["mean"].copy_(r["moments"].mean, non_blocking=True)
        outs_host["var"].copy_(r["moments"].variance, non_blocking=True)
        gs_host.copy_(r["global_sum"], non_blocking=True)

    def run(n, start=None):
        issue_copy(0, start)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            compute(i)

    run(2)  # warm-up of both buffers and streams
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(e2e_steps, e0)  # the first copy starts after e0
    e1.record(stream)  # after the last compute, which waited for every copy, and the last read-back
    torch.cuda.synchronize(dev)
    e2e_ms = dist.max(e0.elapsed_time(e1))
    e2e_value = dist.sum(step_bytes * e2e_steps) / (e2e_ms / 1e3) / 1e9
    h2d = ROWS * COLS * 4
    d2h = ROWS * 4 * 5 + 4
    return {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": e2e_steps, "pipelined": "the copy of step i + 1 overlaps the compute of step i"}


def emit(args, dist, pk, value, total_ms, step_bytes, dom, achieved, traffic, per_kernel_ms, bytes_per, e2e, launches,
         clocks, cpu, ops, rows) -> int:
    if dist.rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": dist.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "row reductions: X [65536, 4096] f32 ~N(0,1) per GPU; per-row sum, max, argmax, "
                                   "softmax, layer-norm moments; global sum over all ranks (one f64 all-reduce)",
                       "rows_per_gpu": rows, "cols": COLS, "parallelism": f"rows sharded over {dist.world} GPU(s)",
                       "l2": "inputs larger than L2 (1.07 GB per pass), no flush",
                       "bytes_per_step_per_gpu": step_bytes},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
                         "peak_source": pk["source"]},
            "kernels_ms": {k: round(v, 4) for k, v in per_kernel_ms.items()},
            "kernels_frac_of_hbm": {k: round(bytes_per[k] / (v / 1e3) / 1e9 / pk["hbm_gbs"], 4)
                                    for k, v in per_kernel_ms.items()},
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "ops": ops,
        }
        print(json.dumps(line), flush=True)
    dist.close()
    return 0


def run_reference(args) -> int:
    """The reference's CPU path (oracle port, all host threads), bounded sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    from oracle import oracle as orc

    threads = orc.threads()
    rows = args.cpu_rows
    rng = np.random.default_rng(1)
    x = rng.standard_normal((rows, COLS)).astype(np.float32)
    b = sum(row_bytes(rows, COLS).values())

    def step():
        orc.row_reduce(x, 0, threads)
        orc.row_reduce(x, 3, threads)
        orc.argmax_rows(x, threads)
        orc.row_stats(x, 1e-5, threads, which=("softmax",))
        orc.row_stats(x, 1e-5, threads, which=("mean", "variance"))
        orc.sum_f64(x, threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = b / dt / 1e9
    sample = (f"{rows} of {ROWS} rows x {COLS} f32 per step through sum, max, argmax, softmax, moments, global sum "
              f"(oracle port of the reference's f64 algorithms, {threads} threads); GB/s extrapolated per byte "
              f"from the {rows}-row sample to the {ROWS}-row workload")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "row reductions: X [65536, 4096] f32 ~N(0,1); per-row sum, max, argmax, softmax, "
                               "layer-norm moments; global sum", "rows_per_gpu": ROWS, "cols": COLS,
                   "sample_rows": rows, "extrapolated": True},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_profile(args) -> int:
    """Runs one workload a few times (for ncu captures of a single kernel)."""
    import torch

    from forma_b200 import api
    from forma_b200.api import AttentionOptions, ConvOptions, ReduceOp

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    name = args.profile
    if name in ("conv_c3a", "conv_c3b"):
        cin, k, pad = (256, 3, 1) if name == "conv_c3a" else (1024, 1, 0)
        x = torch.randn(256, 14, 14, cin, device=dev, generator=g).bfloat16().permute(0, 3, 1, 2)
        w = (torch.randn(256, k, k, cin, device=dev, generator=g) * 0.02).bfloat16().permute(0, 3, 1, 2)
        o = ConvOptions([1, 1], [1, 1], [pad, pad], [pad, pad])
        fn = lambda: api.conv_low_f32(x, w, o)  # noqa: E731
    elif name in ("attn_c4", "attn_c4_small"):
        b = 8 if name == "attn_c4" else 2
        q = torch.randn(b, 32, 4096, 128, device=dev, generator=g).bfloat16()
        k_ = torch.randn(b, 32, 4096, 128, device=dev, generator=g).bfloat16()
        v = torch.randn(b, 32, 4096, 128, device=dev, generator=g).bfloat16()
        fn = lambda: api.attention_low_f32(q, k_, v, None, AttentionOptions(causal=0))  # noqa: E731
    elif name == "decode_gqa":
        # the decode entry: one query per head, 32 query heads over 8 key/value heads, 8192 keys, D 128
        q = torch.randn(8, 32, 1, 128, device=dev, generator=g).bfloat16()
        k_ = torch.randn(8, 8, 8192, 128, device=dev, generator=g).bfloat16()
        v = torch.randn(8, 8, 8192, 128, device=dev, generator=g).bfloat16()
        fn = lambda: api.attention_low_f32(q, k_, v, None, AttentionOptions())  # noqa: E731
    elif name == "conv_c1":
        x = torch.rand(8, 64, 56, 56, device=dev, generator=g) * 2 - 1
        w = torch.randn(64, 64, 3, 3, device=dev, generator=g) * 0.06
        o = ConvOptions([1, 1], [1, 1], [1, 1], [1, 1])
        fn = lambda: api.conv(x, w, o)  # noqa: E731
    elif name == "rows_softmax":
        x = torch.randn(args.rows, COLS, device=dev, generator=g)
        fn = lambda: api.softmax(x, [1])  # noqa: E731
    elif name == "rows_argmax":
        x = torch.randn(args.rows, COLS, device=dev, generator=g)
        fn = lambda: api.argmax(x, 1)  # noqa: E731
    elif name == "rows_moments":
        x = torch.randn(args.rows, COLS, device=dev, generator=g)
        fn = lambda: api.moments(x, [1])  # noqa: E731
    elif name == "rows_max_argmax_moments":
        x = torch.randn(args.rows, COLS, device=dev, generator=g)

        def fn():
            api.reduce_f32(ReduceOp.Max, x, [1])
            api.argmax(x, 1)
            api.moments(x, [1])
    elif name in ("c5_qkv", "c5_fc1"):
        # one C5 layer projection as a 1x1 convolution on channels-last tokens:
        # QKV [64*197, 768] x [768, 2304] rounded to BF16, or fc1 (x 3072) with GELU
        cout = 2304 if name == "c5_qkv" else 3072
        t = torch.randn(64, 197, 768, device=dev, generator=g).bfloat16()
        w = (torch.randn(cout, 768, 1, 1, device=dev, generator=g) * 768 ** -0.5).bfloat16()
        o = torch.empty(64, 1, 197, cout, dtype=torch.bfloat16, device=dev)
        xin, ov = t.view(64, 1, 197, 768).permute(0, 3, 1, 2), o.permute(0, 3, 1, 2)
        one = ConvOptions([1, 1], [1, 1], [0, 0], [0, 0])
        if name == "c5_qkv":
            fn = lambda: api.conv_low_into(xin, w, one, ov)  # noqa: E731
        else:
            fn = lambda: api.conv_low_gelu_into(xin, w, one, ov)  # noqa: E731
    elif name == "c5_proj":
        # the C5 attention output projection: [64*197, 768] x [768, 768] added
        # into the f32 tokens in the GEMM epilogue
        t = torch.randn(64, 197, 768, device=dev, generator=g).bfloat16()
        w = (torch.randn(768, 768, 1, 1, device=dev, generator=g) * 768 ** -0.5).bfloat16()
        x = torch.randn(64, 1, 197, 768, device=dev, generator=g)
        xin, xv = t.view(64, 1, 197, 768).permute(0, 3, 1, 2), x.permute(0, 3, 1, 2)
        one = ConvOptions([1, 1], [1, 1], [0, 0], [0, 0])
        fn = lambda: api.conv_low_f32_accumulate(xin, w, one, xv)  # noqa: E731
    elif name == "c5_attn":
        # one C5 layer's attention: [64, 12 heads, 197 tokens, 64] BF16 views of
        # the packed QKV rows, BF16 rows out
        qkv = torch.randn(64, 197, 3, 12, 64, device=dev, generator=g).bfloat16()
        qv, kv, vv = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
        out = torch.empty(64, 197, 12, 64, dtype=torch.bfloat16, device=dev)
        fn = lambda: api.attention_low_into(qv, kv, vv, None, AttentionOptions(), out.permute(0, 2, 1, 3))  # noqa: E731
    elif name == "vit_c5":
        from forma_b200.vit import ViTConfig, ViTEncoder

        cfg = ViTConfig()
        enc = ViTEncoder(cfg, dev)
        img = torch.randn(cfg.batch, cfg.channels, cfg.image, cfg.image, device=dev, generator=g).bfloat16()
        fn = lambda: enc.forward(img)  # noqa: E731
    else:
        raise SystemExit(f"unknown profile workload {name}")
    for _ in range(max(1, args.steps)):
        fn()
    torch.cuda.synchronize()
    status = api.device_status()
    print(json.dumps({"profile": name, "launches": api.launch_count(), "device_status": status}))
    return 0 if status == 0 else 1


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["forma", "reference"], default="forma")
    ap.add_argument("--cpu-rows", type=int, default=2048)
    ap.add_argument("--no-ops", action="store_true", help="skip the conv/attention workloads")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-clocks", action="store_true", help="skip clock sampling (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end pass (profiling runs)")
    ap.add_argument("--rows", type=int, default=ROWS, help="rows per GPU (profiling runs use fewer)")
    ap.add_argument("--profile", default=None,
                    help="run one workload --steps times and exit (conv_c3a, conv_c3b, attn_c4, attn_c4_small, vit_c5, "
                         "c5_qkv, c5_fc1, decode_gqa, "
                         "rows_max_argmax_moments, "
                         "conv_c1, rows_softmax, rows_argmax, rows_moments)")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "forma":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)
    return run_forma(args)


if __name__ == "__main__":
    sys.exit(main())
