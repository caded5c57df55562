"""Prepared programs: operator sequences captured once and replayed as CUDA
graphs give the eager results, and follow in-place input updates."""

import numpy as np
import pytest
import torch

from forma_b200 import api
from forma_b200.api import AttentionOptions, ReduceOp
from forma_b200.program import Program
from forma_b200.vit import ViTConfig, ViTEncoder

pytestmark = pytest.mark.gpu


def test_encoder_forward_replays_bit_identical(cuda):
    cfg = ViTConfig(batch=4, image=64, channels=3, patch=16, embed=128, heads=2, layers=2, mlp=256)
    enc = ViTEncoder(cfg, cuda, seed=5)
    img = torch.randn(cfg.batch, 3, 64, 64, generator=torch.Generator(device="cpu").manual_seed(6)).bfloat16().to(cuda)
    eager = enc.forward(img).clone()
    prog = Program(enc.forward, img)
    for _ in range(2):
        out = prog.run()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    assert api.device_status() == 0


def test_program_follows_in_place_inputs(cuda):
    g = torch.Generator(device="cpu").manual_seed(7)
    q, k, v = (torch.randn(1, 2, 256, 64, generator=g).bfloat16().to(cuda) for _ in range(3))
    x = torch.randn(64, 4096, generator=g).to(cuda)

    def step():
        a = api.attention_low_f32(q, k, v, None, AttentionOptions(None, 0))
        return a, api.reduce_f32(ReduceOp.Sum, x, [1]), api.softmax(x, [1])

    prog = Program(step)
    for seed in (8, 9):
        src = torch.Generator(device="cpu").manual_seed(seed)
        q.copy_(torch.randn(1, 2, 256, 64, generator=src).bfloat16())
        x.copy_(torch.randn(64, 4096, generator=src))
        got = [t.clone() for t in prog.run()]
        want = step()
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a, b)
    assert api.device_status() == 0
