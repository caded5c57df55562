"""The encoder chain (patch convolution, then per layer: layer norm, QKV
projection, attention, output projection with the residual add, layer norm,
GELU MLP with the residual add) composed from the oracle's operators, in f64
with the chain's 16-bit rounding points.

TEST INFRASTRUCTURE ONLY, like the rest of ``oracle/``: imported by
``tests/`` (the encoder's parity tests) and ``bench.py``'s CPU-baseline leg.

Weights are numpy arrays: ``w_patch`` [E, C, p, p], ``pos`` [1, L, E],
``cls`` [1, 1, E], and per layer ``qkv`` [3E, E, 1, 1], ``proj`` [E, E, 1, 1],
``fc1`` [M, E, 1, 1], ``fc2`` [E, M, 1, 1] (the projections are 1x1
convolutions over channels-last tokens; as matrix products here).
"""

from __future__ import annotations

import numpy as np

from . import oracle as orc


def low(x, dtype: str = "bf16") -> np.ndarray:
    """Nearest-even rounding to a 16-bit format and back."""
    return orc.decode_bits(orc.round_bits(np.asarray(x, np.float32), dtype), dtype).astype(np.float64)


def gelu_tanh(x):
    """tanh GELU in f64 (tensor-core/src/host_tensor/activation.rs:9-20)."""
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def f32(x) -> np.ndarray:
    """f32 storage of an f64 result (the chain's f32 tensors)."""
    return np.asarray(x, np.float64).astype(np.float32).astype(np.float64)


def forward(img: np.ndarray, w_patch: np.ndarray, pos: np.ndarray, cls: np.ndarray, blocks: list, heads: int,
            patch: int, eps: float, nthreads: int = 1) -> np.ndarray:
    """Tokens [B, L, E] (f32 values) of the encoder on images [B, C, H, W]."""
    B = img.shape[0]
    E = w_patch.shape[0]
    D = E // heads
    pt = orc.conv(img, w_patch, [patch, patch], [1, 1], [0, 0], [0, 0], nthreads=nthreads)
    patches = f32(pt.reshape(B, E, -1).transpose(0, 2, 1))  # [B, P, E] f32 conv result
    L = patches.shape[1] + 1
    x = np.concatenate([np.broadcast_to(f32(cls + pos[:, :1]), (B, 1, E)), f32(patches + pos[:, 1:])], axis=1)

    def norm(t):
        return orc.row_stats(t.reshape(-1, E).astype(np.float32), eps, which=("norm",))["norm"].astype(
            np.float64).reshape(t.shape)

    def proj(t, weight):
        return f32(t @ weight[:, :, 0, 0].T)

    for blk in blocks:
        h = low(norm(x))
        qkv = proj(h, blk["qkv"]).reshape(B, L, 3, heads, D)
        q, k, v = (low(qkv[:, :, i].transpose(0, 2, 1, 3)) for i in range(3))
        a = orc.attention(q, k, v, nthreads=nthreads)
        a_low = low(np.asarray(a, np.float64).transpose(0, 2, 1, 3).reshape(B, L, E))
        x = f32(x + proj(a_low, blk["proj"]))
        m = proj(low(norm(x)), blk["fc1"])
        x = f32(x + proj(low(gelu_tanh(m)), blk["fc2"]))
    return x
