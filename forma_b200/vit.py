"""A ViT-style encoder forward chained from the operator API.

The composite workload that exercises the three hot-path families together:
convolution (the patch embedding and the token projections as 1x1
convolutions on a channels-last token map), layer norm, and fused attention,
joined by residual additions and a GELU.  Pre-norm blocks::

    x  = [cls; patches(img) W_p] + pos                 conv 16x16 stride 16
    for each layer:
        h  = LN(x)                                     layer_norm, eps 1e-5, rounded to BF16 as stored
        q, k, v = heads(h W_qkv)                       1x1 conv rounded to BF16 in its epilogue
        x  = x + concat_heads(attention(q, k, v)) W_o  fused attention rounded to BF16 in its epilogue,
                                                       1x1 conv adding into x
        h  = LN(x)
        x  = x + GELU(h W_1) W_2                        1x1 convs, GELU rounded to BF16, the second
                                                       conv adding into x

Tokens live as a channels-last [B, 1, L, E] map, so every projection is a
1x1 convolution whose input rows are the tokens (the tensor-core implicit
GEMM reads them in place) and whose result is written channels-last through
a permuted output view.  The residual additions and the fc1 GELU are applied
to the GEMM's f32 sums in its epilogue (the same arithmetic as the separate
add and GELU passes, so the results are identical); operands of the
contractions are rounded to the low dtype at the marked points; everything
else is f32.
Weights are random (seeded); no checkpoint is involved.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import api
from .api import AttentionOptions, ConvOptions

_ONE = ConvOptions([1, 1], [1, 1], [0, 0], [0, 0])  # 1x1, stride 1, no padding


@dataclass(frozen=True)
class ViTConfig:
    batch: int = 64
    image: int = 224
    channels: int = 3
    patch: int = 16
    embed: int = 768
    heads: int = 12
    layers: int = 12
    mlp: int = 3072
    eps: float = 1e-5

    @property
    def grid(self) -> int:
        return self.image // self.patch

    @property
    def tokens(self) -> int:
        return self.grid * self.grid + 1

    @property
    def head_dim(self) -> int:
        return self.embed // self.heads

    def flops(self) -> dict:
        """Multiply-add FLOPs (2 per MAC) of each stage of one forward."""
        B, L, E, M = self.batch, self.tokens, self.embed, self.mlp
        P = self.grid * self.grid
        K = self.channels * self.patch * self.patch
        per_layer = {
            "qkv": 2 * B * L * E * 3 * E,
            "attention": 4 * B * self.heads * L * L * self.head_dim,
            "proj": 2 * B * L * E * E,
            "mlp": 2 * 2 * B * L * E * M,
        }
        out = {"patch": 2 * B * P * E * K}
        for k, v in per_layer.items():
            out[k] = v * self.layers
        out["total"] = sum(out.values())
        return out


class ViTEncoder:
    """Random-init encoder; ``forward(img)`` takes [B, C, H, W] in the low dtype
    and returns the final tokens [B, L, E] (f32)."""

    def __init__(self, cfg: ViTConfig, device, dtype=torch.bfloat16, seed: int = 0):
        self.cfg, self.dtype, self.device = cfg, dtype, torch.device(device)
        g = torch.Generator(device="cpu").manual_seed(seed)
        E, M, K = cfg.embed, cfg.mlp, cfg.channels * cfg.patch * cfg.patch

        def w(o, i, kh=1, kw=1, fan=None):
            t = torch.randn(o, i, kh, kw, generator=g) / math.sqrt(fan or i * kh * kw)
            return t.to(dtype).to(self.device)

        self.w_patch = w(E, cfg.channels, cfg.patch, cfg.patch, fan=K)
        self.cls = (torch.randn(1, 1, E, generator=g) * 0.02).to(self.device)
        self.pos = (torch.randn(1, cfg.tokens, E, generator=g) * 0.02).to(self.device)
        self.blocks = []
        for _ in range(cfg.layers):
            self.blocks.append({
                "qkv": w(3 * E, E),
                "proj": w(E, E),
                "fc1": w(M, E),
                "fc2": w(E, M),
            })
        self._bufs = None

    def _buffers(self, B: int):
        if self._bufs is not None and self._bufs["B"] == B:
            return self._bufs
        cfg, dev, low = self.cfg, self.device, self.dtype
        L, E, M, H, D = cfg.tokens, cfg.embed, cfg.mlp, cfg.heads, cfg.head_dim
        G = cfg.grid
        self._bufs = {
            "B": B,
            "x": torch.empty(B, L, E, device=dev),
            "patches": torch.empty(B, G, G, E, device=dev),      # channels-last conv result
            "h_low": torch.empty(B, L, E, dtype=low, device=dev),
            "qkv_low": torch.empty(B, 1, L, 3 * E, dtype=low, device=dev),   # [B, L, 3, H, D] rounded once
            "a_low": torch.empty(B, L, E, dtype=low, device=dev),            # attention output, [B, L, H, D] order
            "m_low": torch.empty(B, 1, L, M, dtype=low, device=dev),
        }
        return self._bufs

    @staticmethod
    def _tokens(x_low: torch.Tensor) -> torch.Tensor:
        """Channels-last tokens [B, L, C] as the logical [B, C, 1, L] input of a 1x1 convolution."""
        B, L, Cin = x_low.shape
        return x_low.view(B, 1, L, Cin).permute(0, 3, 1, 2)

    @staticmethod
    def _residual(x_low: torch.Tensor, weight: torch.Tensor, x: torch.Tensor) -> None:
        """x [B, L, E] (f32) += 1x1 convolution of channels-last tokens x_low [B, L, Cin]."""
        B, L, E = x.shape
        api.conv_low_f32_accumulate(ViTEncoder._tokens(x_low), weight, _ONE, x.view(B, 1, L, E).permute(0, 3, 1, 2))

    def forward(self, img: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        B = img.shape[0]
        L, E, H, D, M = cfg.tokens, cfg.embed, cfg.heads, cfg.head_dim, cfg.mlp
        b = self._buffers(B)
        x = b["x"]
        # patch embedding (space-to-depth + tensor-core GEMM), then [cls; patches] + pos
        p = cfg.patch
        api.conv_low_f32_into(img, self.w_patch, ConvOptions([p, p], [1, 1], [0, 0], [0, 0]),
                              b["patches"].permute(0, 3, 1, 2))
        api.add(b["patches"].view(B, L - 1, E), self.pos[:, 1:].expand(B, L - 1, E), out=x[:, 1:])
        api.add(self.cls.expand(B, 1, E), self.pos[:, :1].expand(B, 1, E), out=x[:, :1])
        opts = AttentionOptions()  # default scale 1/sqrt(D), non-causal
        for blk in self.blocks:
            # attention sub-block
            api.layer_norm_low(x, [2], cfg.eps, self.dtype, out=b["h_low"])  # rounded as stored
            # QKV rounded once in the GEMM epilogue (conv_low), read by the
            # attention kernel as head-interleaved views of one buffer
            api.conv_low_into(self._tokens(b["h_low"]), blk["qkv"], _ONE, b["qkv_low"].permute(0, 3, 1, 2))
            qkv = b["qkv_low"].view(B, L, 3, H, D)
            q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))   # [B, H, L, D] views
            # attention rounded to the low dtype in its epilogue (attention_low)
            api.attention_low_into(q, k, v, None, opts, b["a_low"].view(B, L, H, D).permute(0, 2, 1, 3))
            self._residual(b["a_low"], blk["proj"], x)                  # x += proj (GEMM epilogue)
            # MLP sub-block
            api.layer_norm_low(x, [2], cfg.eps, self.dtype, out=b["h_low"])
            # fc1 with GELU and the 16-bit rounding in the GEMM epilogue
            # (bit-identical to conv_low_f32 then gelu_to_low; the f32 fc1
            # result never reaches HBM)
            api.conv_low_gelu_into(self._tokens(b["h_low"]), blk["fc1"], _ONE, b["m_low"].permute(0, 3, 1, 2))
            self._residual(b["m_low"].view(B, L, M), blk["fc2"], x)     # x += fc2
        return x
