"""Drop-in for the reference's fp8_linear module (fp8_linear.py): block-FP8 weight-only linear layers.

`quantize` / `dequantize` / `convert` keep the reference's signatures and arithmetic
(fp8_linear.py:30-39, :67-75). `FP8Linear.forward` runs every row count through the sm_100a
block-FP8 GEMV (dm3::fp8_gemv) instead of the Triton `_gemv` for rows <= 2 and the dequantise +
F.linear path for longer inputs (fp8_linear.py:54-64); rows are processed four per launch.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import ops

BLOCK = 128


def quantize(w: torch.Tensor):
    """1x128 absmax/448 e4m3 quantisation of a [N, K] weight (fp8_linear.py:30-34): one fp32 scale
    per output row and 128-wide K block, s[N, K / 128]."""
    N, K = w.shape
    b = w.float().view(N, K // BLOCK, BLOCK)
    s = b.abs().amax(-1).clamp(min=1e-12) / 448.0
    return (b / s[..., None]).view(N, K).to(torch.float8_e4m3fn), s.contiguous()


def dequantize(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """float(q) * s, fp32 (fp8_linear.py:37-39)."""
    N, K = q.shape
    return (q.float().view(N, K // BLOCK, BLOCK) * s[..., None]).view(N, K)


class FP8Linear(nn.Module):
    """Block-FP8 weights (e4m3 q [N, K] + 1x128 scales s [N, K/128]) with the bias of the linear
    it replaces. Same buffers and attributes as the reference module (fp8_linear.py:42-52)."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        q, s = quantize(linear.weight.data)
        self.register_buffer("q", q)
        self.register_buffer("s", s)
        self.bias = linear.bias
        self.weight = torch.empty(0, dtype=linear.weight.dtype, device=linear.weight.device)
        self.out_features, self.in_features = q.shape

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.reshape(-1, self.in_features)
        out_fp32 = x.dtype == torch.float32
        y = ops.fp8_gemv(rows.to(torch.bfloat16), self.q, self.s, self.bias, out_fp32)
        return y.to(x.dtype).view(*x.shape[:-1], self.out_features)


def convert(module: nn.Module, skip=lambda name, m: False, min_out: int = 512) -> int:
    """Swaps every nn.Linear with in_features % 128 == 0 and out_features >= min_out (and not
    skipped) for an FP8Linear; returns the count (fp8_linear.py:67-75)."""
    swapped = 0
    for name, child in list(module.named_modules()):
        for attr, sub in list(child.named_children()):
            full = f"{name}.{attr}" if name else attr
            if isinstance(sub, nn.Linear) and sub.in_features % BLOCK == 0 and sub.out_features >= min_out and not skip(full, sub):
                setattr(child, attr, FP8Linear(sub))
                swapped += 1
    return swapped
