"""Drop-in for the reference's fp8_linear module: weight-only block-FP8 linear layers.

The public names and their behaviour follow fp8_linear.py:
  quantize / dequantize   1x128 absmax/448 e4m3 quantisation and its inverse (fp8_linear.py:30-39);
                          the bytes and scales must be identical, so the arithmetic is the same
  FP8Linear(linear)       module holding `q` / `s` buffers, `bias`, `in_features`, `out_features`
                          and an empty `weight` placeholder (fp8_linear.py:42-52)
  convert(module, ...)    swaps qualifying nn.Linear children for FP8Linear (fp8_linear.py:67-75)

FP8Linear.forward runs on the sm_100a kernels: up to 4 rows through the block-FP8 GEMV
(dm3::fp8_gemv, the reference's Triton `_gemv` path for <= 2 rows, fp8_linear.py:56-59) and more
rows through the block-FP8 GEMM (dm3::fp8_gemm, where the reference dequantises and calls
F.linear, fp8_linear.py:60-61).
"""

from __future__ import annotations

from typing import Callable, Iterator, Optional, Tuple

import torch
import torch.nn as nn

from . import ops

BLOCK = 128
E4M3_MAX = 448.0


def quantize(w: torch.Tensor):
    """e4m3 weights and fp32 scales s[N, K / 128] = max(absmax of the row's 128-block, 1e-12) / 448."""
    rows, cols = w.shape
    blocks = w.float().reshape(rows, cols // BLOCK, BLOCK)
    scale = blocks.abs().amax(dim=2).clamp(min=1e-12) / E4M3_MAX
    q = (blocks / scale.unsqueeze(2)).reshape(rows, cols).to(torch.float8_e4m3fn)
    return q, scale.contiguous()


def dequantize(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 weight float(q) * s with one scale per row and 128-wide K block."""
    rows, cols = q.shape
    return (q.float().reshape(rows, cols // BLOCK, BLOCK) * s.unsqueeze(2)).reshape(rows, cols)


class FP8Linear(nn.Module):
    """y = x @ dequant(q, s).T (+ bias) with e4m3 q [out, in] and fp32 s [out, in / 128].

    Built from an nn.Linear (quantised here) or, with `linear=None`, from ready q / s buffers."""

    def __init__(self, linear: Optional[nn.Linear] = None, *, q: Optional[torch.Tensor] = None,
                 s: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None):
        super().__init__()
        if linear is not None:
            q, s = quantize(linear.weight.data)
            bias = linear.bias
            ref = linear.weight
        elif q is None or s is None:
            raise ValueError("FP8Linear needs an nn.Linear or both q and s")
        else:
            ref = torch.empty(0, dtype=torch.bfloat16, device=q.device)
        self.register_buffer("q", q)
        self.register_buffer("s", s)
        self.bias = bias
        # the module is still asked for .weight's dtype and device by code written for nn.Linear
        self.weight = torch.empty(0, dtype=ref.dtype, device=ref.device)
        self.out_features, self.in_features = q.shape

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rows = x.reshape(-1, self.in_features).to(torch.bfloat16)
        fp32 = x.dtype == torch.float32
        if rows.shape[0] <= ops.MAX_ROWS:
            y = ops.fp8_gemv(rows, self.q, self.s, self.bias, fp32)
        else:
            y = ops.fp8_gemm(rows, self.q, self.s, self.bias, fp32)
        return y.to(x.dtype).reshape(*x.shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def _linear_sites(root: nn.Module) -> Iterator[Tuple[nn.Module, str, str, nn.Linear]]:
    """(parent, attribute, dotted name, layer) of every nn.Linear below root, parents first."""
    for parent_name, parent in list(root.named_modules()):
        for attr, child in list(parent.named_children()):
            if isinstance(child, nn.Linear):
                yield parent, attr, (f"{parent_name}.{attr}" if parent_name else attr), child


def convert(module: nn.Module, skip: Callable[[str, nn.Module], bool] = lambda name, m: False,
            min_out: int = 512) -> int:
    """Replaces every nn.Linear whose in_features is a multiple of 128 and whose out_features is at
    least min_out, unless skip(dotted_name, layer) says otherwise; returns how many were replaced."""
    chosen = [(parent, attr) for parent, attr, name, lin in _linear_sites(module)
              if lin.in_features % BLOCK == 0 and lin.out_features >= min_out and not skip(name, lin)]
    for parent, attr in chosen:
        setattr(parent, attr, FP8Linear(getattr(parent, attr)))
    return len(chosen)
