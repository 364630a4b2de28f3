"""Drop-in for fish-speech `fp8_moe.fp8_moe_forward` as the reference engine calls it
(engine.py:16 import; :147 OnDemandExperts.forward over ExpertStore slots; :236 Speaker)."""

from __future__ import annotations

import torch

from . import ops


def fp8_moe_forward(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, w13: torch.Tensor,
                    s13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor) -> torch.Tensor:
    """y[t] = sum_j weights[t, j] * down_e(silu(gate_e(x[t])) * up_e(x[t])), e = ids[t, j].

    x [T, H] bf16; ids [T, k] int64 indexing dim 0 of the expert tensors (ExpertStore slots or
    speaker experts); weights [T, k] bf16; w13 [E, 2I, H] e4m3 (gate rows then up rows), s13 its
    block scales; w2 [E, H, I] e4m3, s2 its block scales. Dim-0 strides may be those of the
    ExpertStore slot buffer (3 * I * H bytes, engine.py:32-34). Returns bf16 [T, H]."""
    return ops.moe_forward(x, ids, weights, w13, s13, w2, s2)
