"""Seeded synthetic inputs shared by the fixture generator and the tests (CPU torch.Generator).

Shapes follow the Drama-3 speaker MoE: hidden H = 2048, expert intermediate I = 512, 32 distilled
experts with top-8 routing, and a 256-expert bf16 router. Weights are N(0, 0.02); activations are
N(0, 1) rows RMS-normalised as exp3_distill.rms (exp3_distill.py:51-52), then bf16.
"""

from __future__ import annotations

import torch

H, I, E_SPK, E_ALL = 2048, 512, 32, 256
BF16 = torch.bfloat16


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def rms(x: torch.Tensor) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)


def decode_rows(t: int, seed: int, h: int = H) -> torch.Tensor:
    return rms(torch.randn(t, h, generator=gen(seed))).to(BF16)


def block_quant_input() -> torch.Tensor:
    """[2, 256, 384] fp32 with an all-zero block, a large-magnitude block and subnormal-range values."""
    w = torch.randn(2, 256, 384, generator=gen(1)) * 0.02
    w[0, :128, :128] = 0.0
    w[1, 128:, 256:] *= 1e4
    w[0, 128:, 128:256] *= 1e-6
    return w


def row_quant_input() -> torch.Tensor:
    return (torch.randn(96, 512, generator=gen(2)) * 0.02).to(BF16)


def gemv_case():
    """x [3, 512] bf16, weight [200, 512] bf16 (N not a multiple of the Triton tile)."""
    x = torch.randn(3, 512, generator=gen(3)).to(BF16)
    w = (torch.randn(200, 512, generator=gen(4)) * 0.02).to(BF16)
    return x, w


def speaker_params(seed: int = 10, e: int = E_SPK, h: int = H, i: int = I) -> dict:
    """Distilled speaker layer: gate [E, H] fp32, bias [H] fp32, w13 [E, 2I, H], w2 [E, H, I] (fp32,
    block-quantised by Speaker / fp8_block)."""
    g = gen(seed)
    return {
        "gate": torch.randn(e, h, generator=g) * 0.02,
        "bias": torch.randn(h, generator=g) * 0.02,
        "w13": torch.randn(e, 2 * i, h, generator=g) * 0.02,
        "w2": torch.randn(e, h, i, generator=g) * 0.02,
    }


class SharedMLP(torch.nn.Module):
    """A shared expert with gate/up/down bf16 linears: down(silu(gate(x)) * up(x))."""

    def __init__(self, gate, up, down):
        super().__init__()
        self.gate_proj = torch.nn.Linear(gate.shape[1], gate.shape[0], bias=False, dtype=BF16)
        self.up_proj = torch.nn.Linear(up.shape[1], up.shape[0], bias=False, dtype=BF16)
        self.down_proj = torch.nn.Linear(down.shape[1], down.shape[0], bias=False, dtype=BF16)
        with torch.no_grad():
            self.gate_proj.weight.copy_(gate)
            self.up_proj.weight.copy_(up)
            self.down_proj.weight.copy_(down)

    def forward(self, x):
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


def shared_weights(seed: int = 20, h: int = H, i: int = I) -> dict:
    g = gen(seed)
    return {
        "gate": (torch.randn(i, h, generator=g) * 0.02).to(BF16),
        "up": (torch.randn(i, h, generator=g) * 0.02).to(BF16),
        "down": (torch.randn(h, i, generator=g) * 0.02).to(BF16),
    }


def shared_mlp(seed: int = 20) -> SharedMLP:
    w = shared_weights(seed)
    return SharedMLP(w["gate"], w["up"], w["down"])


def shared_gate_weight(seed: int = 21, h: int = H) -> torch.Tensor:
    return (torch.randn(1, h, generator=gen(seed)) * 0.02).to(BF16)


def shared_gate_linear(seed: int = 21) -> torch.nn.Linear:
    w = shared_gate_weight(seed)
    lin = torch.nn.Linear(w.shape[1], 1, bias=False, dtype=BF16)
    with torch.no_grad():
        lin.weight.copy_(w)
    return lin


def router256(seed: int = 30, e: int = E_ALL, h: int = H) -> torch.Tensor:
    return (torch.randn(e, h, generator=gen(seed)) * 0.02).to(BF16)


def zipf_bias(seed: int, e: int = E_ALL, s: float = 1.1) -> torch.Tensor:
    """Per-expert logit bias b_e = -s * ln(rank_e), rank a seeded permutation of 1..E."""
    rank = torch.randperm(e, generator=gen(seed)).float() + 1.0
    return -s * torch.log(rank)
