"""The reference's decode MoE layer as its own torch code would run it on host cores (fp32).

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY: bench.py times this as the CPU baseline (`cpu_baseline`,
kind "port", and the `--impl reference` arm). It restates, in torch fp32 on CPU:
  router      bf16 nn.Linear logits -> softmax(fp32) -> topk -> renormalise -> bf16
              (exp1_routing.py:59-60, engine.py:233-235); an fp32 router for the speaker
  experts     fp8_moe_forward restated per exp3_distill.py:38-45, dequantising the touched experts
              on every call as FP8Linear's multi-row path does (fp8_linear.py:61)
  shared      bf16 gate/up/down linears + sigmoid(bf16 gate) (engine.py:158)
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16


def _deq(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """float(q) * scale for a [R, C] weight with 128x128 or 1x128 scales."""
    r, c = q.shape
    srows = 128 if s.shape[0] * 128 >= r and s.shape[0] != r else 1
    sc = s.repeat_interleave(srows, 0)[:r].repeat_interleave(128, 1)[:, :c]
    return q.float() * sc


def decode_layer(x: torch.Tensor, layer: dict, top_k: int = 8) -> torch.Tensor:
    """One MoE layer over rows x [T, H] bf16 on the CPU in torch fp32: 2 decode rows, or the
    hundreds of a prompt (prefill), with an optional per-expert logit bias."""
    gate = layer["gate"]
    logits = F.linear(x, gate) if gate.dtype == BF16 else x.float() @ gate.T  # bf16 / fp32 (speaker) router
    if "logit_bias" in layer:  # the prefill router's per-expert bias, added to the logits before softmax
        logits = logits.float() + layer["logit_bias"]
    probs = torch.softmax(logits.float(), -1)
    w, ids = probs.topk(top_k, -1)
    w = (w / w.sum(-1, keepdim=True)).to(BF16)
    xf = x.float()
    out = torch.zeros_like(xf)
    for e in ids.unique().tolist():
        row, col = (ids == e).nonzero(as_tuple=True)
        w13 = _deq(layer["w13"][e], layer["s13"][e])
        w2 = _deq(layer["w2"][e], layer["s2"][e])
        g, up = (xf[row] @ w13.T).chunk(2, -1)
        h = (F.silu(g) * up).to(BF16).float()
        out.index_add_(0, row, (h @ w2.T) * w[row, col, None].float())
    y = out.to(BF16)
    if "bias" in layer:
        y = (y.float() + layer["bias"]).to(BF16)
    if "sh_w13" in layer:
        i = layer["sh_w2"].shape[1]
        sw13 = _deq(layer["sh_w13"], layer["sh_s13"]).to(BF16)
        sw2 = _deq(layer["sh_w2"], layer["sh_s2"]).to(BF16)
        a = F.silu(F.linear(x, sw13[:i])) * F.linear(x, sw13[i:])
        sh = F.linear(a, sw2)
        y = y + torch.sigmoid(F.linear(x, layer["sh_gate"].reshape(1, -1))) * sh
    return y
