"""Drop-in for the audio-head lines of the reference's CUDA-graph decode step (CfgGraphs.run,
engine.py:409-411, :423-424, :428) and its direction_score (engine.py:476-479).

    head = AudioHead(model.backbone.lm_head.weight, candidates, vocab_size)   # once
    guided, logits = head(hidden, strength)          # replaces the GEMV, index_copy and its buffer
    head.score_into(score, sample[0, 0], eos_id, semantic_begin)   # replaces score.add_(direction_score)

The head rows (eos + the semantic band) are quantised once to block-FP8 (1x128 scales, the
FP8Linear layout), so each frame reads 8.4 MB instead of the bf16 copy's 16.8 MB; logits are rounded
to bf16 like the reference's bf16 matmul before the fp32 guidance.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .fp8_linear import quantize


class AudioHead:
    """The candidate rows of the LM head in block-FP8 plus the persistent -inf vocabulary buffer."""

    def __init__(self, lm_head_weight: Optional[torch.Tensor], candidates: torch.Tensor, vocab_size: int,
                 q: Optional[torch.Tensor] = None, s: Optional[torch.Tensor] = None,
                 rows: Optional[torch.Tensor] = None):
        dev = candidates.device
        self.candidates = candidates.to(torch.int64).contiguous()
        self.rows = None if rows is None else rows.to(device=dev, dtype=torch.int64).contiguous()
        if q is None:
            w = lm_head_weight[self.candidates] if rows is None else lm_head_weight
            q, s = quantize(w.to(dev))
        self.q, self.s = q.contiguous(), s.contiguous()
        # CfgGraphs.logits: [1, vocab] of -inf; only the candidate columns are ever rewritten
        self.vocab = torch.full((1, vocab_size), -torch.inf, dtype=torch.float32, device=dev)
        self.logits = self.lse = None

    def __call__(self, hidden: torch.Tensor, strength: torch.Tensor):
        """Returns (guided [1, vocab] fp32, logits [2, Nc] fp32) for hidden [2, K]."""
        self.logits, self.lse = ops.audio_head(hidden, self.q, self.s, strength, self.candidates,
                                               self.vocab.view(-1), self.rows, True)
        return self.vocab, self.logits

    def score_into(self, score: torch.Tensor, token: torch.Tensor, eos_id: int, semantic_begin: int) -> None:
        """score += direction_score(logits, token) of the last call (device-side, no host sync)."""
        ops.direction_score(self.logits, self.lse, token.reshape(1).to(torch.int64), eos_id, semantic_begin, score)
