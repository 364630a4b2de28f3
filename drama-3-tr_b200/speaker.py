"""Drop-ins for the Drama-3 speaker pieces of the reference engine (engine.py:150-257).

  fp8_block          128x128 block quantiser (engine.py:214-219); byte-identical output
  Speaker            distilled top-k MoE for decode rows (engine.py:222-237), one fused launch
  read_speaker_file  reader of the speaker checkpoint written by release/convert_weights.py
                     (`layers.{i}.{selected,gate,bias,w13,s13,w2,s2}`) or of the .pt list
  speakers_from_file kernel-ready Speaker objects, one per layer, straight from such a file
  speaker_forward    SparseMoeBlock.forward for decode rows (engine.py:153-158): the speaker, the
                     shared expert and its sigmoid gate fused into one launch when the shared
                     expert's linears are block-FP8 (the TTS_FP8 configuration, engine.py:201-206)
  install            points a loaded reference `engine` module at all of the above

The reference's own load_speaker / attach_speaker (engine.py:240-257) look up `Speaker` in their
module, so after `install(engine)` they build these Speaker objects without being replaced.
"""

from __future__ import annotations

import re
from pathlib import Path
from typing import Dict, List, Optional

import torch

from . import ops

BF16 = torch.bfloat16
FP8 = torch.float8_e4m3fn

# tensors of one speaker layer in the release file (release/convert_weights.py:14-18)
SPEAKER_TENSORS = ("selected", "gate", "bias", "w13", "s13", "w2", "s2")
_SPEAKER_KEY = re.compile(r"layers\.(\d+)\.(\w+)")


def fp8_block(w: torch.Tensor):
    """e4m3 q and fp32 scales with one scale = max(absmax, 1e-12) / 448 per 128x128 block of the
    last two dims, scales shaped [..., R / 128, C / 128]."""
    *lead, rows, cols = w.shape
    tiles = w.float().reshape(*lead, rows // 128, 128, cols // 128, 128)
    scale = tiles.abs().amax(dim=(-3, -1)).clamp(min=1e-12) / 448.0
    q = (tiles / scale.unsqueeze(-1).unsqueeze(-3)).reshape(*lead, rows, cols).to(FP8)
    return q, scale.float()


class Speaker:
    """The distilled speaker MoE of one layer: fp32 router [E, H], fp32 bias [H], block-FP8 experts.

    __call__(x) = (fp8_moe_forward(x, top-k routing of softmax(x.float() @ gate.T)) + bias).bf16,
    computed by one dm3::moe_layer launch per 4 rows (engine.py:232-237). `p` holds gate, bias and
    either the quantised experts (w13, s13, w2, s2) or bf16 / fp32 w13 and w2, which are quantised
    here with fp8_block."""

    top_k = 8

    def __init__(self, p: Dict[str, torch.Tensor], device="cuda"):
        dev = torch.device(device)
        self.gate = p["gate"].to(device=dev, dtype=torch.float32).contiguous()
        self.bias = p["bias"].to(device=dev, dtype=torch.float32).contiguous()
        w13, w2 = p["w13"].to(dev), p["w2"].to(dev)
        if "s13" in p and "s2" in p:
            as_fp8 = lambda t: t.view(FP8) if t.dtype == torch.uint8 else t  # noqa: E731
            self.w13, self.w2 = as_fp8(w13), as_fp8(w2)
            self.s13, self.s2 = p["s13"].to(dev).float(), p["s2"].to(dev).float()
        else:
            self.w13, self.s13 = fp8_block(w13)
            self.w2, self.s2 = fp8_block(w2)
        hidden, inter = self.w13.shape[2], self.w13.shape[1] // 2
        ops.moe_workspace(dev, hidden, inter)  # created now so CUDA-graph capture never allocates it

    def route_and_combine(self, x: torch.Tensor, shared: Optional["SharedExpert"] = None):
        sh = shared.tensors() if shared is not None else (None, None, None, None, None)
        return ops.moe_layer(x, self.gate, self.top_k, False, None, self.w13, self.s13, self.w2, self.s2, *sh,
                             self.bias)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.route_and_combine(x)[0]


class SharedExpert:
    """A block-FP8 shared expert packed for the fused kernel: w13 = [gate; up] e4m3 [2I, H] with
    scales, w2 = down e4m3 [H, I] with scales, and the bf16 sigmoid-gate row [H]."""

    def __init__(self, w13, s13, w2, s2, gate_row):
        self.w13, self.s13, self.w2, self.s2 = w13.contiguous(), s13.contiguous(), w2.contiguous(), s2.contiguous()
        self.gate_row = None if gate_row is None else gate_row.to(BF16).reshape(-1).contiguous()

    def tensors(self):
        return self.w13, self.s13, self.w2, self.s2, self.gate_row

    @staticmethod
    def from_block(block) -> "SharedExpert | None":
        """Packs block.shared_expert (gate_proj / up_proj / down_proj) if all three are FP8Linear
        (ours or the reference's: both hold q e4m3 [out, in] and 1x128 scales s); None otherwise."""
        se = getattr(block, "shared_expert", None)
        lins = [getattr(se, n, None) for n in ("gate_proj", "up_proj", "down_proj")]
        if not all(hasattr(m, "q") and hasattr(m, "s") for m in lins):
            return None
        if any(getattr(m, "bias", None) is not None for m in lins):
            return None
        g, u, d = lins
        gate_lin = getattr(block, "shared_expert_gate", None)
        if gate_lin is not None and getattr(gate_lin, "bias", None) is not None:
            return None
        gate_row = None if gate_lin is None else gate_lin.weight.detach()
        return SharedExpert(torch.cat([g.q, u.q]), torch.cat([g.s, u.s]), d.q, d.s, gate_row)


def read_speaker_file(path) -> List[Dict[str, torch.Tensor]]:
    """Per-layer speaker tensors (CPU) of a release safetensors file, or the list stored in a .pt file.

    The safetensors keys are `layers.{i}.{name}` with name in SPEAKER_TENSORS; layers must be
    numbered 0..L-1 without gaps. Raises ValueError on any other key."""
    path = Path(path)
    if path.suffix != ".safetensors":
        return list(torch.load(path, mmap=True))
    from safetensors import safe_open

    per_layer: Dict[int, Dict[str, torch.Tensor]] = {}
    with safe_open(str(path), framework="pt") as f:
        for key in f.keys():
            m = _SPEAKER_KEY.fullmatch(key)
            if m is None or m.group(2) not in SPEAKER_TENSORS:
                raise ValueError(f"{path}: unexpected tensor {key!r} in a speaker file")
            per_layer.setdefault(int(m.group(1)), {})[m.group(2)] = f.get_tensor(key)
    if sorted(per_layer) != list(range(len(per_layer))):
        raise ValueError(f"{path}: layers {sorted(per_layer)} are not numbered 0..{len(per_layer) - 1}")
    return [per_layer[i] for i in range(len(per_layer))]


def speakers_from_file(path, device="cuda") -> List[Speaker]:
    """One kernel-ready Speaker per layer of a speaker file, tensors moved to `device`."""
    return [Speaker(p, device=device) for p in read_speaker_file(path)]


def make_speaker_forward(routed_forward, batch):
    """Builds SparseMoeBlock.forward for the reference engine (engine.py:153-158).

    routed_forward: the original SparseMoeBlock.forward (prefill rows); batch(): the current
    OnDemandExperts.batch. Decode rows (<= batch) with a speaker attached run the speaker, the
    shared expert and its sigmoid gate in one fused launch when the shared expert is block-FP8;
    with bf16 shared linears, the speaker runs fused and the shared expert through the block's own
    modules, summed as the reference does."""

    def speaker_forward(self, x):
        flat = x.reshape(-1, x.shape[-1])
        e = self.experts
        if e.speaker is None or flat.shape[0] > batch():
            return routed_forward(self, x)
        sp = e.speaker
        if isinstance(sp, Speaker):
            pack = getattr(self, "_dm3_shared", False)
            if pack is False:
                pack = SharedExpert.from_block(self)
                self._dm3_shared = pack
            if pack is not None:
                return sp.route_and_combine(flat, pack)[0].view_as(x)
        return (sp(flat) + torch.sigmoid(self.shared_expert_gate(flat)) * self.shared_expert(flat)).view_as(x)

    return speaker_forward


def install(engine) -> None:
    """Points a loaded reference `engine` module at the B200 kernels: fp8_moe_forward (used by
    OnDemandExperts.forward), Speaker and fp8_block (so the engine's own load_speaker /
    attach_speaker build fused speakers), and the patched SparseMoeBlock.forward. FP8 dense layers
    come from `drama3_b200.fp8_linear.convert`."""
    from . import fp8_moe

    engine.fp8_moe_forward = fp8_moe.fp8_moe_forward
    engine.fp8_block = fp8_block
    engine.Speaker = Speaker
    fwd = make_speaker_forward(engine.routed_forward, lambda: engine.OnDemandExperts.batch)
    engine.speaker_forward = fwd
    engine.SparseMoeBlock.forward = fwd
