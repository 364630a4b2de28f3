"""Drop-ins for the Drama-3 speaker pieces of the reference engine (engine.py:150-257).

  fp8_block        128x128 block quantiser (engine.py:214-219)
  Speaker          distilled top-k MoE for decode rows (engine.py:222-237), one fused launch
  load_speaker     speaker checkpoint reader (engine.py:240-250)
  attach_speaker   installs a Speaker per layer (engine.py:253-257)
  speaker_forward  SparseMoeBlock.forward for decode rows (engine.py:153-158): the speaker, the
                   shared expert and its sigmoid gate fused into one launch when the shared
                   expert's linears are block-FP8 (the TTS_FP8 configuration, engine.py:201-206)
  install          patches a loaded reference `engine` module to use all of the above
"""

from __future__ import annotations

import torch

from . import ops

BF16 = torch.bfloat16


def fp8_block(w: torch.Tensor):
    """Block quantiser of engine.fp8_block: one fp32 scale = absmax/448 (clamped at 1e-12) per
    128x128 block of the last two dims; q = e4m3(w / scale)."""
    *lead, r, c = w.shape
    b = w.float().view(*lead, r // 128, 128, c // 128, 128)
    scale = b.abs().amax(dim=(-3, -1)).clamp(min=1e-12) / 448.0
    q = (b / scale[..., :, None, :, None]).view(*lead, r, c).to(torch.float8_e4m3fn)
    return q, scale.float()


class Speaker:
    """The distilled speaker MoE of one layer: fp32 router [E, H], fp32 bias [H], block-FP8 experts.

    __call__(x) = (fp8_moe_forward(x, top-k routing of softmax(x.float() @ gate.T)) + bias).bf16,
    computed by one dm3::moe_layer launch per 4 rows (engine.py:232-237)."""

    top_k = 8

    def __init__(self, p: dict, device="cuda"):
        self.gate = p["gate"].to(device).float().contiguous()
        self.bias = p["bias"].to(device).float().contiguous()
        if "s13" in p:
            self.w13, self.s13, self.w2, self.s2 = (p[k].to(device) for k in ("w13", "s13", "w2", "s2"))
        else:
            self.w13, self.s13 = fp8_block(p["w13"].to(device))
            self.w2, self.s2 = fp8_block(p["w2"].to(device))
        H, I = self.w13.shape[2], self.w13.shape[1] // 2
        ops.moe_workspace(self.gate.device, H, I)  # created now so CUDA-graph capture never allocates it

    def route_and_combine(self, x: torch.Tensor, shared=None):
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


def load_speaker(path):
    """Per-layer speaker tensors from a .pt list or a safetensors file keyed
    `layers.{i}.{selected,gate,bias,w13,s13,w2,s2}` (engine.py:240-250)."""
    if not str(path).endswith(".safetensors"):
        return torch.load(path, mmap=True)
    from safetensors.torch import load_file

    flat, layers = load_file(path), []
    for key, t in flat.items():
        i, name = key.split(".", 2)[1:]
        layers += [{} for _ in range(int(i) + 1 - len(layers))]
        layers[int(i)][name] = t
    return layers


def attach_speaker(model, path):
    """One Speaker per decoder layer (engine.py:253-257)."""
    for layer, p in zip(model.backbone.model.layers, load_speaker(path)):
        layer.mlp.experts.speaker = Speaker(p)
        if "reader" in p:
            layer.mlp.experts.reader = Speaker(p["reader"])


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
    OnDemandExperts.forward), Speaker, fp8_block, load/attach_speaker and the patched
    SparseMoeBlock.forward. FP8 dense layers come from `drama3_b200.fp8_linear.convert`."""
    from . import fp8_moe

    engine.fp8_moe_forward = fp8_moe.fp8_moe_forward
    engine.fp8_block = fp8_block
    engine.Speaker = Speaker
    engine.load_speaker = load_speaker
    engine.attach_speaker = attach_speaker
    fwd = make_speaker_forward(engine.routed_forward, lambda: engine.OnDemandExperts.batch)
    engine.speaker_forward = fwd
    engine.SparseMoeBlock.forward = fwd
