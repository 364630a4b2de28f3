"""HBM-resident routed-expert table read from the Drama-3 checkpoint.

The reference pages experts into an LRU of GPU slots on demand (ExpertStore, engine.py:26-125,
with NVMe streaming in disk.py) because its 30 GiB of block-FP8 experts do not fit a 16 GB card.
A B200 holds them all, so here every layer's experts live in HBM for the whole run, in the
ExpertStore slot layout (engine.py:32-36): per expert one uint8 row of 3 * I * H bytes holding
w13 = [gate; up] as [2I, H] followed by w2 = down as [I -> H] [H, I], plus fp32 block scales
s13 [2I / 128, H / 128] and s2 [H / 128, I / 128]. The slot of expert e is e, so the reference's
ids.unique() / slot_map / host synchronisation per layer (engine.py:143-146) disappears: the
fused kernels take the router's ids directly, with the slot stride 3 * I * H.

Checkpoint keys (checkpoint.py:21-23, :89-96): `model.language_model.layers.{l}.mlp.experts.{e}.
{gate_proj,up_proj,down_proj}.{weight,weight_scale_inv}`; weights e4m3 [I, H] / [H, I], scales
fp32 with one value per 128x128 block. Shards are read through `model.safetensors.index.json`
(or a single .safetensors file).
"""

from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Dict, Iterable, Iterator, List, Optional, Tuple

import torch
import torch.nn as nn

from .fp8_moe import fp8_moe_forward

FP8 = torch.float8_e4m3fn
CHECKPOINT_PREFIX = "model.language_model."
_EXPERT_KEY = re.compile(r"layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\.(weight|weight_scale_inv)")
_PROJ = ("gate_proj", "up_proj", "down_proj")
_KIND = ("weight", "weight_scale_inv")


def _shard_files(source: Path) -> List[Path]:
    """Shard files of a checkpoint directory (via its index) or a single safetensors file."""
    if source.is_file():
        return [source]
    index = source / "model.safetensors.index.json"
    if index.exists():
        names = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        return [source / n for n in names]
    files = sorted(source.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"{source}: no model.safetensors.index.json and no .safetensors files")
    return files


def read_expert_checkpoint(source, prefix: str = CHECKPOINT_PREFIX,
                           layers: Optional[Iterable[int]] = None) -> Iterator[Tuple[int, int, str, str, torch.Tensor]]:
    """Yields (layer, expert, projection, kind, CPU tensor) for every routed-expert tensor of the
    checkpoint, optionally limited to some layers. Other keys are skipped."""
    from safetensors import safe_open

    wanted = None if layers is None else set(int(l) for l in layers)
    for path in _shard_files(Path(source)):
        with safe_open(str(path), framework="pt") as f:
            for key in f.keys():
                if not key.startswith(prefix):
                    continue
                m = _EXPERT_KEY.fullmatch(key[len(prefix):])
                if m is None:
                    continue
                layer = int(m.group(1))
                if wanted is not None and layer not in wanted:
                    continue
                yield layer, int(m.group(2)), m.group(3), m.group(4), f.get_tensor(key)


class ExpertTable:
    """Every routed expert of `n_layers` layers resident on one device in the slot layout.

    buf [L, E, 3 I H] uint8; s13 [L, E, 2I / 128, H / 128] fp32; s2 [L, E, H / 128, I / 128] fp32.
    `layer(l)` returns (w13, s13, w2, s2) views for fp8_moe_forward with dim-0 stride 3 I H bytes."""

    def __init__(self, n_layers: int, n_experts: int, hidden: int, intermediate: int, device="cuda"):
        if hidden % 128 or intermediate % 128:
            raise ValueError("hidden and intermediate sizes must be multiples of 128")
        self.n_layers, self.n_experts, self.hidden, self.intermediate = n_layers, n_experts, hidden, intermediate
        self.device = torch.device(device)
        H, I = hidden, intermediate
        self.slot_bytes = 3 * I * H
        self.buf = torch.zeros((n_layers, n_experts, self.slot_bytes), dtype=torch.uint8, device=self.device)
        self.s13 = torch.zeros((n_layers, n_experts, 2 * I // 128, H // 128), dtype=torch.float32, device=self.device)
        self.s2 = torch.zeros((n_layers, n_experts, H // 128, I // 128), dtype=torch.float32, device=self.device)
        self._filled = torch.zeros((n_layers, n_experts, 3, 2), dtype=torch.bool)

    def layer(self, l: int):
        """(w13 e4m3 [E, 2I, H], s13, w2 e4m3 [E, H, I], s2) of layer l, views into the table."""
        H, I, E = self.hidden, self.intermediate, self.n_experts
        row = self.buf[l]
        w13 = row[:, : 2 * I * H].view(E, 2 * I, H).view(FP8)
        w2 = row[:, 2 * I * H:].view(E, H, I).view(FP8)
        return w13, self.s13[l], w2, self.s2[l]

    def _target(self, l: int, e: int, proj: str, kind: str) -> torch.Tensor:
        H, I = self.hidden, self.intermediate
        if kind == "weight":
            w13, _, w2, _ = self.layer(l)
            if proj == "down_proj":
                return w2[e]
            return w13[e, :I] if proj == "gate_proj" else w13[e, I:]
        half = I // 128
        if proj == "down_proj":
            return self.s2[l, e]
        return self.s13[l, e, :half] if proj == "gate_proj" else self.s13[l, e, half:]

    def put(self, l: int, e: int, proj: str, kind: str, t: torch.Tensor) -> None:
        """Copies one checkpoint tensor into its place (shape and dtype checked)."""
        if not (0 <= l < self.n_layers and 0 <= e < self.n_experts):
            raise ValueError(f"expert ({l}, {e}) is outside a table of {self.n_layers} x {self.n_experts}")
        dst = self._target(l, e, proj, kind)
        if tuple(t.shape) != tuple(dst.shape):
            raise ValueError(f"layer {l} expert {e} {proj}.{kind}: shape {tuple(t.shape)}, expected {tuple(dst.shape)}")
        if kind == "weight" and t.dtype not in (FP8, torch.uint8):
            raise ValueError(f"layer {l} expert {e} {proj}.weight: dtype {t.dtype}, expected float8_e4m3fn")
        dst.copy_(t.view(FP8) if t.dtype == torch.uint8 else (t.float() if kind != "weight" else t))
        self._filled[l, e, _PROJ.index(proj), _KIND.index(kind)] = True

    def missing(self) -> List[Tuple[int, int, str, str]]:
        """(layer, expert, projection, kind) of every tensor not yet loaded."""
        idx = torch.nonzero(~self._filled).tolist()
        return [(l, e, _PROJ[p], _KIND[k]) for l, e, p, k in idx]

    def load(self, source, prefix: str = CHECKPOINT_PREFIX, first_layer: int = 0) -> "ExpertTable":
        """Fills the table from a checkpoint (directory with an index, or one safetensors file): table
        layer l takes checkpoint layer first_layer + l. Raises if any expert tensor is missing."""
        layers = range(first_layer, first_layer + self.n_layers)
        for l, e, proj, kind, t in read_expert_checkpoint(source, prefix, layers):
            self.put(l - first_layer, e, proj, kind, t)
        gone = self.missing()
        if gone:
            raise ValueError(f"{len(gone)} expert tensors missing from {source}, e.g. {gone[:3]}")
        return self

    @classmethod
    def from_checkpoint(cls, source, n_layers: int, n_experts: int, hidden: int, intermediate: int,
                        device="cuda", prefix: str = CHECKPOINT_PREFIX) -> "ExpertTable":
        return cls(n_layers, n_experts, hidden, intermediate, device).load(source, prefix)


class ResidentExperts(nn.Module):
    """OnDemandExperts.forward (engine.py:138-147) over an ExpertTable: the same speaker / reader
    short cuts, then fp8_moe_forward on the layer's resident experts with the router's ids as slots.

    `batch` and `light` play the roles of OnDemandExperts.batch / .light."""

    batch = 1
    light = False

    def __init__(self, layer: int, table: ExpertTable):
        super().__init__()
        self.layer, self.table = layer, table
        self.speaker = self.reader = None

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        if self.speaker is not None and x.shape[0] <= ResidentExperts.batch:
            return self.speaker(x)
        if self.reader is not None and ResidentExperts.light:
            return self.reader(x)
        w13, s13, w2, s2 = self.table.layer(self.layer)
        return fp8_moe_forward(x, ids, weights, w13, s13, w2, s2)


def attach_expert_table(layers: Iterable[nn.Module], table: ExpertTable) -> Dict[int, ResidentExperts]:
    """Replaces `layer.mlp.experts` of each decoder layer by a ResidentExperts over the table,
    keeping any speaker / reader already attached. Returns the new modules by layer index."""
    out = {}
    for i, layer in enumerate(layers):
        old = layer.mlp.experts
        new = ResidentExperts(i, table)
        new.speaker, new.reader = getattr(old, "speaker", None), getattr(old, "reader", None)
        layer.mlp.experts = new
        out[i] = new
    return out
