"""Shared test utilities (tolerances and seeded weight builders)."""

import torch

# Output tolerance of the north-star contract: relative L2 error <= 2e-2 against the oracle
# (bf16 activations, fp32 accumulation). Indices and permutations must match exactly.
REL_L2_TOL = 2e-2


def rel_l2(a, b) -> float:
    a = a.detach().float().cpu()
    b = b.detach().float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def experts(e: int, h: int, i: int, seed: int, srows: int = 128):
    """Seeded block-FP8 experts: w13 [E, 2I, H], w2 [E, H, I] from N(0, 0.02), quantised with
    128x128 (srows=128) or 1x128 (srows=1) scales."""
    import oracle

    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(e, 2 * i, h, generator=g) * 0.02
    w2 = torch.randn(e, h, i, generator=g) * 0.02
    if srows == 128:
        q13, s13 = oracle.fp8_block(w13)
        q2, s2 = oracle.fp8_block(w2)
    else:
        qs = [oracle.quantize_rows(w) for w in w13]
        q13, s13 = torch.stack([a for a, _ in qs]), torch.stack([b for _, b in qs])
        qs = [oracle.quantize_rows(w) for w in w2]
        q2, s2 = torch.stack([a for a, _ in qs]), torch.stack([b for _, b in qs])
    return {"w13": q13, "s13": s13, "w2": q2, "s2": s2}


def to_dev(d: dict, dev="cuda"):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def routed_layer(seed, srows=128, shared=True, h=2048, i=512, e=256):
    """Seeded routed layer: block-FP8 experts, a bf16 router and optionally a shared expert
    with its bf16 gate row."""
    from tests.golden import inputs

    ex = experts(e, h, i, seed=seed, srows=srows)
    gate = inputs.router256(seed + 1, e=e, h=h)
    out = {"experts": ex, "gate": gate}
    if shared:
        sw = experts(1, h, i, seed=seed + 2, srows=srows)
        out["sh"] = {k: v[0] for k, v in sw.items()}
        out["sh_gate"] = inputs.shared_gate_weight(seed + 3, h=h)
    return out


def oracle_shared(layer, srows):
    """The shared expert as the oracle's (q, s, srows) gate / up / down triples."""
    sh = layer["sh"]
    i = sh["w2"].shape[1]
    k = i // srows  # scale rows covering the gate half of w13
    return {"gate": (sh["w13"][:i], sh["s13"][:k], srows), "up": (sh["w13"][i:], sh["s13"][k:], srows),
            "down": (sh["w2"], sh["s2"], srows)}
