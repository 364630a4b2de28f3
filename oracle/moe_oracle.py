"""CPU restatement of the reference's MoE feed-forward / block-FP8 GEMV arithmetic.

TEST INFRASTRUCTURE ONLY: this module is the parity checker for the CUDA path; the shipped
package never imports it.

Each function names the reference lines it restates. Floating-point products and sums are
taken in float64 (numpy) and rounded where the reference rounds (fp32 logits, bf16 activations
and outputs), so the oracle is at least as accurate as the reference's own fp32 path; casts to
bf16 / float8_e4m3fn use torch's CPU conversions (round to nearest even), as the reference does.
"""

from __future__ import annotations

import numpy as np
import torch

BLOCK = 128  # fp8_linear.py:7
FP8_MAX = 448.0  # largest e4m3 magnitude: engine.py:217, fp8_linear.py:33

BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn


# ----------------------------------------------------------------------------- quantisers
def fp8_block(w: torch.Tensor):
    """128x128 block quantiser, engine.py:214-219 (also release/convert_weights.py:14-15).

    scale = absmax(block) / 448 (clamped at 1e-12), q = e4m3(w / scale), both per block of
    128 rows x 128 columns of the last two dims.
    """
    *lead, r, c = w.shape
    b = w.float().reshape(*lead, r // BLOCK, BLOCK, c // BLOCK, BLOCK)
    scale = b.abs().amax(dim=(-3, -1)).clamp(min=1e-12) / FP8_MAX
    q = (b / scale[..., :, None, :, None]).reshape(*lead, r, c).to(E4M3)
    return q, scale.float()


def quantize_rows(w: torch.Tensor):
    """1x128 quantiser of fp8_linear.quantize (fp8_linear.py:30-34): one scale per output row
    and 128-wide K block, s[N, K / 128]."""
    n, k = w.shape
    b = w.float().reshape(n, k // BLOCK, BLOCK)
    s = b.abs().amax(-1).clamp(min=1e-12) / FP8_MAX
    return (b / s[..., None]).reshape(n, k).to(E4M3), s.contiguous()


def dequant(q: torch.Tensor, s: torch.Tensor, srows: int) -> np.ndarray:
    """float(q) * scale for one weight [R, C] with scales [ceil(R / srows), C / 128] (float64).

    srows = 1 is fp8_linear.dequantize (fp8_linear.py:37-39); srows = 128 is the inverse of
    engine.fp8_block."""
    r, c = q.shape
    qf = q.float().numpy().astype(np.float64)
    sf = s.float().numpy().astype(np.float64)
    rows = np.arange(r) // srows
    sc = np.repeat(sf[rows], BLOCK, axis=1)[:, :c]
    return qf * sc


# ----------------------------------------------------------------------------- GEMV
def gemv(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, srows: int = 1, bias=None, out_dtype=BF16):
    """Block-FP8 GEMV of the Triton `_gemv` (fp8_linear.py:15-27): for each 128-wide K block the
    product x[:, kb] . q[n, kb] is scaled by s[n, kb] and accumulated; output in x's dtype
    (fp8_linear.py:57), + bias (fp8_linear.py:62-63)."""
    xd = x.float().numpy().astype(np.float64)
    y = xd @ dequant(q, s, srows).T
    out = torch.from_numpy(y).float()
    if bias is not None:
        out = out + bias.float()
    return out.to(out_dtype)


def linear_dequant(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, srows: int = 1, bias=None):
    """FP8Linear.forward for more than 2 rows (fp8_linear.py:60-63): the weight dequantised
    (float(q) * scale), cast to x's dtype (bf16), then F.linear in bf16 (products summed exactly
    here, rounded once to bf16), + bias in bf16."""
    w = torch.from_numpy(dequant(q, s, srows)).float().to(BF16).double().numpy()
    y = x.float().numpy().astype(np.float64) @ w.T
    out = torch.from_numpy(y).float().to(BF16)
    if bias is not None:
        out = out + bias.to(BF16)
    return out


# ----------------------------------------------------------------------------- routing
def router_logits(x: torch.Tensor, gate: torch.Tensor, logits_bf16: bool, logit_bias=None) -> torch.Tensor:
    """fp32 logits x.float() @ gate.T (engine.py:233; exp3_distill.py:36), taken exactly (float64)
    and rounded once to fp32. logits_bf16 rounds them to bf16 as a bf16 nn.Linear router does
    (the 256-expert gate whose output exp1_routing.py:54 captures). logit_bias (fp32) is added
    after rounding."""
    xd = x.float().numpy().astype(np.float64)
    gd = gate.float().numpy().astype(np.float64)
    logits = torch.from_numpy(xd @ gd.T).float()
    if logits_bf16:
        logits = logits.to(BF16).float()
    if logit_bias is not None:
        logits = logits + logit_bias.float()
    return logits


def route(x: torch.Tensor, gate: torch.Tensor, top_k: int = 8, logits_bf16: bool = False, logit_bias=None):
    """softmax -> top-k -> renormalise -> bf16, engine.py:233-235 (exp3_distill.py:36-37,
    exp1_routing.py:59-60).

    Selection order: descending logit, ties to the lower expert index (softmax is monotonic, so
    this is the order of descending probability). Returns (ids int64 [T, k], w bf16 [T, k])."""
    logits = router_logits(x, gate, logits_bf16, logit_bias)
    probs = torch.softmax(logits, -1)
    ln = logits.numpy()
    t, e = ln.shape
    ids = np.empty((t, top_k), dtype=np.int64)
    for i in range(t):
        order = np.lexsort((np.arange(e), -ln[i].astype(np.float64)))
        ids[i] = order[:top_k]
    ids_t = torch.from_numpy(ids)
    w = torch.gather(probs, 1, ids_t)
    w = (w / w.sum(-1, keepdim=True)).to(BF16)
    return ids_t, w


def permutation(ids: torch.Tensor, n_experts: int):
    """Token-to-expert dispatch order: the flattened (token, k) pairs stably sorted by expert,
    i.e. argsort(ids.flatten(), stable=True), with per-expert offsets [E + 1]. This is the grouping
    the reference's routed path performs per expert (`(ids == e).nonzero()` in expert order,
    exp3_distill.py:39-40; `ids.unique()` in OnDemandExperts.forward, engine.py:143)."""
    flat = ids.reshape(-1).numpy()
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return torch.from_numpy(order.astype(np.int64)), torch.from_numpy(offsets)


# ----------------------------------------------------------------------------- MoE
def _silu(v: np.ndarray) -> np.ndarray:
    return v / (1.0 + np.exp(-v))


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(a).float().to(BF16).float().numpy().astype(np.float64)


def moe_forward(x, ids, weights, w13, s13, w2, s2, srows: int = 128, expert_cache=None):
    """fish-speech `fp8_moe_forward(x, ids, w, w13, s13, w2, s2)` (called at engine.py:147, :236),
    restated after exp3_distill.SpeakerMoE.forward (exp3_distill.py:38-45): for each expert e in
    ascending order, rows (t, j) with ids[t, j] == e; g, up = (x[t] @ W13[e].T).chunk(2)
    (w13 rows 0..I-1 gate, I..2I-1 up: engine.py:84-89); h = silu(g) * up, rounded to bf16;
    out[t] += weights[t, j] * (h @ W2[e].T). Weights are block-FP8 dequantised (float(q) * scale).
    Output bf16 [T, H]."""
    xd = x.float().numpy().astype(np.float64)
    idn = ids.numpy()
    wn = weights.float().numpy().astype(np.float64)
    t, h = xd.shape
    out = np.zeros((t, h), dtype=np.float64)
    for e in np.unique(idn):
        rows, cols = np.nonzero(idn == e)
        if expert_cache is not None and int(e) in expert_cache:
            W13, W2 = expert_cache[int(e)]
        else:
            W13 = dequant(w13[e], s13[e], srows)
            W2 = dequant(w2[e], s2[e], srows)
            if expert_cache is not None:
                expert_cache[int(e)] = (W13, W2)
        gu = xd[rows] @ W13.T
        i = gu.shape[1] // 2
        hh = _bf16(_silu(gu[:, :i]) * gu[:, i:])
        y = hh @ W2.T
        np.add.at(out, rows, y * wn[rows, cols][:, None])
    return torch.from_numpy(out).float().to(BF16)


def speaker(x, p: dict, top_k: int = 8, srows: int = 128):
    """engine.Speaker.__call__ (engine.py:232-237): fp32 router over the distilled experts,
    softmax / top-k / renormalise to bf16, fp8_moe_forward, then (y.float() + bias).to(bf16).
    p holds gate [E, H] fp32, bias [H] fp32, w13/s13/w2/s2 (block-FP8, engine.py:226-230)."""
    ids, w = route(x, p["gate"].float(), top_k, logits_bf16=False)
    y = moe_forward(x, ids, w, p["w13"], p["s13"], p["w2"], p["s2"], srows)
    return (y.float() + p["bias"].float()).to(BF16), ids, w


def shared_expert(x, sw: dict):
    """The always-on shared expert as bf16 nn.Linear modules (a Qwen-style MLP: down(silu(gate(x))
    * up(x)); every linear output and the elementwise product rounded to bf16. sw holds either bf16
    `gate`/`up`/`down` [out, in] weights, or block-FP8 ones as (q, s, srows) tuples."""
    xd = x.float().numpy().astype(np.float64)

    def lin(inp, name):
        v = sw[name]
        wmat = dequant(*v) if isinstance(v, tuple) else v.float().numpy().astype(np.float64)
        return _bf16(inp @ wmat.T)

    g = lin(xd, "gate")
    u = lin(xd, "up")
    a = _bf16(_bf16(_silu(g)) * u)
    return torch.from_numpy(lin(a, "down")).float().to(BF16)


def shared_gate(x, g: torch.Tensor):
    """sigmoid(shared_expert_gate(x)) with a bf16 [1, H] linear (engine.py:158): bf16 logit,
    sigmoid in fp32, rounded to bf16."""
    xd = x.float().numpy().astype(np.float64)
    logit = torch.from_numpy(xd @ g.float().reshape(-1).numpy().astype(np.float64)).float().to(BF16)
    return torch.sigmoid(logit.float()).to(BF16)


def speaker_forward(x, p: dict, sw: dict, g: torch.Tensor, top_k: int = 8, srows: int = 128):
    """engine.speaker_forward for decode rows (engine.py:153-158):
    speaker(x) + sigmoid(shared_expert_gate(x)) * shared_expert(x), in bf16 tensor arithmetic."""
    y, ids, w = speaker(x, p, top_k, srows)
    sg = shared_gate(x, g)
    sh = shared_expert(x, sw)
    prod = (sg.float()[:, None] * sh.float()).to(BF16)
    return (y.float() + prod.float()).to(BF16), ids, w


def moe_layer(x, gate, experts: dict, top_k=8, logits_bf16=True, logit_bias=None, sw=None, g=None,
              out_bias=None, srows=128, expert_cache=None):
    """One MoE feed-forward decode row set: router (bf16 256-wide gate by default) -> top-k ->
    fp8_moe_forward over the routed experts, + bias, + sigmoid-gated shared expert, each sum
    rounded to bf16 like the reference's tensor ops (engine.py:153-158, :232-237)."""
    ids, w = route(x, gate, top_k, logits_bf16=logits_bf16, logit_bias=logit_bias)
    y = moe_forward(x, ids, w, experts["w13"], experts["s13"], experts["w2"], experts["s2"], srows,
                    expert_cache=expert_cache)
    if out_bias is not None:
        y = (y.float() + out_bias.float()).to(BF16)
    if sw is not None:
        sg = shared_gate(x, g) if g is not None else torch.ones(x.shape[0], dtype=BF16)
        sh = shared_expert(x, sw)
        y = (y.float() + (sg.float()[:, None] * sh.float()).to(BF16).float()).to(BF16)
    return y, ids, w


# ----------------------------------------------------------------------------- audio head
def audio_head(hidden, q, s, srows: int, candidates, vocab_size: int, strength: float):
    """CfgGraphs.run's head lines (engine.py:423-424) with the block-FP8 head: logits = the head GEMV
    in the activations' dtype (bf16, as the Triton `_gemv` or the bf16 matmul returns), .float();
    guided = a [1, vocab] -inf buffer with the candidate columns set to l1 + strength * (l0 - l1)
    (fp32, torch's own ops). Returns (logits fp32 [2, Nc], guided fp32 [1, vocab])."""
    logits = gemv(hidden, q, s, srows).float()
    st = torch.tensor(strength, dtype=torch.float32)
    guided = torch.full((1, vocab_size), -torch.inf).index_copy(1, candidates, logits[1:] + st * (logits[:1] - logits[1:]))
    return logits, guided


def direction_score(logits, token: int, eos_id: int, semantic_begin: int):
    """engine.direction_score (engine.py:476-479): log-softmax of both rows at the sampled token's
    column (0 for eos, else token - semantic_begin + 1), conditional minus unconditional."""
    index = 0 if token == eos_id else token - semantic_begin + 1
    picked = torch.log_softmax(logits.float(), dim=-1)[:, index]
    return (picked[0] - picked[1]).reshape(())
