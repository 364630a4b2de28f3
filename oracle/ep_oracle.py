"""Expert-parallel restatement of the prefill MoE layer on CPU ranks (TEST INFRASTRUCTURE ONLY).

Only tests/ may use this module, as the checker of the expert-parallel algorithm that the
drama3_b200 kernels implement over NVLink: rank r of `world` owns the experts
[r * E / world, (r + 1) * E / world) and routes its own tokens (the router of
exp1_routing.py:59-60 / engine.py:233-235, restated in moe_oracle.route); every (token, k) pair
travels to its expert's owner, which evaluates fp8_moe_forward's per-pair product
(exp3_distill.py:38-45, restated in moe_oracle.moe_forward) and sends the output row back; the
source combines its tokens in k order, adds the bias and the gated shared expert (engine.py:158,
:236-237). The exchange runs over torch.distributed (gloo) all_to_all, so the same per-rank code
runs as real processes.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .moe_oracle import BF16, _bf16, _silu, dequant, route, shared_expert, shared_gate


def owner(e: int, n_experts: int, world: int) -> int:
    return e // (n_experts // world)


def _exchange(send: list, world: int, width: int) -> list:
    """all_to_all of per-destination [n_d, width] float64 blocks of varying n_d."""
    counts = torch.tensor([b.shape[0] for b in send], dtype=torch.int64)
    rcounts = torch.empty(world, dtype=torch.int64)
    dist.all_to_all_single(rcounts, counts)
    m = torch.tensor([int(max(int(counts.max()), 1))], dtype=torch.int64)
    dist.all_reduce(m, op=dist.ReduceOp.MAX)  # one block height for every rank
    m = int(m.item())
    inp = torch.zeros(world * m, width, dtype=torch.float64)
    for d, b in enumerate(send):
        inp[d * m: d * m + b.shape[0]] = torch.from_numpy(b)
    out = torch.empty_like(inp)
    dist.all_to_all_single(out, inp)
    return [out[s * m: s * m + int(rcounts[s])].numpy() for s in range(world)]


def ep_rank_layer(x_local: torch.Tensor, gate: torch.Tensor, experts_local: dict, n_experts: int, top_k: int,
                  logit_bias=None, sw=None, g=None, srows: int = 128):
    """This rank's part of the layer (call on every rank of the default group). experts_local
    holds w13 / s13 / w2 / s2 of this rank's experts in local index order. Returns
    (y bf16 [T, H], ids, weights)."""
    world, rank = dist.get_world_size(), dist.get_rank()
    el = n_experts // world
    ids, w = route(x_local, gate, top_k, logits_bf16=True, logit_bias=logit_bias)
    t, h = x_local.shape
    xd = x_local.float().numpy().astype(np.float64)
    idn = ids.numpy()
    # send every pair (local expert, source pair index, the token's row) to its expert's owner
    send = [[] for _ in range(world)]
    for i in range(t * top_k):
        e = int(idn.reshape(-1)[i])
        d = owner(e, n_experts, world)
        send[d].append(np.concatenate([[e - d * el, i], xd[i // top_k]]))
    blocks = [np.array(b, dtype=np.float64).reshape(-1, h + 2) for b in send]
    recv = _exchange(blocks, world, h + 2)
    # this rank's experts over the pairs it received
    W13 = [dequant(experts_local["w13"][e], experts_local["s13"][e], srows) for e in range(el)]
    W2 = [dequant(experts_local["w2"][e], experts_local["s2"][e], srows) for e in range(el)]
    back = []
    for s in range(world):
        rows = []
        for r in recv[s]:
            e = int(r[0])
            gu = r[2:] @ W13[e].T
            i = gu.shape[0] // 2
            hh = _bf16(_silu(gu[:i]) * gu[i:])
            rows.append(np.concatenate([[r[1]], hh @ W2[e].T]))
        back.append(np.array(rows, dtype=np.float64).reshape(-1, h + 1))
    ret = _exchange(back, world, h + 1)
    out_rows = np.zeros((t * top_k, h), dtype=np.float64)
    for s in range(world):
        for r in ret[s]:
            out_rows[int(r[0])] = r[1:]
    wn = w.float().numpy().astype(np.float64)
    y = np.zeros((t, h), dtype=np.float64)
    for tok in range(t):
        for j in range(top_k):
            y[tok] += out_rows[tok * top_k + j] * wn[tok, j]
    y = torch.from_numpy(y).float().to(BF16)
    if sw is not None:
        sg = shared_gate(x_local, g) if g is not None else torch.ones(t, dtype=BF16)
        sh = shared_expert(x_local, sw)
        y = (y.float() + (sg.float()[:, None] * sh.float()).to(BF16).float()).to(BF16)
    return y, ids, w
