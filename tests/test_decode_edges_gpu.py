"""Decode-layer edge cases on the GPU against the oracle:

* a chain of 40 distinct 256-expert layers (block-FP8, bf16 router, FP8 shared expert: the depth of
  the speaker's backbone), each layer's input the previous layer's output, captured in one CUDA
  graph and replayed; every layer's routing and output checked against the oracle evaluated on that
  layer's input;
* rows with an outlier element a thousand times the rest (real hidden states have them: the exact
  e4m3 hi / lo split of x is exact only within 2^9 of a row's maximum), and rows scaled by 1e-6
  (tiny outputs: the layer sums its contributions as 64-bit fixed point in units chosen from each
  row's magnitude).
"""

import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
H, I, E = 2048, 512, 256


class _LazyExperts:
    """Expert e of a device tensor, copied to the host only when the oracle asks for it."""

    def __init__(self, t):
        self.t = t

    def __getitem__(self, e):
        return self.t[int(e)].cpu()


def _layer(dm3, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    L = {"gate": (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)}
    L["w13"], L["s13"] = dm3.fp8_block(torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02)
    L["w2"], L["s2"] = dm3.fp8_block(torch.randn(E, H, I, generator=g, device=dev) * 0.02)
    L["sh13"], L["shs13"] = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
    L["sh2"], L["shs2"] = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
    L["shg"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return L


def _call(dm3, L, x):
    return dm3.ops.moe_layer(x, L["gate"], 8, True, None, L["w13"], L["s13"], L["w2"], L["s2"], L["sh13"],
                             L["shs13"], L["sh2"], L["shs2"], L["shg"], None)


def _oracle(L, x):
    ex = {k: _LazyExperts(L[k]) for k in ("w13", "s13", "w2", "s2")}
    sw = {"gate": (L["sh13"][:I].cpu(), L["shs13"][:I // 128].cpu(), 128),
          "up": (L["sh13"][I:].cpu(), L["shs13"][I // 128:].cpu(), 128),
          "down": (L["sh2"].cpu(), L["shs2"].cpu(), 128)}
    return oracle.moe_layer(x.cpu(), L["gate"].cpu(), ex, 8, logits_bf16=True, sw=sw, g=L["shg"].cpu())


def test_routed_chain_in_cuda_graph_matches_oracle(dm3):
    dev = torch.device("cuda", torch.cuda.current_device())
    layers = [_layer(dm3, 7000 + l, dev) for l in range(40)]
    x0 = inputs.decode_rows(2, seed=7100).to(dev)

    def chain(x):
        outs = []
        for L in layers:
            y, ids, w = _call(dm3, L, x)
            outs.append((x, y, ids, w))
            x = y
        return outs

    chain(x0)  # eager warm-up creates the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = chain(x0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for l, (L, (x, y, ids, w)) in enumerate(zip(layers, outs)):
        ry, rids, rw = _oracle(L, x)
        assert torch.equal(ids.cpu(), rids), l
        assert torch.equal(w.cpu(), rw) or (w.cpu().float() - rw.float()).abs().max() <= 2 ** -8, l
        assert rel_l2(y, ry) < 5e-3, l
    assert dm3.ops.moe_status(dm3.ops.moe_workspace(dev, H, I)) == 0


@pytest.mark.parametrize("case", ["outlier", "tiny"])
def test_outlier_and_tiny_rows(dm3, case):
    dev = torch.device("cuda", torch.cuda.current_device())
    L = _layer(dm3, 7200, dev)
    x = inputs.decode_rows(2, seed=7201).float()
    if case == "outlier":
        x[0, 17] = 1000.0 * x[0].abs().max()   # one element three orders above the rest of its row
        x[1, 1999] = -1000.0 * x[1].abs().max()
    else:
        x = x * 1e-6                           # tiny rows and tiny outputs
    x = x.to(torch.bfloat16)
    y, ids, w = _call(dm3, L, x.to(dev))
    ry, rids, rw = _oracle(L, x)
    assert torch.equal(ids.cpu(), rids)
    for r in range(2):
        assert rel_l2(y[r], ry[r]) < REL_L2_TOL, r
        assert rel_l2(y[r], ry[r]) < 5e-3, r
    assert torch.isfinite(y.float()).all()
    # the speaker path (fp32 router, bias) on the same rows
    p = inputs.speaker_params()
    pq = dict(p)
    pq["w13"], pq["s13"] = oracle.fp8_block(p["w13"])
    pq["w2"], pq["s2"] = oracle.fp8_block(p["w2"])
    sp = dm3.Speaker({k: pq[k] for k in ("gate", "bias", "w13", "s13", "w2", "s2")})
    ys, sids, _ = sp.route_and_combine(x.to(dev))
    rys, rsids, _ = oracle.speaker(x, pq)
    assert torch.equal(sids.cpu(), rsids)
    assert rel_l2(ys, rys) < 5e-3
