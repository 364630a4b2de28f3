"""Prefill (prompt-reading) MoE kernels on the GPU against the oracle: router indices and the
dispatch permutation bit-exact, routing weights within one bf16 ulp, outputs within the relative-L2
tolerance, workspace status clean."""

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, experts, oracle_shared, rel_l2, routed_layer, to_dev

pytestmark = pytest.mark.gpu
H, I = 2048, 512


@pytest.fixture(scope="module")
def layer256():
    """256 block-FP8 experts (128x128 scales), bf16 router, shared expert + gate, on the GPU."""
    layer = routed_layer(200)
    layer["dev"] = {"ex": to_dev(layer["experts"]), "sh": to_dev(layer["sh"]), "gate": layer["gate"].cuda(),
                    "sh_gate": layer["sh_gate"].cuda()}
    return layer


def _status_clean(dm3):
    for ws in dm3.ops._pf_workspaces.values():
        assert dm3.ops.moe_status(ws) == 0


def _ulp_diff(a, b):
    return (a.cpu().view(torch.int16).int() - b.cpu().view(torch.int16).int()).abs().max().item()


def _prefill(dm3, layer, x, bias=None, shared=True, logits_bf16=True):
    d = layer["dev"]
    ex = d["ex"]
    sh = d["sh"] if shared else {"w13": None, "s13": None, "w2": None, "s2": None}
    return dm3.ops.moe_prefill(x.cuda(), d["gate"], 8, logits_bf16, None if bias is None else bias.cuda(), ex["w13"],
                               ex["s13"], ex["w2"], ex["s2"], sh["w13"], sh["s13"], sh["w2"], sh["s2"],
                               d["sh_gate"] if shared else None, None)


def _oracle_layer(layer, x, bias=None, shared=True, logits_bf16=True):
    cache = layer.setdefault("cache", {})
    return oracle.moe_layer(x, layer["gate"], layer["experts"], 8, logits_bf16=logits_bf16, logit_bias=bias,
                            sw=oracle_shared(layer, 128) if shared else None, g=layer["sh_gate"] if shared else None,
                            expert_cache=cache)


@pytest.mark.parametrize("t,bias_seed", [(1, None), (37, None), (512, 31), (300, 33)])
def test_route_matches_oracle(dm3, layer256, t, bias_seed):
    x = inputs.decode_rows(t, seed=210 + t)
    bias = None if bias_seed is None else inputs.zipf_bias(bias_seed)
    ids, w = dm3.ops.route(x.cuda(), layer256["dev"]["gate"], 8, True, None if bias is None else bias.cuda())
    rids, rw = oracle.route(x, layer256["gate"], 8, logits_bf16=True, logit_bias=bias)
    assert torch.equal(ids.cpu(), rids)
    assert _ulp_diff(w, rw) <= 1
    _status_clean(dm3)


def test_route_fp32_logits(dm3, layer256):
    """A bf16 router whose logits stay fp32 (no bf16 rounding before the softmax)."""
    x = inputs.decode_rows(96, seed=230)
    ids, w = dm3.ops.route(x.cuda(), layer256["dev"]["gate"], 8, False, None)
    rids, rw = oracle.route(x, layer256["gate"], 8, logits_bf16=False)
    assert torch.equal(ids.cpu(), rids)
    assert _ulp_diff(w, rw) <= 1


def test_prefill_layer_zipf_t512(dm3, layer256):
    """The prompt-reading configuration: T = 512, 256 experts, Zipf(1.1)-biased routing, shared expert."""
    x = inputs.decode_rows(512, seed=240)
    bias = inputs.zipf_bias(31)
    y, ids, w, perm, offsets = _prefill(dm3, layer256, x, bias)
    ry, rids, rw = _oracle_layer(layer256, x, bias)
    assert torch.equal(ids.cpu(), rids)
    assert _ulp_diff(w, rw) <= 1
    rperm, roff = oracle.permutation(rids, 256)
    assert torch.equal(perm.cpu(), rperm)
    assert torch.equal(offsets.cpu(), roff)
    err = rel_l2(y, ry)
    assert err < REL_L2_TOL, err
    assert err < 5e-3, err
    _status_clean(dm3)


@pytest.mark.parametrize("t", [1, 5, 70, 129])
def test_prefill_ragged_without_shared(dm3, layer256, t):
    x = inputs.decode_rows(t, seed=250 + t)
    y, ids, w, perm, offsets = _prefill(dm3, layer256, x, shared=False)
    ry, rids, rw = _oracle_layer(layer256, x, shared=False)
    assert torch.equal(ids.cpu(), rids)
    rperm, roff = oracle.permutation(rids, 256)
    assert torch.equal(perm.cpu(), rperm) and torch.equal(offsets.cpu(), roff)
    assert rel_l2(y, ry) < 5e-3
    _status_clean(dm3)


def test_prefill_row_scales_small_dims(dm3):
    """1x128 (per-row) scales, H = 1024, I = 256, 64 experts, a shared expert with a gate."""
    h, i, e = 1024, 256, 64
    layer = routed_layer(260, srows=1, h=h, i=i, e=e)
    x = inputs.decode_rows(150, seed=261, h=h)
    ex, sh = to_dev(layer["experts"]), to_dev(layer["sh"])
    y, ids, w, perm, offsets = dm3.ops.moe_prefill(x.cuda(), layer["gate"].cuda(), 8, True, None, ex["w13"], ex["s13"],
                                                   ex["w2"], ex["s2"], sh["w13"], sh["s13"], sh["w2"], sh["s2"],
                                                   layer["sh_gate"].cuda(), None)
    ry, rids, rw = oracle.moe_layer(x, layer["gate"], layer["experts"], 8, logits_bf16=True,
                                    sw=oracle_shared(layer, 1), g=layer["sh_gate"], srows=1)
    assert torch.equal(ids.cpu(), rids)
    assert rel_l2(y, ry) < 5e-3
    _status_clean(dm3)


@pytest.mark.parametrize("t", [6, 300])
def test_grouped_forward_given_routing(dm3, t):
    """fp8_moe_forward with more rows than the decode kernels take: the grouped path, with the
    speaker's 32 experts and fp32 router providing the routing."""
    p = inputs.speaker_params()
    q13, s13 = oracle.fp8_block(p["w13"])
    q2, s2 = oracle.fp8_block(p["w2"])
    x = inputs.decode_rows(t, seed=270 + t)
    ids, w = oracle.route(x, p["gate"], 8)
    y = dm3.fp8_moe_forward(x.cuda(), ids.cuda(), w.cuda(), q13.cuda(), s13.cuda(), q2.cuda(), s2.cuda())
    ref = oracle.moe_forward(x, ids, w, q13, s13, q2, s2)
    assert rel_l2(y, ref) < 5e-3
    _status_clean(dm3)


def test_grouped_bad_ids_are_skipped_and_flagged(dm3):
    h, i, e = 1024, 256, 16
    ex = experts(e, h, i, seed=280)
    x = inputs.decode_rows(20, seed=281, h=h)
    g = torch.Generator().manual_seed(282)
    ids = torch.stack([torch.randperm(e, generator=g)[:8] for _ in range(20)])
    w = torch.softmax(torch.randn(20, 8, generator=g), -1).to(torch.bfloat16)
    ids_bad = ids.clone()
    ids_bad[3, 2] = e + 5
    ids_bad[11, 0] = -1
    d = to_dev(ex)
    y = dm3.fp8_moe_forward(x.cuda(), ids_bad.cuda(), w.cuda(), d["w13"], d["s13"], d["w2"], d["s2"])
    wz = w.clone()
    wz[3, 2] = 0
    wz[11, 0] = 0
    ids_ok = ids_bad.clamp(0, e - 1)
    ref = oracle.moe_forward(x, ids_ok, wz, ex["w13"], ex["s13"], ex["w2"], ex["s2"])
    assert rel_l2(y, ref) < 5e-3
    ws = dm3.ops._pf_workspaces[torch.cuda.current_device()]
    assert dm3.ops.moe_status(ws) == 2  # STATUS_BAD_EXPERT
    assert dm3.ops.moe_status(ws) == 0


def test_prefill_graph_replay(dm3, layer256):
    """The prefill chain captured in a CUDA graph replays to the eager result."""
    x = inputs.decode_rows(256, seed=290).cuda()
    bias = inputs.zipf_bias(31).cuda()
    eager = _prefill(dm3, layer256, x, bias)[0].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = _prefill(dm3, layer256, x, bias)[0]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_router_error_window_is_conservative(dm3, layer256):
    """The select kernel treats |approximate - exact logit| <= 2^-10 |x| |w_e| as proven. Measure the
    tensor-core partial sums the logits kernel leaves in the workspace against exact logits: the
    observed error must sit far inside the window (below 2^-16 |x| |w_e|)."""
    t, e = 512, 256
    x = inputs.decode_rows(t, seed=300)
    dm3.ops.route(x.cuda(), layer256["dev"]["gate"], 8, True, None)
    torch.cuda.synchronize()
    ws = dm3.ops._pf_workspaces[torch.cuda.current_device()]
    ks = H // 512
    lpart = ws[128: 128 + ks * t * e * 4].view(torch.float32).view(ks, t, e).sum(0).double().cpu()
    xd = x.double()
    gd = layer256["gate"].double()
    exact = xd @ gd.T
    bound = xd.norm(dim=1, keepdim=True) * gd.norm(dim=1)[None, :]
    ratio = ((lpart - exact).abs() / bound).max().item()
    assert ratio < 2.0 ** -16, ratio
    np.testing.assert_array_less(-1, ratio)
