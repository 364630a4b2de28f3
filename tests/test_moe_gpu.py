"""Fused decode MoE kernels on the GPU against the oracle: routing bit-exact, outputs within the
relative-L2 tolerance, workspace status clean after every call."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, experts, oracle_shared as _oracle_shared, rel_l2, routed_layer as _routed_layer, to_dev

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"
H, I = 2048, 512


def _ws_clean(dm3, h=H, i=I):
    ws = dm3.ops.moe_workspace(torch.device("cuda"), h, i)
    assert dm3.ops.moe_status(ws) == 0


@pytest.fixture(scope="module")
def spk():
    p = inputs.speaker_params()
    pq = dict(p)
    pq["w13"], pq["s13"] = oracle.fp8_block(p["w13"])
    pq["w2"], pq["s2"] = oracle.fp8_block(p["w2"])
    return pq


@pytest.mark.parametrize("t", [1, 2, 3, 4])
def test_moe_forward_given_routing(dm3, spk, t):
    x = inputs.decode_rows(t, seed=40 + t)
    ids, w = oracle.route(x, spk["gate"], 8)
    d = to_dev(spk)
    y = dm3.fp8_moe_forward(x.cuda(), ids.cuda(), w.cuda(), d["w13"], d["s13"], d["w2"], d["s2"])
    ref = oracle.moe_forward(x, ids, w, spk["w13"], spk["s13"], spk["w2"], spk["s2"])
    err = rel_l2(y, ref)
    assert err < REL_L2_TOL, err
    assert err < 5e-3, err
    _ws_clean(dm3)


def test_moe_forward_expertstore_slots(dm3):
    """Experts addressed through ExpertStore's slot buffer: one uint8 [slots, 3*I*H] buffer with
    w13 = buf[:, :2IH] and w2 = buf[:, 2IH:] views (engine.py:32-34), so dim-0 strides are 3*I*H."""
    h, i, slots = 1024, 256, 12
    ex = experts(slots, h, i, seed=50)
    buf = torch.empty(slots, 3 * i * h, dtype=torch.uint8)
    buf[:, : 2 * i * h] = ex["w13"].view(torch.uint8).reshape(slots, -1)
    buf[:, 2 * i * h:] = ex["w2"].view(torch.uint8).reshape(slots, -1)
    bd = buf.cuda()
    w13 = bd[:, : 2 * i * h].view(slots, 2 * i, h).view(torch.float8_e4m3fn)
    w2 = bd[:, 2 * i * h:].view(slots, h, i).view(torch.float8_e4m3fn)
    assert w13.stride(0) == 3 * i * h and w2.stride(0) == 3 * i * h
    x = inputs.decode_rows(2, seed=51, h=h)
    ids = torch.tensor([[3, 7, 0, 11, 5, 2, 9, 1], [7, 4, 10, 6, 8, 3, 0, 2]])
    w = torch.softmax(torch.randn(2, 8, generator=torch.Generator().manual_seed(52)), -1).to(torch.bfloat16)
    y = dm3.fp8_moe_forward(x.cuda(), ids.cuda(), w.cuda(), w13, ex["s13"].cuda(), w2, ex["s2"].cuda())
    ref = oracle.moe_forward(x, ids, w, ex["w13"], ex["s13"], ex["w2"], ex["s2"])
    assert rel_l2(y, ref) < 5e-3
    _ws_clean(dm3, h, i)


def test_moe_forward_row_scales_and_repeats(dm3):
    """1x128 scales, a duplicated expert across rows, and two calls in a row on one workspace."""
    h, i, e = 512, 128, 5
    ex = experts(e, h, i, seed=60, srows=1)
    x = inputs.decode_rows(2, seed=61, h=h)
    ids = torch.tensor([[0, 1, 4], [4, 1, 2]])
    w = torch.tensor([[0.5, 0.25, 0.25], [0.6, 0.3, 0.1]]).to(torch.bfloat16)
    d = to_dev(ex)
    ref = oracle.moe_forward(x, ids, w, ex["w13"], ex["s13"], ex["w2"], ex["s2"], srows=1)
    for _ in range(2):
        y = dm3.fp8_moe_forward(x.cuda(), ids.cuda(), w.cuda(), d["w13"], d["s13"], d["w2"], d["s2"])
        assert rel_l2(y, ref) < 5e-3
    _ws_clean(dm3, h, i)


def test_moe_forward_bad_expert_id_is_flagged(dm3):
    h, i, e = 256, 128, 4
    ex = to_dev(experts(e, h, i, seed=70))
    x = inputs.decode_rows(1, seed=71, h=h).cuda()
    ids = torch.tensor([[1, 9]]).cuda()  # 9 is out of range: skipped, not read
    w = torch.tensor([[0.5, 0.5]]).to(torch.bfloat16).cuda()
    dm3.fp8_moe_forward(x, ids, w, ex["w13"], ex["s13"], ex["w2"], ex["s2"])
    ws = dm3.ops.moe_workspace(torch.device("cuda"), h, i)
    assert dm3.ops.moe_status(ws) == 2  # STATUS_BAD_EXPERT
    assert dm3.ops.moe_status(ws) == 0  # cleared by the read


@pytest.mark.parametrize("t", [1, 2, 4])
def test_speaker_layer_fused(dm3, spk, t):
    x = inputs.decode_rows(t, seed=80 + t)
    d = to_dev(spk)
    y, ids, w = dm3.ops.moe_layer(x.cuda(), d["gate"], 8, False, None, d["w13"], d["s13"], d["w2"], d["s2"],
                                  None, None, None, None, None, d["bias"])
    ry, rids, rw = oracle.speaker(x, spk)
    assert torch.equal(ids.cpu(), rids)
    assert (w.cpu().view(torch.int16).int() - rw.view(torch.int16).int()).abs().max() <= 1  # within one bf16 ulp
    assert rel_l2(y, ry) < 5e-3
    _ws_clean(dm3)


def test_speaker_matches_reference_golden(dm3, spk):
    g = np.load(G / "speaker_ref.npz")
    sp = dm3.Speaker({k: spk[k] for k in ("gate", "bias", "w13", "s13", "w2", "s2")})
    for t in (1, 2):
        x = inputs.decode_rows(t, seed=100 + t).cuda()
        y, ids, w = sp.route_and_combine(x)
        assert np.array_equal(ids.cpu().numpy(), g[f"ids_t{t}"])
        ref = torch.from_numpy(g[f"y_t{t}"]).view(torch.bfloat16)
        assert rel_l2(y, ref) < 5e-3


@pytest.mark.parametrize("srows", [128, 1])
def test_routed_256_layer_with_shared(dm3, srows):
    layer = _routed_layer(90, srows=srows)
    x = inputs.decode_rows(2, seed=91)
    ex, sh = to_dev(layer["experts"]), to_dev(layer["sh"])
    y, ids, w = dm3.ops.moe_layer(x.cuda(), layer["gate"].cuda(), 8, True, None, ex["w13"], ex["s13"], ex["w2"],
                                  ex["s2"], sh["w13"], sh["s13"], sh["w2"], sh["s2"], layer["sh_gate"].cuda(), None)
    ry, rids, rw = oracle.moe_layer(x, layer["gate"], layer["experts"], 8, logits_bf16=True,
                                    sw=_oracle_shared(layer, srows), g=layer["sh_gate"], srows=srows)
    assert torch.equal(ids.cpu(), rids)
    assert rel_l2(y, ry) < 5e-3
    _ws_clean(dm3)


def test_routed_layer_with_zipf_bias(dm3):
    layer = _routed_layer(95, shared=False)
    bias = inputs.zipf_bias(96)
    x = inputs.decode_rows(4, seed=97)
    ex = to_dev(layer["experts"])
    y, ids, w = dm3.ops.moe_layer(x.cuda(), layer["gate"].cuda(), 8, True, bias.cuda(), ex["w13"], ex["s13"], ex["w2"],
                                  ex["s2"], None, None, None, None, None, None)
    ry, rids, rw = oracle.moe_layer(x, layer["gate"], layer["experts"], 8, logits_bf16=True, logit_bias=bias)
    assert torch.equal(ids.cpu(), rids)
    assert rel_l2(y, ry) < 5e-3
    _ws_clean(dm3)


def test_fused_layer_cuda_graph_chain(dm3, spk):
    """Several chained layers captured in one CUDA graph and replayed, as the engine's decode step is."""
    d = to_dev(spk)
    xs = inputs.decode_rows(2, seed=120).cuda()
    layers = 6

    def chain(x):
        for _ in range(layers):
            x = dm3.ops.moe_layer(x, d["gate"], 8, False, None, d["w13"], d["s13"], d["w2"], d["s2"], None, None,
                                  None, None, None, d["bias"])[0]
        return x

    eager = chain(xs).clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = chain(xs)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    _ws_clean(dm3)
