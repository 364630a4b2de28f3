"""Host-side logic on CPU: the drop-in quantisers (bit-exact to the oracle, which is pinned to the
reference), scale-layout inference, FP8Linear/convert bookkeeping, shared-expert packing and the
expert-parallel placement helpers."""

import torch

import oracle
from tests.golden import inputs


def test_fp8_block_mirror_bit_exact(dm3):
    w = inputs.block_quant_input()
    q, s = dm3.fp8_block(w)
    qo, so = oracle.fp8_block(w)
    assert torch.equal(q.view(torch.uint8), qo.view(torch.uint8)) and torch.equal(s, so)


def test_quantize_mirror_bit_exact(dm3):
    w = inputs.row_quant_input()
    q, s = dm3.quantize(w)
    qo, so = oracle.quantize_rows(w)
    assert torch.equal(q.view(torch.uint8), qo.view(torch.uint8)) and torch.equal(s, so)
    # fp32 products, as fp8_linear.dequantize computes them; the oracle's float64 product is exact
    assert torch.equal(dm3.dequantize(q, s), torch.from_numpy(oracle.dequant(qo, so, 1)).float())


def test_scale_layout_inference(dm3):
    sr = dm3.ops.scale_rows
    assert sr(1024, 8) == 128 and sr(1024, 1024) == 1
    assert sr(4097, 33) == 128 and sr(4097, 4097) == 1
    assert sr(2048, 16) == 128 and sr(512, 4) == 128


def test_convert_and_fp8linear_buffers(dm3):
    m = torch.nn.Sequential(torch.nn.Linear(256, 512, bias=False), torch.nn.Linear(512, 64), torch.nn.Linear(100, 600))
    n = dm3.convert(m)
    assert n == 1  # only the first: out >= 512 and in % 128 == 0 (fp8_linear.py:72)
    f = m[0]
    assert isinstance(f, dm3.FP8Linear)
    assert f.q.dtype == torch.float8_e4m3fn and f.q.shape == (512, 256) and f.s.shape == (512, 2)
    assert f.out_features == 512 and f.in_features == 256 and f.weight.numel() == 0


def test_shared_expert_packing(dm3):
    mlp = inputs.SharedMLP(*(inputs.shared_weights(h=256, i=128)[k] for k in ("gate", "up", "down")))
    gate = torch.nn.Linear(256, 1, bias=False, dtype=torch.bfloat16)
    block = type("B", (), {})()
    block.shared_expert, block.shared_expert_gate = mlp, gate
    assert dm3.SharedExpert.from_block(block) is None  # bf16 linears are not packed
    dm3.convert(mlp, min_out=128)
    pack = dm3.SharedExpert.from_block(block)
    assert pack.w13.shape == (256, 256) and pack.s13.shape == (256, 2)
    assert pack.w2.shape == (256, 128) and pack.s2.shape == (256, 1)
    assert torch.equal(pack.w13[:128].view(torch.uint8), mlp.gate_proj.q.view(torch.uint8))
    assert torch.equal(pack.w13[128:].view(torch.uint8), mlp.up_proj.q.view(torch.uint8))
    assert pack.gate_row.shape == (256,)


def test_fake_impls_trace_on_meta(dm3):
    x = torch.empty(2, 2048, dtype=torch.bfloat16, device="meta")
    q = torch.empty(4096, 2048, dtype=torch.float8_e4m3fn, device="meta")
    s = torch.empty(4096, 16, device="meta")
    y = torch.ops.dm3.fp8_gemv(x, q, s)
    assert y.shape == (2, 4096) and y.dtype == torch.bfloat16
    w13 = torch.empty(32, 1024, 2048, dtype=torch.float8_e4m3fn, device="meta")
    s13 = torch.empty(32, 8, 16, device="meta")
    w2 = torch.empty(32, 2048, 512, dtype=torch.float8_e4m3fn, device="meta")
    s2 = torch.empty(32, 16, 4, device="meta")
    g = torch.empty(32, 2048, device="meta")
    y, ids, w = torch.ops.dm3.moe_layer(x, g, 8, False, None, w13, s13, w2, s2, None, None, None, None, None, None)
    assert y.shape == (2, 2048) and ids.shape == (2, 8) and ids.dtype == torch.int64 and w.dtype == torch.bfloat16


def test_tile_balanced_placement(dm3):
    """A placement from observed counts: every rank holds E / world experts with local indices
    0 .. E / world - 1, and the ranks' tile totals differ by at most the largest expert's tiles
    (greedy longest-processing-time on tiles of 64 tokens)."""
    E, world = 256, 4
    r = torch.arange(1, E + 1, dtype=torch.float64)
    counts = torch.floor(4096 * r.pow(-1.1) / r.pow(-1.1).sum()).long()  # Zipf-skewed pair counts
    counts = counts[torch.randperm(E, generator=torch.Generator().manual_seed(3))]
    owner = dm3.ep.tile_balanced_placement(counts, world)
    o = owner.long()
    assert all(int(((o >> 16) == k).sum()) == E // world for k in range(world))
    for k in range(world):
        mine = dm3.ep.local_experts(owner, k)
        assert sorted((o[mine] & 0xFFFF).tolist()) == list(range(E // world))
    tiles = torch.ceil(counts.double() / 64)
    per = [float(tiles[(o >> 16) == k].sum()) for k in range(world)]
    assert max(per) - min(per) <= float(tiles.max())
