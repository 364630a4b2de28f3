"""The reference-facing drop-ins on the GPU: speaker_forward (fused with a block-FP8 shared
expert, or with the block's own bf16 shared expert) against the reference's golden outputs, and
the engine patch helper."""

import types
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


def _block(dm3, fp8_shared: bool):
    p = inputs.speaker_params()
    sp = dm3.Speaker(p)  # quantises with fp8_block on the GPU (engine.py:229-230)
    shared = inputs.shared_mlp().cuda()
    if fp8_shared:
        assert dm3.convert(shared) == 3
    gate = inputs.shared_gate_linear().cuda()
    experts = types.SimpleNamespace(speaker=sp)
    return types.SimpleNamespace(experts=experts, shared_expert=shared, shared_expert_gate=gate)


@pytest.mark.parametrize("fp8_shared", [True, False])
def test_speaker_forward_matches_reference(dm3, fp8_shared):
    g = np.load(G / "speaker_forward_ref.npz")
    block = _block(dm3, fp8_shared)

    def routed(self, x):
        raise AssertionError("decode rows must take the speaker path")

    fwd = dm3.make_speaker_forward(routed, lambda: 2)
    x = inputs.decode_rows(2, seed=202).cuda()
    y = fwd(block, x[None])[0]
    if fp8_shared:
        assert isinstance(block._dm3_shared, dm3.SharedExpert)  # fused path taken
    ref = torch.from_numpy(g["y_fp8_shared" if fp8_shared else "y_bf16_shared"]).view(torch.bfloat16)
    assert rel_l2(y, ref) < 5e-3


def test_speaker_forward_routes_prefill_rows_to_routed_path(dm3):
    block = _block(dm3, True)
    seen = []

    def routed(self, x):
        seen.append(tuple(x.shape))
        return x

    fwd = dm3.make_speaker_forward(routed, lambda: 2)
    x = inputs.decode_rows(3, seed=7).cuda()
    fwd(block, x[None])
    assert seen == [(1, 3, 2048)]


def test_install_patches_engine_namespace(dm3):
    class SparseMoeBlock:
        def forward(self, x):
            return "routed"

    eng = types.SimpleNamespace(routed_forward=SparseMoeBlock.forward, SparseMoeBlock=SparseMoeBlock,
                                OnDemandExperts=types.SimpleNamespace(batch=1), fp8_moe_forward=None)
    dm3.install(eng)
    assert eng.fp8_moe_forward is dm3.fp8_moe_forward and eng.Speaker is dm3.Speaker
    assert SparseMoeBlock.forward is eng.speaker_forward
    blk = types.SimpleNamespace(experts=types.SimpleNamespace(speaker=None))
    assert eng.speaker_forward(blk, torch.zeros(1, 2, 8)) == "routed"


def test_fp8_block_on_gpu_matches_cpu(dm3):
    """engine.fp8_block runs on the GPU in the reference (engine.py:229). torch's CUDA division by
    the scalar 448 may differ from the CPU's by one ulp, so scales agree to 1 ulp and e4m3 codes
    agree except where such an ulp moves a value across a rounding boundary."""
    w = inputs.block_quant_input()
    q, s = dm3.fp8_block(w.cuda())
    qo, so = oracle.fp8_block(w)
    assert torch.allclose(s.cpu(), so, rtol=2.0**-23, atol=0)
    diff = (q.cpu().view(torch.uint8).int() - qo.view(torch.uint8).int()).abs()
    assert diff.max() <= 1 and diff.float().mean() < 1e-3
