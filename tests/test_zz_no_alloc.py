"""The allocation-free fused MoE layer (dm3_moe_layer_noalloc) against the regular entry point.

Some callers cannot allocate device memory: code that runs inside another runtime's memory pool,
plugin hosts that only hand out their own buffers, or paths where cudaMalloc is not allowed. For
them the library keeps the layer's scratch in a static device array. This test calls that entry
point through the C ABI twice in a row (the second call relies on the first leaving the shared
scratch clean) and checks each result against dm3_moe_layer with a caller-provided workspace.
The file name sorts last so a run that stops at the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from tests.golden import inputs
from tests.helpers import REL_L2_TOL, experts, rel_l2, to_dev

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_noalloc_layer_matches_workspace_layer(dm3):
    h, i, e = 512, 128, 16
    g = torch.Generator().manual_seed(77)
    ex = to_dev(experts(e, h, i, seed=78))
    sh = {k: v[0] for k, v in to_dev(experts(1, h, i, seed=79)).items()}
    gate = (torch.randn(e, h, generator=g) * 0.02).cuda()
    bias = (torch.randn(h, generator=g) * 0.02).cuda()
    sh_gate = inputs.shared_gate_weight(80, h=h).reshape(-1).cuda()
    lib = dm3._lib.load()
    for call in range(2):
        x = inputs.decode_rows(2, seed=81 + call, h=h).cuda()
        y_ref, ids_ref, w_ref = dm3.ops.moe_layer(x, gate, 8, False, None, ex["w13"], ex["s13"], ex["w2"], ex["s2"],
                                                  sh["w13"], sh["s13"], sh["w2"], sh["s2"], sh_gate, bias)
        y = torch.empty_like(y_ref)
        ids = torch.empty_like(ids_ref)
        w = torch.empty_like(w_ref)
        rc = lib.dm3_moe_layer_noalloc(
            _ptr(x), 2, h, i, _ptr(gate), 0, e, 8, 0, None,
            _ptr(ex["w13"]), ex["w13"].stride(0), _ptr(ex["s13"]), ex["s13"].stride(0),
            _ptr(ex["w2"]), ex["w2"].stride(0), _ptr(ex["s2"]), ex["s2"].stride(0), 128,
            _ptr(sh["w13"]), _ptr(sh["s13"]), _ptr(sh["w2"]), _ptr(sh["s2"]), 128, _ptr(sh_gate), _ptr(bias),
            _ptr(y), _ptr(ids), _ptr(w), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.dm3_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref)
        assert torch.equal(w, w_ref)
        assert rel_l2(y, y_ref) < REL_L2_TOL
        assert torch.isfinite(y.float()).all()


def test_noalloc_rejects_oversized_dims(dm3):
    lib = dm3._lib.load()
    p = ctypes.c_void_p(256)
    rc = lib.dm3_moe_layer_noalloc(p, 2, 4096, 512, p, 0, 32, 8, 0, None, p, 0, p, 0, p, 0, p, 0, 128,
                                   None, None, None, None, 128, None, None, p, None, None, None)
    assert rc != 0
    assert lib.dm3_last_error()  # a clear reason is reported
