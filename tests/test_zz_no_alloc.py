"""The allocation-free fused MoE layer (dm3_moe_layer_noalloc) against the regular entry point.

Some callers cannot allocate device memory: code that runs inside another runtime's memory pool,
plugin hosts that only hand out their own buffers, or paths where cudaMalloc is not allowed. For
them the library keeps the layer's scratch in a static device array. This test calls that entry
point through the C ABI twice in a row (the second call relies on the first leaving the shared
scratch clean) and checks each result against dm3_moe_layer with a caller-provided workspace:
both run the same kernels, whose output sums are exact fixed-point integers, so the outputs must
be identical. It covers a small layer and the full Drama-3 shape (H 2048, I 512, 256 experts),
whose workspace nearly fills the static array. The file name sorts last so a run that stops at
the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from tests.golden import inputs
from tests.helpers import experts, to_dev

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dev_experts(e, h, i, seed, dev):
    """Seeded block-FP8 experts, quantised on the device for the large shape."""
    if e * h * i <= (1 << 24):
        return to_dev(experts(e, h, i, seed=seed))
    import drama3_b200 as dm3

    g = torch.Generator(device=dev).manual_seed(seed)
    w13, s13 = dm3.fp8_block(torch.randn(e, 2 * i, h, generator=g, device=dev) * 0.02)
    w2, s2 = dm3.fp8_block(torch.randn(e, h, i, generator=g, device=dev) * 0.02)
    return {"w13": w13, "s13": s13, "w2": w2, "s2": s2}


@pytest.mark.parametrize("h,i,e,router_dtype", [(512, 128, 16, torch.float32), (2048, 512, 256, torch.bfloat16)])
def test_noalloc_layer_matches_workspace_layer(dm3, h, i, e, router_dtype):
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(77)
    ex = _dev_experts(e, h, i, 78, dev)
    sh = {k: v[0] for k, v in _dev_experts(1, h, i, 79, dev).items()}
    gate = (torch.randn(e, h, generator=g) * 0.02).to(router_dtype).cuda()
    bias = (torch.randn(h, generator=g) * 0.02).cuda()
    sh_gate = inputs.shared_gate_weight(80, h=h).reshape(-1).cuda()
    rdt, lbf16 = (0, 0) if router_dtype == torch.float32 else (1, 1)
    lib = dm3._lib.load()
    for call in range(2):
        x = inputs.decode_rows(2, seed=81 + call, h=h).cuda()
        y_ref, ids_ref, w_ref = dm3.ops.moe_layer(x, gate, 8, bool(lbf16), None, ex["w13"], ex["s13"], ex["w2"],
                                                  ex["s2"], sh["w13"], sh["s13"], sh["w2"], sh["s2"], sh_gate, bias)
        y = torch.empty_like(y_ref)
        ids = torch.empty_like(ids_ref)
        w = torch.empty_like(w_ref)
        rc = lib.dm3_moe_layer_noalloc(
            _ptr(x), 2, h, i, _ptr(gate), rdt, e, 8, lbf16, None,
            _ptr(ex["w13"]), ex["w13"].stride(0), _ptr(ex["s13"]), ex["s13"].stride(0),
            _ptr(ex["w2"]), ex["w2"].stride(0), _ptr(ex["s2"]), ex["s2"].stride(0), 128,
            _ptr(sh["w13"]), _ptr(sh["s13"]), _ptr(sh["w2"]), _ptr(sh["s2"]), 128, _ptr(sh_gate), _ptr(bias),
            _ptr(y), _ptr(ids), _ptr(w), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.dm3_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref)
        assert torch.equal(w, w_ref)
        assert torch.equal(y, y_ref)
        assert torch.isfinite(y.float()).all()
    assert dm3.ops.noalloc_status() == 0


def test_noalloc_rejects_oversized_dims(dm3):
    lib = dm3._lib.load()
    p = ctypes.c_void_p(256)
    rc = lib.dm3_moe_layer_noalloc(p, 2, 4096, 512, p, 0, 32, 8, 0, None, p, 0, p, 0, p, 0, p, 0, 128,
                                   None, None, None, None, 128, None, None, p, None, None, None)
    assert rc == dm3._lib.DM3_ENOSPACE
    assert b"static" in lib.dm3_last_error()
