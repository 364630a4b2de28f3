"""Failure detection on the GPU without a GPU fault: a bounded device-side wait runs out.

The expert-parallel prefill waits (bounded) for every peer rank's flags. Here rank 0 of a world of
2 runs on one GPU with a second local arena standing in for rank 1, which nobody ever signals, and
a 10 ms wait limit. The call must return, the workspace status word must carry the timeout bit,
and the GPU context must stay usable: the single-GPU prefill afterwards gives the same result as
before the failure. Nothing here faults, traps or hangs the device: every access stays inside the
two arenas and the workspace, and every wait ends at its limit.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

H, I, E, K, T = 2048, 512, 256, 8, 64


def _layer(dm3, dev):
    g = torch.Generator(device=dev).manual_seed(900)
    L = {"gate": (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)}
    L["w13"], L["s13"] = dm3.fp8_block(torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02)
    L["w2"], L["s2"] = dm3.fp8_block(torch.randn(E, H, I, generator=g, device=dev) * 0.02)
    L["sh13"], L["shs13"] = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
    L["sh2"], L["shs2"] = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
    L["shg"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=dev)
    L["x"] = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    return L


def _prefill(dm3, L):
    return dm3.ops.moe_prefill(L["x"], L["gate"], K, True, None, L["w13"], L["s13"], L["w2"], L["s2"], L["sh13"],
                               L["shs13"], L["sh2"], L["shs2"], L["shg"], None)


def test_expert_parallel_wait_runs_out_and_context_survives(dm3):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = dm3._lib.load()
    L = _layer(dm3, dev)
    ref = _prefill(dm3, L)
    torch.cuda.synchronize()
    assert dm3.ops.moe_status(dm3.ops._pf_workspaces[0]) == 0

    world, tl = 2, T
    nbytes = lib.dm3_ep_arena_bytes(world, tl, K, H)
    arenas = []
    for _ in range(world):
        p = ctypes.c_void_p()
        dm3._lib.check(lib.dm3_ep_alloc(nbytes, ctypes.byref(p)), "dm3_ep_alloc")
        arenas.append(p.value)
    el = E // world
    try:
        dm3.ops.set_wait_limit(10_000_000)  # 10 ms
        y, ids, w = dm3.ep.moe_prefill_ep(L["x"], L["gate"], K, True, None, L["w13"][:el], L["s13"][:el],
                                          L["w2"][:el], L["s2"][:el], L["sh13"], L["shs13"], L["sh2"], L["shs2"],
                                          L["shg"], None, world, 0, tl, arenas)
        torch.cuda.synchronize()
        status = dm3.ops.moe_status(dm3.ep._ep_workspaces[0])
        assert status & 1, f"expected the timeout bit, got status {status}"
        # routing happens before any wait: it is intact
        assert torch.equal(ids, ref[1]) and torch.equal(w, ref[2])
    finally:
        dm3.ops.set_wait_limit(1_000_000_000)
        torch.cuda.synchronize()
        for a in arenas:
            lib.dm3_ep_free(ctypes.c_void_p(a))
    # the context is usable and the regular path is unaffected
    again = _prefill(dm3, L)
    torch.cuda.synchronize()
    assert dm3.ops.moe_status(dm3.ops._pf_workspaces[0]) == 0
    for a, b in zip(again, ref):
        assert torch.equal(a, b)
