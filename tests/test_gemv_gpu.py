"""Block-FP8 GEMV on the GPU against the oracle (and the reference Triton kernel's golden output)."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"

# (K, N) of the block-FP8 GEMV sweep, plus ragged / small cases and (2048, 6144): three resident
# 16-row tiles per CTA, the last one partly filled
SHAPES = [(2048, 4096), (4096, 2048), (2048, 8192), (2048, 512), (2048, 4097), (512, 200), (8192, 128), (128, 1),
          (384, 33), (2048, 6144)]


def _case(k, n, seed, srows):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    if srows == 1:
        return oracle.quantize_rows(w)
    pad = (-n) % 128
    wp = torch.cat([w, torch.zeros(pad, k)]) if pad else w
    q, s = oracle.fp8_block(wp)
    return q[:n].contiguous(), s


@pytest.mark.parametrize("k,n", SHAPES)
@pytest.mark.parametrize("srows", [1, 128])
def test_gemv_parity(dm3, k, n, srows):
    q, s = _case(k, n, seed=k * 7 + n, srows=srows)
    x = inputs.decode_rows(4, seed=n + 1, h=k)
    qd, sd, xd = q.cuda(), s.cuda(), x.cuda()
    for m in (1, 2, 3, 4):
        y = dm3.ops.fp8_gemv(xd[:m], qd, sd)
        ref = oracle.gemv(x[:m], q, s, srows)
        err = rel_l2(y, ref)
        assert err < REL_L2_TOL, (m, err)
        assert err < 5e-3, (m, err)


def test_gemv_bias_fp32_out_and_many_rows(dm3):
    q, s = _case(2048, 1024, seed=3, srows=1)
    x = inputs.decode_rows(11, seed=4)
    bias = (torch.randn(1024, generator=torch.Generator().manual_seed(5)) * 0.1).to(torch.bfloat16)
    y = dm3.ops.fp8_gemv(x.cuda(), q.cuda(), s.cuda(), bias.cuda(), True)
    assert y.dtype == torch.float32
    ref = oracle.gemv(x, q, s, 1, bias=bias, out_dtype=torch.float32)
    assert rel_l2(y, ref) < 1e-3


def test_gemv_matches_reference_triton_golden(dm3):
    d = np.load(G / "gemv_ref.npz")
    x, w = inputs.gemv_case()
    q, s = oracle.quantize_rows(w)
    for m in (1, 2):
        y = dm3.ops.fp8_gemv(x[:m].cuda(), q.cuda(), s.cuda()).cpu()
        ref = torch.from_numpy(d[f"y_m{m}"]).view(torch.bfloat16)
        assert rel_l2(y, ref) < 5e-3
        assert (y.view(torch.int16) == ref.view(torch.int16)).float().mean() > 0.9


def test_fp8linear_reference_self_test(dm3):
    """fp8_linear.py:81-90: FP8Linear against the bf16 linear within rel-L2 0.05 at M = 1, 2, 64."""
    for n, k in [(9216, 2048), (2048, 6144), (512, 2048)]:
        g = torch.Generator().manual_seed(n + k)
        lin = torch.nn.Linear(k, n, bias=False, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
        lin = lin.cuda()
        f = dm3.FP8Linear(lin)
        x = torch.randn(64, k, generator=g).to(torch.bfloat16).cuda()
        for m in (1, 2, 64):
            assert rel_l2(f(x[:m]), lin(x[:m])) < 0.05


def test_gemv_gather_audio_head(dm3):
    """Audio head restricted to eos + a 4096-row band gathered from a larger matrix (engine.py:409-411)."""
    g = torch.Generator().manual_seed(9)
    full = torch.randn(12000, 2048, generator=g) * 0.02
    rows = torch.cat([torch.tensor([11999]), torch.arange(3000, 3000 + 4096)])
    q, s = oracle.quantize_rows(full)
    x = inputs.decode_rows(2, seed=10)
    lib = dm3._lib.load()
    qd, sd, xd, rd = q.cuda(), s.cuda(), x.cuda(), rows.cuda()
    y = torch.empty(2, rows.numel(), dtype=torch.float32, device="cuda")
    rc = lib.dm3_fp8_gemv_gather(ctypes.c_void_p(xd.data_ptr()), 2, 2048, rows.numel(), ctypes.c_void_p(qd.data_ptr()),
                                 2048, 12000, ctypes.c_void_p(rd.data_ptr()), ctypes.c_void_p(sd.data_ptr()), 16, 1,
                                 ctypes.c_void_p(y.data_ptr()), rows.numel(), 1,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    ref = oracle.gemv(x, q[rows], s[rows], 1, out_dtype=torch.float32)
    assert rel_l2(y, ref) < 1e-3


def test_gemv_cuda_graph_replay(dm3):
    q, s = _case(2048, 4096, seed=12, srows=128)
    x = inputs.decode_rows(2, seed=13).cuda()
    qd, sd = q.cuda(), s.cuda()
    y0 = dm3.ops.fp8_gemv(x, qd, sd)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = dm3.ops.fp8_gemv(x, qd, sd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y0)
