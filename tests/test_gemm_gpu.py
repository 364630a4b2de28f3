"""Block-FP8 GEMM (dm3::fp8_gemm, many activation rows) on the GPU against the oracle: the exact
block-scaled product (oracle.gemv) within 5e-3 and the reference's dequantise + F.linear path
(oracle.linear_dequant, fp8_linear.py:60-61) within the 2e-2 contract; both scale layouts, ragged
row counts and widths, bias, fp32 output, CUDA-graph replay and the reference's golden M=3 rows."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


def _weights(k, n, seed, srows):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    if srows == 1:
        return oracle.quantize_rows(w)
    pad = (-n) % 128
    q, s = oracle.fp8_block(torch.cat([w, torch.zeros(pad, k)]) if pad else w)
    return q[:n].contiguous(), s


@pytest.mark.parametrize("m,k,n,srows", [(3, 512, 200, 1), (5, 2048, 1024, 128), (17, 2048, 4097, 1),
                                         (64, 6144, 2048, 1), (100, 4096, 129, 128), (256, 2048, 9216, 1),
                                         (300, 1024, 640, 128), (1000, 256, 384, 1)])
def test_gemm_parity(dm3, m, k, n, srows):
    q, s = _weights(k, n, seed=m + k + n, srows=srows)
    x = inputs.decode_rows(m, seed=m * 3 + 1, h=k)
    y = dm3.ops.fp8_gemm(x.cuda(), q.cuda(), s.cuda())
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    exact = oracle.gemv(x, q, s, srows)
    assert rel_l2(y, exact) < 5e-3
    assert rel_l2(y, oracle.linear_dequant(x, q, s, srows)) < REL_L2_TOL
    assert dm3.ops.moe_status(dm3.ops._gemm_workspaces[torch.cuda.current_device()]) == 0


def test_gemm_bias_fp32_out_and_outlier_rows(dm3):
    k, n, m = 2048, 1536, 40
    q, s = _weights(k, n, seed=7, srows=1)
    x = inputs.decode_rows(m, seed=8, h=k).float()
    x[3, 100] = 900.0   # one element three orders above the rest of its row
    x[5] *= 1e-6        # a row of tiny values
    x = x.to(torch.bfloat16)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(9)) * 0.1).to(torch.bfloat16)
    y = dm3.ops.fp8_gemm(x.cuda(), q.cuda(), s.cuda(), bias.cuda(), True)
    assert y.dtype == torch.float32
    ref = oracle.gemv(x, q, s, 1, bias=bias, out_dtype=torch.float32)
    assert rel_l2(y, ref) < 1e-3
    for row in (3, 5):
        assert rel_l2(y[row], ref[row]) < 5e-3, row


def test_gemm_golden_rows_and_fp8linear(dm3):
    d = np.load(G / "gemv_ref.npz")
    x, w = inputs.gemv_case()
    q, s = oracle.quantize_rows(w)
    y = dm3.ops.fp8_gemm(x[:3].cuda(), q.cuda(), s.cuda()).cpu()
    ref = torch.from_numpy(d["y_m3"]).view(torch.bfloat16)  # the reference's FP8Linear, 3 rows
    assert rel_l2(y, ref) < 5e-3
    lin = torch.nn.Linear(2048, 4096, bias=True, dtype=torch.bfloat16).cuda()
    f = dm3.FP8Linear(lin)
    xs = inputs.decode_rows(96, seed=12).cuda()
    yf = f(xs.view(2, 48, 2048))
    assert yf.shape == (2, 48, 4096)
    ref2 = oracle.linear_dequant(xs.cpu(), f.q.cpu(), f.s.cpu(), 1, bias=lin.bias.detach().cpu())
    assert rel_l2(yf.reshape(96, 4096), ref2) < REL_L2_TOL


def test_gemm_cuda_graph_replay(dm3):
    q, s = _weights(2048, 2048, seed=13, srows=128)
    x = inputs.decode_rows(128, seed=14).cuda()
    qd, sd = q.cuda(), s.cuda()
    y0 = dm3.ops.fp8_gemm(x, qd, sd)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = dm3.ops.fp8_gemm(x, qd, sd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y0)
