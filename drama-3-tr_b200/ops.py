"""torch.library custom ops over the C ABI (libdm3.so).

Each op launches hand-written sm_100a kernels on the current CUDA stream, allocates its output
with torch (so CUDA-graph capture draws it from the graph's pool), performs no host
synchronisation, and has a fake (meta) implementation so torch.compile traces it as one opaque
node. There is no fallback: a missing library or a non-CUDA tensor raises.

Ops:
  dm3::fp8_gemv      block-FP8 GEMV, <= 4 rows per launch (fp8_linear.py:10-27 `_gemv`)
  dm3::fp8_gemm      block-FP8 GEMM for more rows (fp8_linear.py:60-61 dequantise + F.linear)
  dm3::moe_forward   grouped SwiGLU over block-FP8 experts with given routing
                     (fish-speech fp8_moe_forward, engine.py:147, :236)
  dm3::moe_layer     fused decode MoE layer: router + top-k + experts + shared expert + bias
                     (engine.py:153-158, :232-237)
  dm3::moe_prefill   prompt-reading MoE layer over T tokens: router, dispatch permutation, grouped
                     tensor-core SwiGLU, combine, shared expert (engine.py:143-147, :153-158)
  dm3::route         the router alone: softmax / top-k / renormalise (engine.py:233-235)
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib

E4M3 = torch.float8_e4m3fn
BF16 = torch.bfloat16
MAX_ROWS = 4  # rows per launch of the skinny kernels

_workspaces: dict = {}
_pf_workspaces: dict = {}


def _ptr(t: Optional[Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts: Optional[Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("drama3_b200 ops run on CUDA tensors only (no CPU fallback)")


def _fp8_bytes(t: Tensor) -> Tensor:
    """e4m3 weights may arrive as float8_e4m3fn or as their uint8 storage (ExpertStore.buf)."""
    if t.dtype not in (E4M3, torch.uint8):
        raise RuntimeError(f"expected float8_e4m3fn (or uint8) weights, got {t.dtype}")
    return t


def scale_rows(w_rows: int, s_rows: int) -> int:
    """Rows per scale for a weight with w_rows rows and a scale table with s_rows rows."""
    if s_rows * 128 >= w_rows and (w_rows + 127) // 128 == s_rows:
        return 128
    if s_rows == w_rows:
        return 1
    raise RuntimeError(f"scale table with {s_rows} rows does not match a weight with {w_rows} rows")


def moe_workspace(device: torch.device, H: int, I: int) -> Tensor:
    """The persistent zero-initialised workspace of the fused MoE kernels on one device.

    Kernels leave its counters at zero after every call, so one workspace per (device, H, I)
    is shared by all calls issued in stream order; calls that could overlap on the GPU (different
    streams without ordering) must pass their own workspace."""
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), H, I)
    ws = _workspaces.get(key)
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "drama3_b200: the MoE workspace must be created before CUDA-graph capture; run the op once "
                "(warm-up) or call drama3_b200.ops.moe_workspace(device, H, I) first")
        nbytes = _lib.load().dm3_moe_workspace_bytes(MAX_ROWS, H, I)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    return ws


def prefill_workspace(device: torch.device, nbytes: int) -> Tensor:
    """A zero-initialised scratch of at least nbytes for the prefill kernels on one device, grown
    on demand and shared by calls issued in stream order (the kernels rewrite what they read)."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _pf_workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "drama3_b200: the prefill workspace must be created before CUDA-graph capture; run the op once "
                "at the largest size first")
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _pf_workspaces[key] = ws
    return ws


def moe_status(ws: Tensor) -> int:
    """Reads and clears the device status word of a workspace (synchronises). 0 = all good."""
    st = ctypes.c_uint32(0)
    rc = _lib.load().dm3_moe_status(_ptr(ws), ctypes.byref(st), _stream(ws.device))
    if rc not in (_lib.DM3_OK, _lib.DM3_ETIMEOUT):
        _lib.check(rc, "dm3_moe_status")
    return int(st.value)


# ----------------------------------------------------------------------------- fp8_gemv
@torch.library.custom_op("dm3::fp8_gemv", mutates_args=())
def fp8_gemv(x: Tensor, q: Tensor, s: Tensor, bias: Optional[Tensor] = None, out_fp32: bool = False) -> Tensor:
    """y[M, N] = x[M, K] @ dequant(q[N, K], s).T (+ bias): block-FP8 GEMV on the GPU.

    x bf16 [M, K]; q e4m3 [N, K] with unit column stride; s fp32 [N, K/128] (1x128) or
    [ceil(N/128), K/128] (128x128). Rows beyond 4 are processed 4 at a time."""
    _require_cuda(x, q, s, bias)
    lib = _lib.load()
    q = _fp8_bytes(q)
    if x.dtype != BF16:
        raise RuntimeError("fp8_gemv expects bf16 activations")
    x = x.contiguous()
    s = s.contiguous()
    M, K = x.shape
    N = q.shape[0]
    if q.stride(1) != 1 or q.shape[1] != K:
        raise RuntimeError("q must be [N, K] with unit column stride")
    srows = scale_rows(N, s.shape[0])
    y = torch.empty((M, N), dtype=torch.float32 if out_fp32 else BF16, device=x.device)
    bias_kind = 0
    if bias is not None:
        if bias.dtype not in (BF16, torch.float32):
            bias = bias.float()
        bias = bias.contiguous()
        bias_kind = 1 if bias.dtype == BF16 else 2
    st = _stream(x.device)
    for m0 in range(0, M, MAX_ROWS):
        m = min(MAX_ROWS, M - m0)
        rc = lib.dm3_fp8_gemv(_ptr(x[m0:]), m, K, N, _ptr(q), q.stride(0), _ptr(s), s.stride(0), srows, _ptr(bias),
                              bias_kind, _ptr(y[m0:]), N, 1 if out_fp32 else 0, st)
        _lib.check(rc, "dm3_fp8_gemv")
    return y


def gemv_status(device=None) -> int:
    """Reads and clears the tensor-core GEMV's status word on the current device (synchronises)."""
    st = ctypes.c_uint32(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    rc = _lib.load().dm3_gemv_status(ctypes.byref(st), _stream(dev))
    if rc not in (_lib.DM3_OK, _lib.DM3_ETIMEOUT):
        _lib.check(rc, "dm3_gemv_status")
    return int(st.value)


@fp8_gemv.register_fake
def _(x, q, s, bias=None, out_fp32=False):
    return x.new_empty((x.shape[0], q.shape[0]), dtype=torch.float32 if out_fp32 else BF16)


# ----------------------------------------------------------------------------- fp8_gemm
_gemm_workspaces: dict = {}


def gemm_workspace(device: torch.device, nbytes: int) -> Tensor:
    """The zero-initialised scratch of the block-FP8 GEMM on one device (activation image, token
    exponents, status word), grown on demand and shared by calls issued in stream order."""
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _gemm_workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("drama3_b200: the GEMM workspace must be created before CUDA-graph capture; run "
                               "the op once at the largest row count first")
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _gemm_workspaces[key] = ws
    return ws


@torch.library.custom_op("dm3::fp8_gemm", mutates_args=())
def fp8_gemm(x: Tensor, q: Tensor, s: Tensor, bias: Optional[Tensor] = None, out_fp32: bool = False) -> Tensor:
    """y[M, N] = x[M, K] @ dequant(q[N, K], s).T (+ bias) for any row count: the block-FP8 GEMM on
    the tensor cores (where the reference dequantises and calls F.linear, fp8_linear.py:60-61).

    x bf16 [M, K]; q e4m3 [N, K] with unit column stride; s fp32 [N, K/128] (1x128) or
    [ceil(N/128), K/128] (128x128)."""
    _require_cuda(x, q, s, bias)
    lib = _lib.load()
    q = _fp8_bytes(q)
    if x.dtype != BF16:
        raise RuntimeError("fp8_gemm expects bf16 activations")
    x = x.contiguous()
    s = s.contiguous()
    M, K = x.shape
    N = q.shape[0]
    if q.stride(1) != 1 or q.shape[1] != K:
        raise RuntimeError("q must be [N, K] with unit column stride")
    srows = scale_rows(N, s.shape[0])
    y = torch.empty((M, N), dtype=torch.float32 if out_fp32 else BF16, device=x.device)
    bias_kind = 0
    if bias is not None:
        if bias.dtype not in (BF16, torch.float32):
            bias = bias.float()
        bias = bias.contiguous()
        bias_kind = 1 if bias.dtype == BF16 else 2
    if M == 0:
        return y
    ws = gemm_workspace(x.device, lib.dm3_fp8_gemm_workspace_bytes(M, K))
    rc = lib.dm3_fp8_gemm(_ptr(x), M, K, N, _ptr(q), q.stride(0), _ptr(s), s.stride(0), srows, _ptr(bias), bias_kind,
                          _ptr(y), N, 1 if out_fp32 else 0, _ptr(ws), ws.numel(), _stream(x.device))
    _lib.check(rc, "dm3_fp8_gemm")
    return y


@fp8_gemm.register_fake
def _(x, q, s, bias=None, out_fp32=False):
    return x.new_empty((x.shape[0], q.shape[0]), dtype=torch.float32 if out_fp32 else BF16)


# ----------------------------------------------------------------------------- moe_forward
def _expert_strides(w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, H: int):
    E, I2, Hw = w13.shape
    if Hw != H or w13.stride(2) != 1 or w13.stride(1) != H:
        raise RuntimeError("w13 must be [E, 2I, H] with contiguous rows")
    I = I2 // 2
    if tuple(w2.shape[1:]) != (H, I) or w2.stride(2) != 1 or w2.stride(1) != I:
        raise RuntimeError("w2 must be [E, H, I] with contiguous rows")
    srows = scale_rows(I2, s13.shape[1])
    if scale_rows(H, s2.shape[1]) != srows:
        raise RuntimeError("s13 and s2 must use the same scale layout")
    if s13.stride(2) != 1 or s13.stride(1) != s13.shape[2] or s2.stride(2) != 1 or s2.stride(1) != s2.shape[2]:
        raise RuntimeError("scale tables must have contiguous rows")
    return E, I, srows, w13.stride(0) * w13.element_size(), s13.stride(0), w2.stride(0) * w2.element_size(), s2.stride(0)


@torch.library.custom_op("dm3::moe_forward", mutates_args=())
def moe_forward(x: Tensor, ids: Tensor, weights: Tensor, w13: Tensor, s13: Tensor, w2: Tensor,
                s2: Tensor) -> Tensor:
    """Grouped SwiGLU over block-FP8 experts with the caller's routing (fp8_moe_forward)."""
    _require_cuda(x, ids, weights, w13, s13, w2, s2)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    E, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    ids = ids.to(torch.int64).contiguous()
    weights = weights.to(BF16).contiguous()
    k = ids.shape[1]
    y = torch.empty((T, H), dtype=BF16, device=x.device)
    st = _stream(x.device)
    if T > MAX_ROWS:
        # many rows: the grouped tensor-core path (dispatch by expert, one pass over each expert)
        ws = prefill_workspace(x.device, lib.dm3_moe_prefill_workspace_bytes(T, H, I, E, k))
        rc = lib.dm3_moe_grouped(_ptr(x), T, H, I, _ptr(ids), _ptr(weights), k, E, _ptr(w13), w13s, _ptr(s13), s13s,
                                 _ptr(w2), w2s, _ptr(s2), s2s, srows, _ptr(y), None, None, _ptr(ws), ws.numel(), st)
        _lib.check(rc, "dm3_moe_grouped")
        return y
    ws = moe_workspace(x.device, H, I)
    for t0 in range(0, T, MAX_ROWS):
        t = min(MAX_ROWS, T - t0)
        rc = lib.dm3_moe_forward(_ptr(x[t0:]), t, H, I, _ptr(ids[t0:]), _ptr(weights[t0:]), k, E, _ptr(w13), w13s,
                                 _ptr(s13), s13s, _ptr(w2), w2s, _ptr(s2), s2s, srows, _ptr(y[t0:]), _ptr(ws),
                                 ws.numel(), st)
        _lib.check(rc, "dm3_moe_forward")
    return y


@moe_forward.register_fake
def _(x, ids, weights, w13, s13, w2, s2):
    return torch.empty_like(x, dtype=BF16)


# ----------------------------------------------------------------------------- moe_layer
@torch.library.custom_op("dm3::moe_layer", mutates_args=())
def moe_layer(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
              w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor], sh_s13: Optional[Tensor],
              sh_w2: Optional[Tensor], sh_s2: Optional[Tensor], sh_gate: Optional[Tensor],
              out_bias: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor]:
    """Fused decode MoE layer (one launch per 4 rows). Returns (y bf16 [T, H], ids int64 [T, k],
    routing weights bf16 [T, k])."""
    _require_cuda(x, router_w, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    E, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    if router_w.dtype not in (torch.float32, BF16) or tuple(router_w.shape) != (E, H):
        raise RuntimeError("router weight must be fp32 or bf16 [E, H] matching the experts")
    router_w = router_w.contiguous()
    rdt = 0 if router_w.dtype == torch.float32 else 1
    if logit_bias is not None:
        logit_bias = logit_bias.float().contiguous()
    sh_srows = 128
    if sh_w13 is not None:
        sh_w13, sh_w2 = _fp8_bytes(sh_w13).contiguous(), _fp8_bytes(sh_w2).contiguous()
        sh_s13, sh_s2 = sh_s13.contiguous(), sh_s2.contiguous()
        if tuple(sh_w13.shape) != (2 * I, H) or tuple(sh_w2.shape) != (H, I):
            raise RuntimeError("shared expert must be w13 [2I, H], w2 [H, I]")
        sh_srows = scale_rows(2 * I, sh_s13.shape[0])
        if scale_rows(H, sh_s2.shape[0]) != sh_srows:
            raise RuntimeError("shared expert s13 and s2 must use the same scale layout")
    if sh_gate is not None:
        sh_gate = sh_gate.to(BF16).reshape(-1).contiguous()
    if out_bias is not None:
        out_bias = out_bias.float().contiguous()
    y = torch.empty((T, H), dtype=BF16, device=x.device)
    ids = torch.empty((T, top_k), dtype=torch.int64, device=x.device)
    wts = torch.empty((T, top_k), dtype=BF16, device=x.device)
    ws = moe_workspace(x.device, H, I)
    st = _stream(x.device)
    for t0 in range(0, T, MAX_ROWS):
        t = min(MAX_ROWS, T - t0)
        rc = lib.dm3_moe_layer(_ptr(x[t0:]), t, H, I, _ptr(router_w), rdt, E, top_k, 1 if logits_bf16 else 0,
                               _ptr(logit_bias), _ptr(w13), w13s, _ptr(s13), s13s, _ptr(w2), w2s, _ptr(s2), s2s, srows,
                               _ptr(sh_w13), _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2), sh_srows, _ptr(sh_gate),
                               _ptr(out_bias), _ptr(y[t0:]), _ptr(ids[t0:]), _ptr(wts[t0:]), _ptr(ws), ws.numel(), st)
        _lib.check(rc, "dm3_moe_layer")
    return y, ids, wts


@moe_layer.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias):
    T = x.shape[0]
    return (torch.empty_like(x, dtype=BF16), x.new_empty((T, top_k), dtype=torch.int64),
            x.new_empty((T, top_k), dtype=BF16))


# ----------------------------------------------------------------------------- moe_prefill
def _shared_args(sh_w13, sh_s13, sh_w2, sh_s2, H: int, I: int):
    sh_srows = 128
    if sh_w13 is not None:
        sh_w13, sh_w2 = _fp8_bytes(sh_w13).contiguous(), _fp8_bytes(sh_w2).contiguous()
        sh_s13, sh_s2 = sh_s13.contiguous(), sh_s2.contiguous()
        if tuple(sh_w13.shape) != (2 * I, H) or tuple(sh_w2.shape) != (H, I):
            raise RuntimeError("shared expert must be w13 [2I, H], w2 [H, I]")
        sh_srows = scale_rows(2 * I, sh_s13.shape[0])
        if scale_rows(H, sh_s2.shape[0]) != sh_srows:
            raise RuntimeError("shared expert s13 and s2 must use the same scale layout")
    return sh_w13, sh_s13, sh_w2, sh_s2, sh_srows


@torch.library.custom_op("dm3::moe_prefill", mutates_args=())
def moe_prefill(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor], sh_s13: Optional[Tensor],
                sh_w2: Optional[Tensor], sh_s2: Optional[Tensor], sh_gate: Optional[Tensor],
                out_bias: Optional[Tensor]) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Prompt-reading MoE layer over T tokens in one chain of launches. Returns (y bf16 [T, H],
    ids int64 [T, k], routing weights bf16 [T, k], dispatch permutation int64 [T * k] (pair indices
    t * k + j stably sorted by expert), per-expert offsets int64 [E + 1])."""
    _require_cuda(x, router_w, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    E, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    if router_w.dtype != BF16 or tuple(router_w.shape) != (E, H):
        raise RuntimeError("the prefill router weight must be bf16 [E, H] matching the experts")
    router_w = router_w.contiguous()
    if logit_bias is not None:
        logit_bias = logit_bias.float().contiguous()
    sh_w13, sh_s13, sh_w2, sh_s2, sh_srows = _shared_args(sh_w13, sh_s13, sh_w2, sh_s2, H, I)
    if sh_gate is not None:
        sh_gate = sh_gate.to(BF16).reshape(-1).contiguous()
    if out_bias is not None:
        out_bias = out_bias.float().contiguous()
    dev = x.device
    y = torch.empty((T, H), dtype=BF16, device=dev)
    ids = torch.empty((T, top_k), dtype=torch.int64, device=dev)
    wts = torch.empty((T, top_k), dtype=BF16, device=dev)
    perm = torch.empty((T * top_k,), dtype=torch.int64, device=dev)
    offsets = torch.empty((E + 1,), dtype=torch.int64, device=dev)
    ws = prefill_workspace(dev, lib.dm3_moe_prefill_workspace_bytes(T, H, I, E, top_k))
    rc = lib.dm3_moe_prefill(_ptr(x), T, H, I, _ptr(router_w), E, top_k, 1 if logits_bf16 else 0, _ptr(logit_bias),
                             _ptr(w13), w13s, _ptr(s13), s13s, _ptr(w2), w2s, _ptr(s2), s2s, srows, _ptr(sh_w13),
                             _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2), sh_srows, _ptr(sh_gate), _ptr(out_bias), _ptr(y),
                             _ptr(ids), _ptr(wts), _ptr(perm), _ptr(offsets), _ptr(ws), ws.numel(), _stream(dev))
    _lib.check(rc, "dm3_moe_prefill")
    return y, ids, wts, perm, offsets


@moe_prefill.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias):
    T = x.shape[0]
    E = w13.shape[0]
    return (torch.empty_like(x, dtype=BF16), x.new_empty((T, top_k), dtype=torch.int64),
            x.new_empty((T, top_k), dtype=BF16), x.new_empty((T * top_k,), dtype=torch.int64),
            x.new_empty((E + 1,), dtype=torch.int64))


# ----------------------------------------------------------------------------- route
@torch.library.custom_op("dm3::route", mutates_args=())
def route(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool,
          logit_bias: Optional[Tensor]) -> tuple[Tensor, Tensor]:
    """softmax(x @ router_w.T (+ bias)) -> top-k -> renormalise -> bf16 for T tokens (bf16 router).
    Returns (ids int64 [T, k] by descending probability, weights bf16 [T, k])."""
    _require_cuda(x, router_w, logit_bias)
    lib = _lib.load()
    x = x.contiguous()
    T, H = x.shape
    if router_w.dtype != BF16 or router_w.shape[1] != H:
        raise RuntimeError("router weight must be bf16 [E, H]")
    router_w = router_w.contiguous()
    E = router_w.shape[0]
    if logit_bias is not None:
        logit_bias = logit_bias.float().contiguous()
    ids = torch.empty((T, top_k), dtype=torch.int64, device=x.device)
    wts = torch.empty((T, top_k), dtype=BF16, device=x.device)
    ws = prefill_workspace(x.device, lib.dm3_route_workspace_bytes(T, H, E, top_k))
    rc = lib.dm3_route(_ptr(x), T, H, _ptr(router_w), E, top_k, 1 if logits_bf16 else 0, _ptr(logit_bias), _ptr(ids),
                       _ptr(wts), _ptr(ws), ws.numel(), _stream(x.device))
    _lib.check(rc, "dm3_route")
    return ids, wts


@route.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias):
    T = x.shape[0]
    return x.new_empty((T, top_k), dtype=torch.int64), x.new_empty((T, top_k), dtype=BF16)


def set_wait_limit(ns: int) -> None:
    """Time limit (nanoseconds) of every bounded device-side wait on the current device; 1 s by
    default. A wait that runs out sets the timeout bit of the status word (moe_status) and the
    kernel stops its work. Call while no kernel of the library runs on the device."""
    _lib.check(_lib.load().dm3_set_wait_limit_ns(int(ns)), "dm3_set_wait_limit_ns")


def noalloc_status() -> int:
    """Status word of the allocation-free layer's static scratch on the current device (synchronises);
    a non-zero word also clears the scratch so that the next call starts clean."""
    st = ctypes.c_uint32(0)
    rc = _lib.load().dm3_moe_noalloc_status(ctypes.byref(st), _stream(torch.device("cuda", torch.cuda.current_device())))
    if rc not in (_lib.DM3_OK, _lib.DM3_ETIMEOUT):
        _lib.check(rc, "dm3_moe_noalloc_status")
    return int(st.value)


# ----------------------------------------------------------------------------- audio head
_head_workspaces: dict = {}


def _head_workspace(device: torch.device, nbytes: int) -> Tensor:
    dev = torch.device(device)
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _head_workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("drama3_b200: run the audio head once before CUDA-graph capture")
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=dev)
        _head_workspaces[key] = ws
    return ws


@torch.library.custom_op("dm3::audio_head", mutates_args=("vocab",))
def audio_head(hidden: Tensor, q: Tensor, s: Tensor, strength: Tensor, candidates: Tensor, vocab: Tensor,
               rows: Optional[Tensor] = None, round_bf16: bool = True) -> tuple[Tensor, Tensor]:
    """The CFG audio head of one frame (engine.py:423-424): logits = (hidden @ head.T).float() with the
    block-FP8 head (rows `rows` of q when given, else q itself), then vocab[candidates] = l1 + strength *
    (l0 - l1) in place (the -inf buffer of CfgGraphs), and each row's log-sum-exp for direction_score.
    hidden bf16 [2, K]; strength fp32 device scalar; candidates int64 [Nc]. Returns (logits fp32 [2, Nc],
    lse fp32 [2])."""
    _require_cuda(hidden, q, s, strength, candidates, vocab, rows)
    lib = _lib.load()
    q = _fp8_bytes(q)
    hidden = hidden.to(BF16).contiguous()
    if hidden.dim() != 2 or hidden.shape[0] != 2:
        raise RuntimeError("the audio head takes the 2 guidance rows [2, K]")
    K = hidden.shape[1]
    Nc = candidates.numel()
    if q.stride(1) != 1 or q.shape[1] != K:
        raise RuntimeError("q must be [rows, K] with unit column stride")
    if vocab.dtype != torch.float32 or not vocab.is_contiguous():
        raise RuntimeError("vocab must be a contiguous fp32 buffer")
    if strength.dtype != torch.float32 or strength.numel() != 1:
        raise RuntimeError("strength must be a one-element fp32 device tensor")
    candidates = candidates.to(torch.int64).contiguous()
    if rows is not None:
        rows = rows.to(torch.int64).contiguous()
        if rows.numel() != Nc:
            raise RuntimeError("rows and candidates must have the same length")
    else:
        if q.shape[0] != Nc:
            raise RuntimeError("without rows, q must hold exactly the candidate rows")
    srows = scale_rows(q.shape[0], s.shape[0])
    s = s.contiguous()
    logits = torch.empty((2, Nc), dtype=torch.float32, device=hidden.device)
    lse = torch.empty((2,), dtype=torch.float32, device=hidden.device)
    ws = _head_workspace(hidden.device, lib.dm3_audio_head_workspace_bytes(Nc))
    rc = lib.dm3_audio_head(_ptr(hidden), K, _ptr(q), q.stride(0), _ptr(s), s.stride(0), srows, _ptr(rows), q.shape[0],
                            Nc, _ptr(strength), _ptr(candidates), _ptr(vocab), vocab.numel(), _ptr(logits), _ptr(lse),
                            1 if round_bf16 else 0, _ptr(ws), ws.numel(), _stream(hidden.device))
    _lib.check(rc, "dm3_audio_head")
    return logits, lse


@audio_head.register_fake
def _(hidden, q, s, strength, candidates, vocab, rows=None, round_bf16=True):
    return (hidden.new_empty((2, candidates.numel()), dtype=torch.float32), hidden.new_empty((2,), dtype=torch.float32))


@torch.library.custom_op("dm3::direction_score", mutates_args=("score",))
def direction_score(logits: Tensor, lse: Tensor, token: Tensor, eos_id: int, semantic_begin: int,
                    score: Tensor) -> None:
    """score += log_softmax(logits)[0, i] - log_softmax(logits)[1, i] with i = 0 for the eos token and
    token - semantic_begin + 1 otherwise (engine.py:476-479), all on the device (token int64 scalar)."""
    _require_cuda(logits, lse, token, score)
    if score.dtype != torch.float32 or token.dtype != torch.int64:
        raise RuntimeError("score must be fp32 and token int64")
    rc = _lib.load().dm3_direction_score(_ptr(logits), _ptr(lse), logits.shape[1], _ptr(token), int(eos_id),
                                         int(semantic_begin), _ptr(score), _stream(logits.device))
    _lib.check(rc, "dm3_direction_score")


@direction_score.register_fake
def _(logits, lse, token, eos_id, semantic_begin, score):
    return None
