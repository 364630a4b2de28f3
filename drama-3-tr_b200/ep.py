"""Expert-parallel prefill MoE over NVLink (one process per GPU).

The reference spreads a prompt's tokens over the experts with ids.unique() / slot_map on one
device (OnDemandExperts.forward, engine.py:138-147). Here each of `world` ranks owns
E / world experts (contiguous blocks, or as a placement table assigns them: `balanced_placement`
on expected loads, `tile_balanced_placement` on observed ones) and routes its own share of the
tokens. The kernels write every (token, k) pair's rows straight into the owning rank's arena and
every output row straight back into the source rank's arena over NVLink, with per-call epoch
flags; there is no host synchronisation, so a call can be captured into a CUDA graph (every rank
must capture and replay the same sequence).

Arenas are plain cudaMalloc allocations shared by CUDA IPC: `ExpertParallel` allocates this
rank's arena, all-gathers the 64-byte IPC handles over the given torch.distributed group (any
backend) and maps every other rank's arena.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional

import torch
from torch import Tensor

from . import _lib
from .ops import BF16, _expert_strides, _fp8_bytes, _ptr, _require_cuda, _shared_args, _stream

MAX_RANKS = 8
_ep_workspaces: dict = {}


def _arena_array(arenas: List[int]):
    arr = (ctypes.c_void_p * MAX_RANKS)()
    for i, a in enumerate(arenas):
        arr[i] = a
    return arr


def balanced_placement(load: Tensor, world: int) -> Tensor:
    """A placement of E experts over `world` ranks, E / world each, that evens out the expected
    load: experts by descending load, each to the rank with the least load among those with room
    (greedy longest-processing-time). Returns int32 [E] of (rank << 16) | local index, local
    indices in ascending expert order on each rank."""
    E = load.numel()
    el = E // world
    order = torch.argsort(load.double().cpu(), descending=True, stable=True).tolist()
    tot = [0.0] * world
    members: list = [[] for _ in range(world)]
    for e in order:
        r = min((r for r in range(world) if len(members[r]) < el), key=lambda r: (tot[r], r))
        members[r].append(e)
        tot[r] += float(load[e])
    owner = torch.empty(E, dtype=torch.int32)
    for r in range(world):
        for i, e in enumerate(sorted(members[r])):
            owner[e] = (r << 16) | i
    return owner


def tile_balanced_placement(counts: Tensor, world: int, tile_tokens: int = 64) -> Tensor:
    """A placement from observed routing: `counts` [E] are the (token, k) pairs each expert received
    over a calibration batch. Balances the experts' tiles of `tile_tokens` tokens rather than their
    pairs: the expert kernels stream each tile's weights once, so a rank's time follows its tiles (a
    cold expert with 3 tokens costs a whole tile). Same return value as `balanced_placement`."""
    c = counts.double().cpu()
    tiles = torch.ceil(c / float(tile_tokens))
    # pairs break ties between experts of equal tiles; the floor spreads unused experts evenly
    return balanced_placement(tiles + c * 1e-4 + 1e-6, world)


def local_experts(owner: Tensor, rank: int) -> Tensor:
    """The global ids of `rank`'s experts in local index order under a placement."""
    o = owner.cpu().long()
    mine = torch.nonzero((o >> 16) == rank).flatten()
    return mine[torch.argsort(o[mine] & 0xFFFF)]


def ep_workspace(device: torch.device, nbytes: int) -> Tensor:
    """The expert-parallel scratch of this rank (grown on demand, zero-initialised)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    ws = _ep_workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("drama3_b200: the expert-parallel workspace must exist before CUDA-graph capture")
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _ep_workspaces[key] = ws
    return ws


class ExpertParallel:
    """The NVLink arenas of one expert-parallel group.

    tokens_per_rank: the most tokens any rank passes to one call; hidden / top_k: the layer's H and k.
    group: the torch.distributed process group of the ranks (default: the world)."""

    def __init__(self, tokens_per_rank: int, hidden: int, top_k: int = 8, group=None):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= MAX_RANKS:
            raise RuntimeError(f"expert parallelism takes 2 to {MAX_RANKS} ranks, got {self.world}")
        self.tokens_per_rank, self.hidden, self.top_k = tokens_per_rank, hidden, top_k
        lib = _lib.load()
        nbytes = lib.dm3_ep_arena_bytes(self.world, tokens_per_rank, top_k, hidden)
        own = ctypes.c_void_p()
        _lib.check(lib.dm3_ep_alloc(nbytes, ctypes.byref(own)), "dm3_ep_alloc")
        self._own = own.value
        handle = (ctypes.c_char * 64)()
        _lib.check(lib.dm3_ep_ipc_handle(ctypes.c_void_p(self._own), handle), "dm3_ep_ipc_handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.arenas: List[int] = []
        self._opened: List[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.arenas.append(self._own)
                continue
            ptr = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(h, 64)
            _lib.check(lib.dm3_ep_ipc_open(buf, ctypes.byref(ptr)), "dm3_ep_ipc_open")
            self.arenas.append(ptr.value)
            self._opened.append(ptr.value)
        dist.barrier(group)

    def close(self) -> None:
        """Unmaps the peers' arenas and frees this rank's (after every rank is done with it)."""
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(self.group)
        lib = _lib.load()
        for ptr in self._opened:
            lib.dm3_ep_ipc_close(ctypes.c_void_p(ptr))
        dist.barrier(self.group)
        lib.dm3_ep_free(ctypes.c_void_p(self._own))
        self._own = None
        self._opened = []

    def moe_prefill(self, x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                    w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor] = None,
                    sh_s13: Optional[Tensor] = None, sh_w2: Optional[Tensor] = None, sh_s2: Optional[Tensor] = None,
                    sh_gate: Optional[Tensor] = None, out_bias: Optional[Tensor] = None,
                    owner: Optional[Tensor] = None):
        """This rank's part of the prefill layer: x [T, H] its tokens, w13 / s13 / w2 / s2 its
        E / world experts (contiguous blocks, or as `owner` places them). Returns (y [T, H],
        ids [T, k], routing weights [T, k])."""
        return moe_prefill_ep(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2,
                              sh_s2, sh_gate, out_bias, self.world, self.rank, self.tokens_per_rank, self.arenas,
                              owner)

    def moe_layer(self, x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                  w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor] = None,
                  sh_s13: Optional[Tensor] = None, sh_w2: Optional[Tensor] = None, sh_s2: Optional[Tensor] = None,
                  sh_gate: Optional[Tensor] = None, out_bias: Optional[Tensor] = None):
        """The sharded decode layer: every rank the same rows x, its own E / world experts (contiguous
        blocks); returns the whole layer's (y, ids, routing weights) on every rank."""
        return moe_layer_ep(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2,
                            sh_s2, sh_gate, out_bias, self.world, self.rank, self.tokens_per_rank, self.arenas)


@torch.library.custom_op("dm3::moe_layer_ep", mutates_args=())
def moe_layer_ep(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                 w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor], sh_s13: Optional[Tensor],
                 sh_w2: Optional[Tensor], sh_s2: Optional[Tensor], sh_gate: Optional[Tensor],
                 out_bias: Optional[Tensor], world: int, rank: int, tokens_per_rank: int,
                 arenas: List[int]) -> tuple[Tensor, Tensor, Tensor]:
    """The fused decode MoE layer sharded over the ranks: every rank passes the same rows and router,
    its own experts (contiguous blocks), and gets the whole layer's output (<= 4 rows per launch)."""
    from .ops import MAX_ROWS, moe_workspace

    _require_cuda(x, router_w, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    El, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    E = router_w.shape[0]
    if router_w.dtype not in (torch.float32, BF16) or router_w.shape[1] != H or E != El * world:
        raise RuntimeError("router weight must be fp32 or bf16 [world x local experts, H]")
    router_w = router_w.contiguous()
    rdt = 0 if router_w.dtype == torch.float32 else 1
    if logit_bias is not None:
        logit_bias = logit_bias.float().contiguous()
    sh_w13, sh_s13, sh_w2, sh_s2, sh_srows = _shared_args(sh_w13, sh_s13, sh_w2, sh_s2, H, I)
    if sh_gate is not None:
        sh_gate = sh_gate.to(BF16).reshape(-1).contiguous()
    if out_bias is not None:
        out_bias = out_bias.float().contiguous()
    y = torch.empty((T, H), dtype=BF16, device=x.device)
    ids = torch.empty((T, top_k), dtype=torch.int64, device=x.device)
    wts = torch.empty((T, top_k), dtype=BF16, device=x.device)
    ws = moe_workspace(x.device, H, I)
    st = _stream(x.device)
    arr = _arena_array(arenas)
    for t0 in range(0, T, MAX_ROWS):
        t = min(MAX_ROWS, T - t0)
        rc = lib.dm3_moe_layer_ep(_ptr(x[t0:]), t, H, I, _ptr(router_w), rdt, E, top_k, 1 if logits_bf16 else 0,
                                  _ptr(logit_bias), _ptr(w13), w13s, _ptr(s13), s13s, _ptr(w2), w2s, _ptr(s2), s2s,
                                  srows, _ptr(sh_w13), _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2), sh_srows, _ptr(sh_gate),
                                  _ptr(out_bias), _ptr(y[t0:]), _ptr(ids[t0:]), _ptr(wts[t0:]), world, rank,
                                  tokens_per_rank, arr, _ptr(ws), ws.numel(), st)
        _lib.check(rc, "dm3_moe_layer_ep")
    return y, ids, wts


@moe_layer_ep.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias,
      world, rank, tokens_per_rank, arenas):
    T = x.shape[0]
    return (torch.empty_like(x, dtype=BF16), x.new_empty((T, top_k), dtype=torch.int64),
            x.new_empty((T, top_k), dtype=BF16))


def _owner(owner: Optional[Tensor], E: int) -> Optional[Tensor]:
    if owner is None:
        return None
    if owner.numel() != E or not owner.is_cuda:
        raise RuntimeError("owner must be an int32 [E] device tensor")
    return owner.to(torch.int32).contiguous()


def _ep_checks(x: Tensor, router_w: Tensor, world: int, E_local: int):
    if router_w.dtype != BF16 or router_w.shape[1] != x.shape[1]:
        raise RuntimeError("the router weight must be bf16 [E, H]")
    if router_w.shape[0] != E_local * world:
        raise RuntimeError("the router width must be world x the experts held by this rank")


@torch.library.custom_op("dm3::moe_prefill_ep", mutates_args=())
def moe_prefill_ep(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                   w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor, sh_w13: Optional[Tensor], sh_s13: Optional[Tensor],
                   sh_w2: Optional[Tensor], sh_s2: Optional[Tensor], sh_gate: Optional[Tensor],
                   out_bias: Optional[Tensor], world: int, rank: int, tokens_per_rank: int,
                   arenas: List[int], owner: Optional[Tensor] = None) -> tuple[Tensor, Tensor, Tensor]:
    """Expert-parallel prefill layer (routing, NVLink dispatch, local experts, NVLink return,
    combine) for this rank's tokens."""
    _require_cuda(x, router_w, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias, owner)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    El, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    _ep_checks(x, router_w, world, El)
    E = router_w.shape[0]
    router_w = router_w.contiguous()
    owner = _owner(owner, E)
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
    ws = ep_workspace(dev, lib.dm3_moe_prefill_ep_workspace_bytes(world, tokens_per_rank, H, I, E, top_k))
    rc = lib.dm3_moe_prefill_ep(_ptr(x), T, H, I, _ptr(router_w), E, top_k, 1 if logits_bf16 else 0,
                                _ptr(logit_bias), _ptr(w13), w13s, _ptr(s13), s13s, _ptr(w2), w2s, _ptr(s2), s2s,
                                srows, _ptr(sh_w13), _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2), sh_srows, _ptr(sh_gate),
                                _ptr(out_bias), _ptr(y), _ptr(ids), _ptr(wts), world, rank, tokens_per_rank,
                                _arena_array(arenas), _ptr(owner), _ptr(ws), ws.numel(), _stream(dev))
    _lib.check(rc, "dm3_moe_prefill_ep")
    return y, ids, wts


@moe_prefill_ep.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias,
      world, rank, tokens_per_rank, arenas, owner=None):
    T = x.shape[0]
    return (torch.empty_like(x, dtype=BF16), x.new_empty((T, top_k), dtype=torch.int64),
            x.new_empty((T, top_k), dtype=BF16))


@torch.library.custom_op("dm3::ep_dispatch", mutates_args=())
def ep_dispatch(x: Tensor, router_w: Tensor, top_k: int, logits_bf16: bool, logit_bias: Optional[Tensor],
                sh_gate: Optional[Tensor], intermediate: int, world: int, rank: int, tokens_per_rank: int,
                arenas: List[int], owner: Optional[Tensor] = None) -> tuple[Tensor, Tensor]:
    """First half of the expert-parallel layer: routes this rank's tokens and sends every (token, k)
    pair to the rank owning its expert. Returns (ids [T, k], routing weights [T, k]); the pairs'
    state stays in this rank's workspace and the owners' arenas for ep_combine."""
    _require_cuda(x, router_w, logit_bias, sh_gate)
    lib = _lib.load()
    x = x.contiguous()
    T, H = x.shape
    E = router_w.shape[0]
    if router_w.dtype != BF16 or router_w.shape[1] != H or E % world:
        raise RuntimeError("the router weight must be bf16 [E, H] with E divisible by the world size")
    router_w = router_w.contiguous()
    if logit_bias is not None:
        logit_bias = logit_bias.float().contiguous()
    if sh_gate is not None:
        sh_gate = sh_gate.to(BF16).reshape(-1).contiguous()
    owner = _owner(owner, E)
    ids = torch.empty((T, top_k), dtype=torch.int64, device=x.device)
    wts = torch.empty((T, top_k), dtype=BF16, device=x.device)
    ws = ep_workspace(x.device, lib.dm3_moe_prefill_ep_workspace_bytes(world, tokens_per_rank, H, intermediate, E,
                                                                         top_k))
    rc = lib.dm3_ep_dispatch(_ptr(x), T, H, intermediate, _ptr(router_w), E, top_k, 1 if logits_bf16 else 0,
                             _ptr(logit_bias), _ptr(sh_gate), _ptr(ids), _ptr(wts), world, rank, tokens_per_rank,
                             _arena_array(arenas), _ptr(owner), _ptr(ws), ws.numel(), _stream(x.device))
    _lib.check(rc, "dm3_ep_dispatch")
    return ids, wts


@ep_dispatch.register_fake
def _(x, router_w, top_k, logits_bf16, logit_bias, sh_gate, intermediate, world, rank, tokens_per_rank, arenas,
      owner=None):
    T = x.shape[0]
    return x.new_empty((T, top_k), dtype=torch.int64), x.new_empty((T, top_k), dtype=BF16)


@torch.library.custom_op("dm3::ep_combine", mutates_args=())
def ep_combine(x: Tensor, router_w: Tensor, top_k: int, w13: Tensor, s13: Tensor, w2: Tensor, s2: Tensor,
               sh_w13: Optional[Tensor], sh_s13: Optional[Tensor], sh_w2: Optional[Tensor], sh_s2: Optional[Tensor],
               sh_gate: Optional[Tensor], out_bias: Optional[Tensor], world: int, rank: int, tokens_per_rank: int,
               arenas: List[int]) -> Tensor:
    """Second half: this rank's experts over the pairs every rank sent here, the output rows sent
    back to their sources, and this rank's tokens combined (+ shared expert, + bias)."""
    _require_cuda(x, router_w, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias)
    lib = _lib.load()
    w13, w2 = _fp8_bytes(w13), _fp8_bytes(w2)
    x = x.contiguous()
    T, H = x.shape
    El, I, srows, w13s, s13s, w2s, s2s = _expert_strides(w13, s13, w2, s2, H)
    _ep_checks(x, router_w, world, El)
    E = router_w.shape[0]
    sh_w13, sh_s13, sh_w2, sh_s2, sh_srows = _shared_args(sh_w13, sh_s13, sh_w2, sh_s2, H, I)
    if sh_gate is not None:
        sh_gate = sh_gate.to(BF16).reshape(-1).contiguous()
    if out_bias is not None:
        out_bias = out_bias.float().contiguous()
    y = torch.empty((T, H), dtype=BF16, device=x.device)
    ws = ep_workspace(x.device, lib.dm3_moe_prefill_ep_workspace_bytes(world, tokens_per_rank, H, I, E, top_k))
    rc = lib.dm3_ep_combine(_ptr(x), T, H, I, _ptr(router_w.contiguous()), E, top_k, _ptr(w13), w13s, _ptr(s13), s13s,
                            _ptr(w2), w2s, _ptr(s2), s2s, srows, _ptr(sh_w13), _ptr(sh_s13), _ptr(sh_w2), _ptr(sh_s2),
                            sh_srows, _ptr(sh_gate), _ptr(out_bias), _ptr(y), world, rank, tokens_per_rank,
                            _arena_array(arenas), _ptr(ws), ws.numel(), _stream(x.device))
    _lib.check(rc, "dm3_ep_combine")
    return y


@ep_combine.register_fake
def _(x, router_w, top_k, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2, sh_gate, out_bias, world, rank,
      tokens_per_rank, arenas):
    return torch.empty_like(x, dtype=BF16)
