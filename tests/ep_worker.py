"""Per-rank bodies of the expert-parallel tests, importable by spawned processes."""

from __future__ import annotations

import os
import traceback

import torch


def _init(rank: int, world: int, store: str, backend: str):
    import datetime

    import torch.distributed as dist

    dist.init_process_group(backend, init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    return dist


def cpu_rank(rank: int, world: int, store: str, out_dir: str) -> None:
    """gloo rank of the CPU expert-parallel restatement: every rank builds the same seeded layer,
    runs its share through oracle.ep_oracle and writes (y, ids, w) for the parent to check."""
    try:
        dist = _init(rank, world, store, "gloo")
        import oracle
        from oracle import ep_oracle
        from tests.golden import inputs
        from tests.helpers import experts, oracle_shared, routed_layer

        h, i, e, k, t = 256, 128, 16, 4, 24
        layer = routed_layer(400, h=h, i=i, e=e)
        bias = inputs.zipf_bias(401, e=e)
        x = inputs.decode_rows(t, seed=402, h=h)
        el = e // world
        local = {n: v[rank * el:(rank + 1) * el] for n, v in layer["experts"].items()}
        tl = t // world
        xs = x[rank * tl:(rank + 1) * tl]
        y, ids, w = ep_oracle.ep_rank_layer(xs, layer["gate"], local, e, k, logit_bias=bias,
                                            sw=oracle_shared(layer, 128), g=layer["sh_gate"])
        torch.save({"y": y, "ids": ids, "w": w}, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.destroy_process_group()
    except Exception:  # reported to the parent through the missing result file
        traceback.print_exc()
        raise


def gpu_rank(rank: int, world: int, store: str, out_dir: str) -> None:
    """One GPU per rank: the expert-parallel prefill (fused op, then the ep_dispatch / ep_combine
    halves, then a CUDA-graph replay) on this rank's tokens and experts, against the one-GPU
    dm3::moe_prefill of all tokens computed on this rank's GPU."""
    try:
        torch.cuda.set_device(rank)
        dist = _init(rank, world, store, "gloo")
        import drama3_b200 as dm3

        dev = torch.device("cuda", rank)
        H, I, E, K, T = 2048, 512, 256, 8, 512
        g = torch.Generator(device=dev).manual_seed(500)
        gate = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w13, s13 = dm3.fp8_block(torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02)
        w2, s2 = dm3.fp8_block(torch.randn(E, H, I, generator=g, device=dev) * 0.02)
        sh13, shs13 = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
        sh2, shs2 = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
        shg = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        gx = torch.Generator(device="cpu").manual_seed(501)
        rank_e = torch.randperm(E, generator=gx).float() + 1.0
        bias = (-1.1 * torch.log(rank_e)).to(dev)
        x = torch.randn(T, H, generator=g, device=dev)
        x = (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
        ref_y, ref_ids, ref_w, _, _ = dm3.ops.moe_prefill(x, gate, K, True, bias, w13, s13, w2, s2, sh13, shs13, sh2,
                                                           shs2, shg, None)
        el, tl = E // world, T // world
        lw = (w13[rank * el:(rank + 1) * el], s13[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el],
              s2[rank * el:(rank + 1) * el])
        xs = x[rank * tl:(rank + 1) * tl].contiguous()
        grp = dm3.ep.ExpertParallel(tl, H, K)
        res = {}
        y, ids, w = grp.moe_prefill(xs, gate, K, True, bias, *lw, sh13, shs13, sh2, shs2, shg, None)
        torch.cuda.synchronize()
        sl = slice(rank * tl, (rank + 1) * tl)
        res["fused_ids"] = bool(torch.equal(ids, ref_ids[sl]))
        res["fused_w"] = bool(torch.equal(w, ref_w[sl]))
        res["fused_y"] = bool(torch.equal(y, ref_y[sl]))
        res["fused_maxdiff"] = float((y.float() - ref_y[sl].float()).abs().max())
        # the two halves as separate ops, twice (the per-call epoch advances)
        for rep in range(2):
            ids2, w2_ = dm3.ep.ep_dispatch(xs, gate, K, True, bias, shg, I, world, rank, tl, grp.arenas)
            y2 = dm3.ep.ep_combine(xs, gate, K, *lw, sh13, shs13, sh2, shs2, shg, None, world, rank, tl, grp.arenas)
            torch.cuda.synchronize()
            res[f"split_y{rep}"] = bool(torch.equal(y2, ref_y[sl])) and bool(torch.equal(ids2, ref_ids[sl]))
        # CUDA graph capture and replay on every rank
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gy, _, _ = grp.moe_prefill(xs, gate, K, True, bias, *lw, sh13, shs13, sh2, shs2, shg, None)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        res["graph_y"] = bool(torch.equal(gy, ref_y[sl]))
        # a load-balanced placement: this rank holds the experts the table gives it, in local order
        owner = dm3.ep.balanced_placement(torch.exp(bias.float().cpu()), world)
        mine = dm3.ep.local_experts(owner, rank).to(dev)
        lw_b = (w13[mine], s13[mine], w2[mine], s2[mine])
        yb, idsb, _ = grp.moe_prefill(xs, gate, K, True, bias, *lw_b, sh13, shs13, sh2, shs2, shg, None,
                                      owner=owner.to(dev))
        torch.cuda.synchronize()
        res["placed_y"] = bool(torch.equal(yb, ref_y[sl])) and bool(torch.equal(idsb, ref_ids[sl]))
        # the sharded decode layer (2 rows): every rank the same rows, its own contiguous experts
        x2 = x[:2].contiguous()
        obias = torch.randn(H, generator=g, device=dev) * 0.02
        dref = dm3.ops.moe_layer(x2, gate, K, True, bias, w13, s13, w2, s2, sh13, shs13, sh2, shs2, shg, obias)
        lwc = (w13[rank * el:(rank + 1) * el], s13[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el],
               s2[rank * el:(rank + 1) * el])
        ok = True
        for rep in range(3):
            dy, dids, dw = grp.moe_layer(x2, gate, K, True, bias, *lwc, sh13, shs13, sh2, shs2, shg, obias)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(dids, dref[1])) and bool(torch.equal(dw, dref[2]))
            err = float((dy.float() - dref[0].float()).norm() / dref[0].float().norm())
            ok = ok and err < 1e-3
            res[f"decode_err{rep}"] = err
        dist.barrier()
        dgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(dgraph):
            gdy = grp.moe_layer(x2, gate, K, True, bias, *lwc, sh13, shs13, sh2, shs2, shg, obias)[0]
        for _ in range(3):
            dgraph.replay()
        torch.cuda.synchronize()
        res["decode_graph_err"] = float((gdy.float() - dref[0].float()).norm() / dref[0].float().norm())
        res["decode_ok"] = ok and res["decode_graph_err"] < 1e-3
        res["decode_status"] = dm3.ops.moe_status(dm3.ops.moe_workspace(dev, H, I))
        del dgraph
        ws = dm3.ep._ep_workspaces[rank]
        res["status"] = dm3.ops.moe_status(ws)
        del graph
        grp.close()
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.destroy_process_group()
    except Exception:
        traceback.print_exc()
        raise
