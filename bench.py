#!/usr/bin/env python
"""Benchmark of the Drama-3 decode MoE feed-forward on B200.

Default workload (`--workload decode`): 40 stacked MoE decode layers of the Drama-3 backbone
shape (hidden 2048, 256 routed block-FP8 experts of intermediate 512 with 128x128 fp32 scales,
top-8 softmax routing by a bf16 router, and an always-on block-FP8 shared expert behind a sigmoid
gate). Each layer has independently seeded weights (N(0, 0.02)) and its own seeded 2-row input
(conditional + unconditional guidance rows, N(0, 1) RMS-normalised, bf16). One step = one frame =
the 40 layers, captured once in a CUDA graph and replayed. Weights total 30 GiB, far above the
126 MB L2, so every replay streams them from HBM (no flush needed).

Prints one JSON line: `value` = layer-frames per second over all ranks (device time, CUDA events,
max over ranks), `us_per_layer`, the roofline of the fused MoE kernel against the measured HBM
copy bandwidth, the CPU baseline (the reference's torch path on host cores), the end-to-end
number through the public op with host buffers, and SM clocks sampled during the timed region.

`--impl reference` times the reference's CPU implementation of the same layer (torch fp32 on all
host cores) with the same metric. Other workloads: `--workload speaker` (40 distilled-speaker
layers, 32 experts, fp32 router, bias) and `--workload gemv` (block-FP8 GEMV sweep).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

H, I, E, TOPK, T = 2048, 512, 256, 8, 2
EXPERT_BYTES = 2 * I * H + H * I + (2 * I // 128) * (H // 128) * 4 + (H // 128) * (I // 128) * 4  # 3,146,496
METRIC = "MoE decode layer throughput (2-row frame x layer / s); us/layer = 1e6 / (value / n_gpus)"
PF_T = 512
SPEAKER_FRAMES = 300  # the distilled-speaker workload: consecutive frames, each with its own rows
PF_METRIC = "prefill MoE layer throughput (tokens / s), T=512 prompt rows, Zipf(1.1)-skewed routing"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def recorded_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(kernel)
    return None


# ----------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [v for v in sm if v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- workload
def rms(x):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)


def make_layer(seed: int, dev, experts=E, router_dtype=torch.bfloat16, shared=True, bias=False):
    import drama3_b200 as dm3

    g = torch.Generator(device=dev).manual_seed(seed)
    L = {"gate": (torch.randn(experts, H, generator=g, device=dev) * 0.02).to(router_dtype)}
    L["w13"], L["s13"] = dm3.fp8_block(torch.randn(experts, 2 * I, H, generator=g, device=dev) * 0.02)
    L["w2"], L["s2"] = dm3.fp8_block(torch.randn(experts, H, I, generator=g, device=dev) * 0.02)
    if shared:
        L["sh_w13"], L["sh_s13"] = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
        L["sh_w2"], L["sh_s2"] = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
        L["sh_gate"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    if bias:
        L["bias"] = torch.randn(H, generator=g, device=dev) * 0.02
    L["x"] = rms(torch.randn(T, H, generator=g, device=dev)).to(torch.bfloat16)
    return L


def layer_call(L, x, logits_bf16=True):
    import drama3_b200 as dm3

    return dm3.ops.moe_layer(x, L["gate"], TOPK, logits_bf16, None, L["w13"], L["s13"], L["w2"], L["s2"],
                             L.get("sh_w13"), L.get("sh_s13"), L.get("sh_w2"), L.get("sh_s2"), L.get("sh_gate"),
                             L.get("bias"))


def layer_bytes(L, ids: torch.Tensor) -> int:
    """Algorithmic HBM bytes of one layer: each distinct routed expert once (weights + scales),
    the router, the shared expert and its gate row, the bias, and the activations in and out."""
    u = int(torch.unique(ids).numel())
    b = u * EXPERT_BYTES + L["gate"].numel() * L["gate"].element_size() + 2 * T * H * 2
    if "sh_w13" in L:
        b += EXPERT_BYTES + H * 2
    if "bias" in L:
        b += H * 4
    return b


def cpu_layer(L) -> dict:
    return {k: v.cpu() for k, v in L.items()}


def time_cpu_port(layers_cpu, budget_s: float):
    """Times oracle.cpu_port.decode_layer on host cores; returns (layer-frames/s, reps, threads)."""
    from oracle import cpu_port

    torch.set_num_threads(os.cpu_count() or 1)
    cpu_port.decode_layer(layers_cpu[0]["x"], layers_cpu[0])  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        L = layers_cpu[reps % len(layers_cpu)]
        cpu_port.decode_layer(L["x"], L)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 200:
            break
    return reps / el, reps, torch.get_num_threads()


def all_ranks_true(flag: bool, world: int) -> bool:
    """True when `flag` holds on every rank (every rank takes this collective at the same point)."""
    if world == 1:
        return flag
    import torch.distributed as dist

    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def check_decode_sharded(grp, world, rank, dev) -> dict:
    """The sharded decode layer against the one-GPU layer on this rank's GPU, same seeded full layer
    on every rank: ids and routing weights identical, outputs within 1e-3 relative L2 (the partial
    sums meet in another order), status word clear."""
    import drama3_b200 as dm3

    L = make_layer(4321, dev)  # identical on every rank (same seed, same generator)
    ref = layer_call(L, L["x"])
    el = E // world
    sl = slice(rank * el, (rank + 1) * el)
    errs, ok = [], True
    for _ in range(2):  # twice: the per-call epoch advances
        y, ids, w = grp.moe_layer(L["x"], L["gate"], TOPK, True, None, L["w13"][sl], L["s13"][sl], L["w2"][sl],
                                  L["s2"][sl], L["sh_w13"], L["sh_s13"], L["sh_w2"], L["sh_s2"], L["sh_gate"], None)
        torch.cuda.synchronize()
        err = float((y.float() - ref[0].float()).norm() / ref[0].float().norm())
        errs.append(err)
        ok = ok and torch.equal(ids, ref[1]) and torch.equal(w, ref[2]) and err < 1e-3
    ok = ok and dm3.ops.moe_status(dm3.ops.moe_workspace(dev, H, I)) == 0
    del L
    ok = all_ranks_true(ok, world)
    return {"ok": ok, "against": "dm3::moe_layer of the full layer on this rank's GPU (ids, weights equal; y rel-L2)",
            "rel_l2": [round(e, 7) for e in errs]}


def observed_placement(gate, logit_bias, world: int, dev, seed: int):
    """Expert placement from observed loads, as a deployment would calibrate it: route a seeded
    calibration batch of PF_T rows (not the measured rows) through the layer's router once and balance
    the experts' 64-token tiles over the ranks (greedy LPT, equal experts per rank): an expert kernel's
    time follows its tiles, each a fixed amount of weight streaming, more than its pairs."""
    import drama3_b200 as dm3

    g = torch.Generator(device=dev).manual_seed(seed)
    calib = rms(torch.randn(PF_T, H, generator=g, device=dev)).to(torch.bfloat16)
    ids, _ = dm3.ops.route(calib, gate, TOPK, True, logit_bias)
    return dm3.ep.tile_balanced_placement(torch.bincount(ids.flatten(), minlength=E), world)


def check_prefill_ep(grp, world, rank, dev, placement) -> dict:
    """The expert-parallel prefill against the one-GPU prefill of all 512 tokens on this rank's GPU,
    the same seeded full layer on every rank: this rank's outputs, ids and weights bit-identical,
    status word clear."""
    import drama3_b200 as dm3

    L = make_prefill_layer(4322, dev)
    ref = prefill_call(L, L["x"])
    tl = PF_T // world
    owner = None
    if placement in ("balanced", "observed"):
        owner = (observed_placement(L["gate"], L["logit_bias"], world, dev, 4322 + 13) if placement == "observed"
                 else dm3.ep.balanced_placement(torch.exp(L["logit_bias"].float().cpu()), world))
        mine = dm3.ep.local_experts(owner, rank).to(dev)
        owner = owner.to(dev)
    else:
        mine = torch.arange(rank * (E // world), (rank + 1) * (E // world), device=dev)
    lw = (L["w13"][mine], L["s13"][mine], L["w2"][mine], L["s2"][mine])
    sl = slice(rank * tl, (rank + 1) * tl)
    xs = L["x"][sl].contiguous()
    ok = True
    for _ in range(2):
        y, ids, w = grp.moe_prefill(xs, L["gate"], TOPK, True, L["logit_bias"], *lw, L["sh_w13"], L["sh_s13"],
                                    L["sh_w2"], L["sh_s2"], L["sh_gate"], None, owner=owner)
        torch.cuda.synchronize()
        ok = ok and torch.equal(y, ref[0][sl]) and torch.equal(ids, ref[1][sl]) and torch.equal(w, ref[2][sl])
    ok = ok and dm3.ops.moe_status(dm3.ep._ep_workspaces[dev.index]) == 0
    del L, lw
    ok = all_ranks_true(ok, world)
    return {"ok": ok, "against": "dm3::moe_prefill of all 512 tokens with all 256 experts on this rank's GPU "
                                 "(y, ids, weights bit-identical)"}


def run_decode_sharded(args, world, rank, local):
    """One 2-row frame of 40 layers sharded over `world` GPUs: every rank the same rows, router and
    routing, its 256 / world experts per layer (rank 0 the shared expert), and an NVLink all-reduce
    of the partial sums inside each layer's combine kernel."""
    import drama3_b200 as dm3
    import torch.distributed as dist

    dev = torch.device("cuda", local)
    n_layers = args.layers
    el = E // world
    layers = []
    for l in range(n_layers):
        seed = 1000 + l
        g = torch.Generator(device=dev).manual_seed(seed)  # replicated parts: same on every rank
        L = {"gate": (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)}
        L["sh_w13"], L["sh_s13"] = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
        L["sh_w2"], L["sh_s2"] = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
        L["sh_gate"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        L["x"] = rms(torch.randn(T, H, generator=g, device=dev)).to(torch.bfloat16)
        gl = torch.Generator(device=dev).manual_seed(seed * 100 + rank)  # this rank's experts
        L["w13"], L["s13"] = dm3.fp8_block(torch.randn(el, 2 * I, H, generator=gl, device=dev) * 0.02)
        L["w2"], L["s2"] = dm3.fp8_block(torch.randn(el, H, I, generator=gl, device=dev) * 0.02)
        layers.append(L)
    grp = dm3.ep.ExpertParallel(PF_T // world, H, TOPK)
    parity = check_decode_sharded(grp, world, rank, dev)

    def call(L, x):
        return grp.moe_layer(x, L["gate"], TOPK, True, None, L["w13"], L["s13"], L["w2"], L["s2"], L["sh_w13"],
                             L["sh_s13"], L["sh_w2"], L["sh_s2"], L["sh_gate"], None)

    outs = [call(L, L["x"]) for L in layers]
    torch.cuda.synchronize()
    barrier(world)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gouts = [call(L, L["x"]) for L in layers]
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    assert dm3.ops.moe_status(dm3.ops.moe_workspace(dev, H, I)) == 0, "device status word set during warm-up"
    for o, g2 in zip(outs, gouts):
        assert torch.equal(o[1], g2[1]), "graph replay routed differently from eager"
    # this rank's HBM bytes per frame: its selected experts, the router, the shared expert on rank 0
    bytes_rank = 0
    for L, o in zip(layers, outs):
        ids = o[1]
        mine = torch.unique(ids[(ids // el) == rank])
        bytes_rank += int(mine.numel()) * EXPERT_BYTES + E * H * 2 + 2 * T * H * 2
        if rank == 0:
            bytes_rank += EXPERT_BYTES + H * 2
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    launches = args.steps * n_layers * dm3._lib.load().dm3_last_launch_count()
    xs_host = torch.stack([L["x"].cpu() for L in layers]).pin_memory()
    y_host = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xs_dev = torch.stack([L["x"] for L in layers])
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        g2outs = [call(L, xs_dev[l])[0] for l, L in enumerate(layers)]

    def e2e_step():
        xs_dev.copy_(xs_host, non_blocking=True)
        g2.replay()
        y_host.copy_(g2outs[-1], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        e2e_step()
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / args.steps, world)
    bt = torch.tensor([float(bytes_rank)], device=dev)
    dist.all_reduce(bt, op=dist.ReduceOp.MAX)
    pk = peaks()
    achieved = float(bt.item()) / (ms * 1e-3) / 1e9
    clk_sum = clk.summary()
    del graph, g2
    grp.close()
    return {
        "parity": parity,
        "metric": METRIC, "value": round(n_layers * 1000.0 / ms, 1), "unit": "layer-frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "us_per_layer": round(ms * 1000.0 / n_layers, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "e4m3 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, RMS-normalised N(0,1) rows)",
        "config": {"workload": "decode_fp8_256x40", "layers": n_layers, "rows": T, "hidden": H, "intermediate": I,
                   "experts": E, "top_k": TOPK, "router": "bf16, logits rounded to bf16",
                   "shared_expert": "block-FP8 128x128 + bf16 sigmoid gate (rank 0)", "scales": "128x128 fp32",
                   "cuda_graph": True,
                   "parallelism": f"sharded x{world}: {el} experts per rank, NVLink all-reduce in the combine kernel"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": f"{pk['source']} HBM copy bandwidth",
                     "kernel": "one sharded decode frame per GPU (the busiest rank's HBM bytes / frame time)",
                     "bytes_per_launch": round(float(bt.item()) / n_layers), "traffic": None},
        "gpu_launches": launches,
        "e2e": {"value": round(n_layers * 1000.0 / ms_e2e, 1), "unit": "layer-frames/s",
                "h2d_bytes_per_step": int(xs_host.numel() * 2), "d2h_bytes_per_step": int(y_host.numel() * 2),
                "ms_per_step": round(ms_e2e, 4),
                "path": "pinned host rows -> H2D -> captured ExpertParallel.moe_layer x 40 -> D2H of the last layer"},
        "clocks": {k: clk_sum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
    }


def run_decode(args, world, rank, local, speaker=False):
    import drama3_b200 as dm3

    if world > 1 and args.decode_mode == "sharded" and not speaker:
        return run_decode_sharded(args, world, rank, local)

    dev = torch.device("cuda", local)
    n_layers = args.layers
    kw = dict(experts=32, router_dtype=torch.float32, shared=True, bias=True) if speaker else {}
    layers = [make_layer(1000 * (rank + 1) + l, dev, **kw) for l in range(n_layers)]
    # every layer's 2 rows of a frame live in xs_in [layers, T, H]; the speaker workload times
    # SPEAKER_FRAMES consecutive frames, each with its own seeded rows, copied into xs_in before
    # the frame's graph replay; the 256-expert decode replays one frame's rows
    if speaker:
        gx = torch.Generator(device=dev).manual_seed(4242 + rank)
        xs_frames = rms(torch.randn(SPEAKER_FRAMES, n_layers, T, H, generator=gx, device=dev)).to(torch.bfloat16)
        xs_in = xs_frames[0].clone()
    else:
        xs_frames = None
        xs_in = torch.stack([L["x"] for L in layers])
    torch.cuda.synchronize()
    logits_bf16 = not speaker
    outs = [layer_call(L, xs_in[l], logits_bf16) for l, L in enumerate(layers)]  # eager warm-up (workspace)
    torch.cuda.synchronize()
    bytes_step = sum(layer_bytes(L, o[1]) for L, o in zip(layers, outs))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gouts = [layer_call(L, xs_in[l], logits_bf16) for l, L in enumerate(layers)]
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    ws = dm3.ops.moe_workspace(dev, H, I)
    assert dm3.ops.moe_status(ws) == 0, "device status word set during warm-up"
    for o, g in zip(outs, gouts):
        assert torch.equal(o[1], g[1]), "graph replay routed differently from eager"

    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = SPEAKER_FRAMES if speaker else args.steps
    with ClockSampler(local) as clk:
        e0.record()
        for f in range(steps):
            if speaker:
                xs_in.copy_(xs_frames[f])  # the frame's rows (320 KB, device to device)
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    # kernels per layer as the library reports them (route, cluster, finish)
    launches = steps * n_layers * dm3._lib.load().dm3_last_launch_count()

    # end to end through the public op with host buffers: every layer's rows H2D from pinned memory
    # (one copy), the captured frame, and the frame's result (the last layer's rows) D2H
    xs_host_all = (xs_frames if speaker else xs_in.unsqueeze(0)).cpu().pin_memory()
    xs_host = xs_host_all[0]
    y_host = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xs_dev = xs_in.clone()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        g2outs = [layer_call(L, xs_dev[l], logits_bf16)[0] for l, L in enumerate(layers)]

    def e2e_step(f=0):
        xs_dev.copy_(xs_host_all[f % xs_host_all.shape[0]], non_blocking=True)
        g2.replay()
        y_host.copy_(g2outs[-1], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for f in range(steps):
        e2e_step(f)
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / steps, world)

    pk = peaks()
    achieved = bytes_step / (ms * 1e-3) / 1e9
    value = world * n_layers * 1000.0 / ms
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "layer-frames/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "us_per_layer": round(ms * 1000.0 / n_layers, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, RMS-normalised N(0,1) rows)",
        "config": {
            "workload": ("speaker_decode_fp8_32x40" if speaker else "decode_fp8_256x40"),
            "layers": n_layers, "rows": T, "hidden": H, "intermediate": I,
            "experts": 32 if speaker else E, "top_k": TOPK,
            "router": "fp32 (speaker)" if speaker else "bf16, logits rounded to bf16",
            "shared_expert": "block-FP8 128x128 + bf16 sigmoid gate",
            "scales": "128x128 fp32", "cuda_graph": True,
            "l2": "no flush: 40 layers stream > 2 GB of weights per step (L2 126 MB)",
            "frames": (f"{SPEAKER_FRAMES} consecutive frames, each with its own seeded rows per layer (one step = one "
                       "frame)" if speaker else "one frame's rows replayed (one step = one frame of 40 layers)"),
            "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4),
            "peak_source": f"{pk['source']} HBM copy bandwidth",
            "kernel": ("one decode layer: dm3::moe route_kernel + layer_kernel (2-CTA clusters) + finish_kernel"
                       if os.environ.get("DM3_CLUSTER", "1") != "0"
                       else "one decode layer: dm3::moe route + up + down + combine kernels"),
            "bytes_per_launch": round(bytes_step / n_layers),
            "traffic": recorded_traffic("moe_decode_layer"),
        },
        "gpu_launches": launches,
        "e2e": {
            "value": round(world * n_layers * 1000.0 / ms_e2e, 1),
            "unit": "layer-frames/s",
            "h2d_bytes_per_step": int(xs_host.numel() * 2),
            "d2h_bytes_per_step": int(y_host.numel() * 2),
            "ms_per_step": round(ms_e2e, 4),
            "path": "pinned host rows -> H2D -> captured drama3_b200.ops.moe_layer x 40 -> D2H of the last layer",
        },
    }
    clk_sum = clk.summary()
    line["clocks"] = {k: clk_sum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu_layers = [cpu_layer(L) for L in layers[:2]]
        v, reps, thr = time_cpu_port(cpu_layers, budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": "layer-frames/s", "cores": thr, "kind": "port",
                                "sample": f"{reps} layer evaluations of the same workload (2 layers cycled), torch fp32 "
                                          "on host cores (oracle/cpu_port.py)"}
    return line


def make_prefill_layer(seed: int, dev):
    """A prompt-reading layer: the decode layer's weights plus a seeded Zipf(s=1.1) logit bias
    b_e = -1.1 ln(rank_e) over a random permutation of ranks, and T=512 RMS-normalised rows."""
    L = make_layer(seed, dev)
    g = torch.Generator(device="cpu").manual_seed(seed + 7)
    rank_e = torch.randperm(E, generator=g).float() + 1.0
    L["logit_bias"] = (-1.1 * torch.log(rank_e)).to(dev)
    gx = torch.Generator(device=dev).manual_seed(seed + 11)
    L["x"] = rms(torch.randn(PF_T, H, generator=gx, device=dev)).to(torch.bfloat16)
    return L


def prefill_call(L, x):
    import drama3_b200 as dm3

    return dm3.ops.moe_prefill(x, L["gate"], TOPK, True, L["logit_bias"], L["w13"], L["s13"], L["w2"], L["s2"],
                               L["sh_w13"], L["sh_s13"], L["sh_w2"], L["sh_s2"], L["sh_gate"], None)


def prefill_bytes(L, ids: torch.Tensor) -> int:
    """Algorithmic HBM bytes of one prefill layer: every touched expert once, the router, the
    shared expert and its gate row, the logit bias, the rows in and the outputs."""
    u = int(torch.unique(ids).numel())
    return (u + 1) * EXPERT_BYTES + E * H * 2 + H * 2 + E * 4 + 2 * PF_T * H * 2


def run_prefill_ep(args, world, rank, local):
    """Expert parallel over `world` GPUs: T=512 tokens in total (512 / world per rank), 256 / world
    experts per rank placed by --ep-placement (default: balanced on observed loads); NVLink dispatch /
    return inside the kernels."""
    import drama3_b200 as dm3

    dev = torch.device("cuda", local)
    el, tl = E // world, PF_T // world
    n_layers = 4
    layers = []
    placement = args.ep_placement
    for l in range(n_layers):
        seed = 2000 + l
        g = torch.Generator(device=dev).manual_seed(seed)
        L = {"gate": (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)}
        L["sh_w13"], L["sh_s13"] = dm3.fp8_block(torch.randn(2 * I, H, generator=g, device=dev) * 0.02)
        L["sh_w2"], L["sh_s2"] = dm3.fp8_block(torch.randn(H, I, generator=g, device=dev) * 0.02)
        L["sh_gate"] = (torch.randn(H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        gl = torch.Generator(device=dev).manual_seed(seed * 100 + rank)  # this rank's experts
        L["w13"], L["s13"] = dm3.fp8_block(torch.randn(el, 2 * I, H, generator=gl, device=dev) * 0.02)
        L["w2"], L["s2"] = dm3.fp8_block(torch.randn(el, H, I, generator=gl, device=dev) * 0.02)
        gb = torch.Generator(device="cpu").manual_seed(seed + 7)
        bias_cpu = -1.1 * torch.log(torch.randperm(E, generator=gb).float() + 1.0)
        L["logit_bias"] = bias_cpu.to(dev)
        # observed: balance the pair counts of a calibration batch; balanced: the expected load
        # exp(bias) = rank^-1.1 (which ignores that a token's top-8 are distinct experts)
        if placement == "observed":
            L["owner"] = observed_placement(L["gate"], L["logit_bias"], world, dev, seed + 13).to(dev)
        elif placement == "balanced":
            L["owner"] = dm3.ep.balanced_placement(torch.exp(bias_cpu), world).to(dev)
        else:
            L["owner"] = None
        gx = torch.Generator(device=dev).manual_seed(seed + 11)
        x = rms(torch.randn(PF_T, H, generator=gx, device=dev)).to(torch.bfloat16)
        L["x"] = x[rank * tl:(rank + 1) * tl].contiguous()
        layers.append(L)
    grp = dm3.ep.ExpertParallel(tl, H, TOPK)
    parity = check_prefill_ep(grp, world, rank, dev, placement)

    def call(L, x):
        return grp.moe_prefill(x, L["gate"], TOPK, True, L["logit_bias"], L["w13"], L["s13"], L["w2"], L["s2"],
                               L["sh_w13"], L["sh_s13"], L["sh_w2"], L["sh_s2"], L["sh_gate"], None, owner=L["owner"])

    outs = [call(L, L["x"]) for L in layers]
    torch.cuda.synchronize()
    barrier(world)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gouts = [call(L, L["x"]) for L in layers]
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    ws = dm3.ep._ep_workspaces[local]
    assert dm3.ops.moe_status(ws) == 0, "device status word set during warm-up"
    for o, g2 in zip(outs, gouts):
        assert torch.equal(o[1], g2[1]), "graph replay routed differently from eager"
    # per-rank load: pairs each rank's experts receive and its touched local experts (from all ranks' routing)
    import torch.distributed as dist

    ids_all = [torch.empty_like(outs[0][1]) for _ in range(world)]
    dist.all_gather(ids_all, outs[0][1])
    ids_cat = torch.cat(ids_all)
    owners = (layers[0]["owner"].long()[ids_cat] >> 16) if layers[0]["owner"] is not None else ids_cat // el
    recv = [int((owners == r).sum()) for r in range(world)]
    touched = int(torch.unique(ids_cat[owners == rank]).numel())
    steps = max(args.steps // n_layers, 1) * n_layers
    reps = steps // n_layers
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    launches = steps * dm3._lib.load().dm3_last_launch_count()
    # end to end: this rank's rows H2D, the captured layers, the outputs D2H
    xs_host = torch.stack([L["x"].cpu() for L in layers]).pin_memory()
    ys_host = torch.empty(n_layers, tl, H, dtype=torch.bfloat16).pin_memory()
    xs_dev = torch.stack([L["x"] for L in layers])
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        g2outs = [call(L, xs_dev[l])[0] for l, L in enumerate(layers)]

    def e2e_pass():
        xs_dev.copy_(xs_host, non_blocking=True)
        g2.replay()
        for l in range(n_layers):
            ys_host[l].copy_(g2outs[l], non_blocking=True)

    for _ in range(2):
        e2e_pass()
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(reps):
        e2e_pass()
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / steps, world)
    # HBM bytes of this rank: its touched experts, the replicated router and shared expert, its rows
    bytes_rank = (touched + 1) * EXPERT_BYTES + E * H * 2 + H * 2 + E * 4 + 2 * tl * H * 2
    bt = torch.tensor([float(bytes_rank)], device=dev)
    dist.all_reduce(bt)
    pk = peaks()
    achieved = float(bt.item()) / world / (ms * 1e-3) / 1e9
    clk_sum = clk.summary()
    del graph, g2
    grp.close()
    return {
        "parity": parity,
        "metric": PF_METRIC,
        "value": round(PF_T * 1000.0 / ms, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "us_per_layer": round(ms * 1000.0, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, RMS-normalised N(0,1) rows, Zipf(1.1) logit bias)",
        "config": {
            "workload": "prefill_fp8_256_T512_zipf", "tokens": PF_T, "hidden": H, "intermediate": I,
            "experts": E, "top_k": TOPK, "router": "bf16, logits rounded to bf16, + Zipf bias",
            "shared_expert": "block-FP8 128x128 + bf16 sigmoid gate (on each token's home rank)",
            "parallelism": f"expert parallel x{world}: {el} experts and {tl} tokens per rank, NVLink peer stores",
            "placement": placement + {"observed": " (greedy LPT on the pair counts of a separate seeded calibration "
                                                  "batch routed once)",
                                      "balanced": " (greedy LPT on the expected load exp(bias))",
                                      "contiguous": " (blocks of 256 / n_gpus experts)"}[placement],
            "pairs_received_per_rank": recv, "cuda_graph": True,
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4), "peak_source": f"{pk['source']} HBM copy bandwidth",
            "kernel": "one expert-parallel prefill layer per GPU (mean HBM bytes over ranks / layer time)",
            "bytes_per_launch": round(float(bt.item()) / world), "traffic": None,
        },
        "gpu_launches": launches,
        "e2e": {"value": round(PF_T * 1000.0 / ms_e2e, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(xs_host[0].numel() * 2), "d2h_bytes_per_step": int(ys_host[0].numel() * 2),
                "ms_per_step": round(ms_e2e, 4),
                "path": "pinned host rows of this rank -> H2D -> captured ExpertParallel.moe_prefill -> D2H"},
        "clocks": {k: clk_sum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
    }


def run_prefill(args, world, rank, local):
    import drama3_b200 as dm3

    if world > 1:
        return run_prefill_ep(args, world, rank, local)

    dev = torch.device("cuda", local)
    n_layers = 4  # distinct layers cycled, 3.2 GB of expert weights: each step streams its experts from HBM
    layers = [make_prefill_layer(2000 * (rank + 1) + l, dev) for l in range(n_layers)]
    torch.cuda.synchronize()
    outs = [prefill_call(L, L["x"]) for L in layers]
    torch.cuda.synchronize()
    bytes_layer = [prefill_bytes(L, o[1]) for L, o in zip(layers, outs)]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gouts = [prefill_call(L, L["x"]) for L in layers]
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    ws = dm3.ops._pf_workspaces[local]
    assert dm3.ops.moe_status(ws) == 0, "device status word set during warm-up"
    for o, g in zip(outs, gouts):
        assert torch.equal(o[1], g[1]) and torch.equal(o[3], g[3]), "graph replay routed differently from eager"
    steps = max(args.steps // n_layers, 1) * n_layers  # whole passes over the 4 layers
    reps = steps // n_layers
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    launches = steps * dm3._lib.load().dm3_last_launch_count()

    # end to end through the public op: the step's 512 rows H2D from pinned memory, the captured
    # layer, its output rows D2H
    xs_host = torch.stack([L["x"].cpu() for L in layers]).pin_memory()
    ys_host = torch.empty(n_layers, PF_T, H, dtype=torch.bfloat16).pin_memory()
    xs_dev = torch.stack([L["x"] for L in layers])
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2):
        g2outs = [prefill_call(L, xs_dev[l])[0] for l, L in enumerate(layers)]

    def e2e_pass():
        xs_dev.copy_(xs_host, non_blocking=True)
        g2.replay()
        for l in range(n_layers):
            ys_host[l].copy_(g2outs[l], non_blocking=True)

    for _ in range(2):
        e2e_pass()
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(reps):
        e2e_pass()
    f1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = max_over_ranks(f0.elapsed_time(f1) / steps, world)

    pk = peaks()
    bytes_step = sum(bytes_layer) / n_layers
    achieved = bytes_step / (ms * 1e-3) / 1e9
    touched = [int(torch.unique(o[1]).numel()) for o in outs]
    line = {
        "metric": PF_METRIC,
        "value": round(world * PF_T * 1000.0 / ms, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "us_per_layer": round(ms * 1000.0, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e4m3 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, RMS-normalised N(0,1) rows, Zipf(1.1) logit bias)",
        "config": {
            "workload": "prefill_fp8_256_T512_zipf", "tokens": PF_T, "hidden": H, "intermediate": I,
            "experts": E, "top_k": TOPK, "router": "bf16, logits rounded to bf16, + Zipf bias",
            "shared_expert": "block-FP8 128x128 + bf16 sigmoid gate", "scales": "128x128 fp32",
            "touched_experts": touched, "cuda_graph": True,
            "l2": "no flush: 4 distinct layers cycled, each step streams ~270 MB of touched experts (L2 126 MB)",
            "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(achieved / pk["hbm_gbs"], 4),
            "peak_source": f"{pk['source']} HBM copy bandwidth",
            "kernel": "one prefill layer: dm3::moe_prefill logits + select + dispatch + up + down + combine kernels",
            "bytes_per_launch": round(bytes_step),
            "traffic": recorded_traffic("moe_prefill_layer"),
        },
        "gpu_launches": launches,
        "e2e": {
            "value": round(world * PF_T * 1000.0 / ms_e2e, 1),
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(xs_host[0].numel() * 2),
            "d2h_bytes_per_step": int(ys_host[0].numel() * 2),
            "ms_per_step": round(ms_e2e, 4),
            "path": "pinned host rows -> H2D -> captured drama3_b200.ops.moe_prefill -> D2H of the layer output",
        },
    }
    clk_sum = clk.summary()
    line["clocks"] = {k: clk_sum[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        v, reps_cpu, thr = time_cpu_port([cpu_layer(layers[0])], budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": round(v * PF_T, 1), "unit": "tokens/s", "cores": thr, "kind": "port",
                                "sample": f"{reps_cpu} evaluations of one T=512 prefill layer, torch fp32 on host "
                                          "cores (oracle/cpu_port.py)"}
    return line


def run_gemv(args, world, rank, local):
    """Block-FP8 GEMV sweep: per shape and scale layout, 40 distinct weight copies in one graph (each
    launch reads cold weights, as the reference's own timing rotates 40 layers, fp8_linear.py:82-103).
    Layouts: 128x128 block scales (fp8_block, the layout the sweep is specified in) and 1x128 row
    scales (fp8_linear.quantize). The audio head also runs as the gather kernel: 4,097 rows (eos + a
    4,096-row band) taken from a seeded 252,000 x 2,048 block-FP8 matrix by an index list; the 40
    copies use 40 band starts so that every launch reads rows L2 does not hold."""
    import ctypes
    import drama3_b200 as dm3

    dev = torch.device("cuda", local)
    res = {}
    copies = 40
    hbm = peaks()["hbm_gbs"]

    def timed(graph, n_calls):
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1000.0 / (args.steps * n_calls)

    def block_quant(w):
        n = w.shape[0]
        pad = (-n) % 128
        q, sc = dm3.fp8_block(torch.nn.functional.pad(w, (0, 0, 0, pad)) if pad else w)
        return q[:n].contiguous(), sc.contiguous()

    for layout in ("128x128", "1x128"):
        for (k, n) in [(2048, 4096), (4096, 2048), (2048, 8192), (2048, 512), (2048, 4097)]:
            g = torch.Generator(device=dev).manual_seed(k + n)
            quant = block_quant if layout == "128x128" else dm3.quantize
            ws = [quant(torch.randn(n, k, generator=g, device=dev) * 0.02) for _ in range(copies)]
            x = rms(torch.randn(2, k, generator=g, device=dev)).to(torch.bfloat16)
            [dm3.ops.fp8_gemv(x, q, sc) for q, sc in ws]
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ys = [dm3.ops.fp8_gemv(x, q, sc) for q, sc in ws]
            us = timed(graph, copies)
            sbytes = ws[0][1].numel() * 4
            nbytes = n * k + sbytes + 2 * k * 2 + 2 * n * 2
            res[f"{k}x{n}/{layout}"] = {"us": round(us, 3), "GBps": round(nbytes / (us * 1e-6) / 1e9, 1),
                                        "frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4)}
            del ws, ys, graph
            torch.cuda.empty_cache()

    # audio head gathered in the kernel from the full-vocabulary matrix (128x128 scales)
    V, K, NH = 252000, 2048, 4097
    g = torch.Generator(device=dev).manual_seed(252000)
    qf = torch.empty(V, K, dtype=torch.float8_e4m3fn, device=dev)
    sf = torch.empty((V + 127) // 128, K // 128, dtype=torch.float32, device=dev)
    for r0 in range(0, V, 16384):
        r1 = min(V, r0 + 16384)
        qb, sb = block_quant(torch.randn(r1 - r0, K, generator=g, device=dev) * 0.02)
        qf[r0:r1] = qb
        sf[r0 // 128:r0 // 128 + sb.shape[0]] = sb
    x = rms(torch.randn(2, K, generator=g, device=dev)).to(torch.bfloat16)
    starts = torch.randperm((V - 1 - NH) // 128, generator=g, device=dev)[:copies] * 128 + 1
    idx = [torch.cat([torch.tensor([V - 1], device=dev), torch.arange(int(s0), int(s0) + NH - 1, device=dev)])
           for s0 in starts.tolist()]
    ys = [torch.empty(2, NH, dtype=torch.float32, device=dev) for _ in range(copies)]
    lib = dm3._lib.load()

    def head_calls():
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for rows, y in zip(idx, ys):
            rc = lib.dm3_fp8_gemv_gather(ctypes.c_void_p(x.data_ptr()), 2, K, NH, ctypes.c_void_p(qf.data_ptr()), K, V,
                                         ctypes.c_void_p(rows.data_ptr()), ctypes.c_void_p(sf.data_ptr()), K // 128,
                                         128, ctypes.c_void_p(y.data_ptr()), NH, 1, st)
            assert rc == 0, lib.dm3_last_error()

    head_calls()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        head_calls()
    us = timed(graph, copies)
    nbytes = NH * K + NH * (K // 128) * 4 + NH * 8 + 2 * K * 2 + 2 * NH * 4
    res["2048x4097/128x128/gathered"] = {"us": round(us, 3), "GBps": round(nbytes / (us * 1e-6) / 1e9, 1),
                                         "frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4)}
    del qf, sf, graph
    main_key = "2048x4096/128x128"
    return {"metric": "block-FP8 GEMV (M=2) per call", "value": res[main_key]["us"], "unit": "us/call",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 x bf16", "data": "synthetic",
            "config": {"workload": "gemv_sweep_m2", "copies": copies, "value_shape": main_key,
                       "l2": "no flush: 40 distinct weight copies per graph, each launch reads cold rows"},
            "roofline": {"bound": "hbm", "achieved": res[main_key]["GBps"], "peak": hbm, "unit": "GB/s",
                         "frac": res[main_key]["frac"], "kernel": "dm3::gemv::gemv_kernel<1> (FP8 mma.sync on raw e4m3 rows), 2048x4096",
                         "traffic": recorded_traffic("gemv_2048x4096")},
            "shapes": res, "gpu_launches": args.steps * copies * 11}


def run_gemm(args, world, rank, local):
    """Block-FP8 GEMM (dm3::fp8_gemm) for a prompt chunk: M = 256 rows against the 9216 x 2048
    projection (1x128 scales, the FP8Linear layout), 40 distinct weight copies per graph, next to the
    reference's own path for more than 2 rows, dequantise + bf16 cast + F.linear (fp8_linear.py:60-61),
    run with torch on the same GPU and inputs."""
    import drama3_b200 as dm3

    dev = torch.device("cuda", local)
    hbm = peaks()["hbm_gbs"]
    M, N, K, copies = 256, 9216, 2048, 40
    g = torch.Generator(device=dev).manual_seed(9216)
    ws = [dm3.quantize(torch.randn(N, K, generator=g, device=dev) * 0.02) for _ in range(copies)]
    x = rms(torch.randn(M, K, generator=g, device=dev)).to(torch.bfloat16)

    def ours():
        return [dm3.ops.fp8_gemm(x, q, sc) for q, sc in ws]

    def reference_path():
        return [torch.nn.functional.linear(x, dm3.dequantize(q, sc).to(x.dtype)) for q, sc in ws]

    res = {}
    for name, fn in (("ours", ours), ("reference_torch_path", reference_path)):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = fn()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(args.steps // 5, 4)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (steps * copies)
        res[name] = {"us": round(us, 2), "outs": outs}
        del graph
    err = float((res["ours"]["outs"][0].float() - res["reference_torch_path"]["outs"][0].float()).norm()
                / res["reference_torch_path"]["outs"][0].float().norm())
    nbytes = N * K + N * (K // 128) * 4 + M * K * 2 + M * N * 2
    flops = 2.0 * M * N * K
    us = res["ours"]["us"]
    return {"workload": "gemm_fp8_m256_9216x2048_1x128", "rows": M, "K": K, "N": N, "copies": copies,
            "us": us, "reference_torch_path_us": res["reference_torch_path"]["us"],
            "speedup_vs_reference_torch_path": round(res["reference_torch_path"]["us"] / us, 2),
            "rel_l2_vs_reference_torch_path": round(err, 6),
            "TFLOPs": round(flops / (us * 1e-6) / 1e12, 1),
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (us * 1e-6) / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4),
                         "bytes_per_launch": nbytes,
                         "note": "weights + scales + x + y once; the hi/lo activation split doubles the MMA work"}}


def run_audio_head(args, world, rank, local):
    """The audio head of one CFG frame: the fused block-FP8 head (GEMV, guidance, index_copy into the
    -inf vocabulary buffer, log-sum-exp) plus direction_score, over 40 distinct head copies per graph,
    next to the reference's own lines run with torch on the same GPU: the bf16 head matmul, .float(),
    index_copy into a new -inf buffer and direction_score's log_softmax (engine.py:423-424, :476-479)."""
    import drama3_b200 as dm3

    dev = torch.device("cuda", local)
    hbm = peaks()["hbm_gbs"]
    V, K, NH, copies = 252000, 2048, 4097, 40
    g = torch.Generator(device=dev).manual_seed(4097)
    cand = torch.cat([torch.tensor([V - 1], device=dev), torch.arange(151000, 151000 + NH - 1, device=dev)])
    heads_bf16 = [(torch.randn(NH, K, generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    ours = [dm3.AudioHead(None, cand, V, *dm3.quantize(w)) for w in heads_bf16]
    hidden = rms(torch.randn(2, K, generator=g, device=dev)).to(torch.bfloat16)
    strength = torch.tensor([1.5], dtype=torch.float32, device=dev)
    token = torch.tensor([151000 + 7], dtype=torch.int64, device=dev)
    score = torch.zeros((), dtype=torch.float32, device=dev)
    ref_buf = torch.full((1, V), -torch.inf, device=dev)

    def fused():
        for h in ours:
            h(hidden, strength)
            h.score_into(score, token, V - 1, 151000)

    def reference_path():
        for w in heads_bf16:
            logits = (hidden @ w.T).float()
            ref_buf.index_copy(1, cand, logits[1:] + strength * (logits[:1] - logits[1:]))
            index = torch.where(token == V - 1, 0, token - 151000 + 1)
            picked = torch.log_softmax(logits.float(), dim=-1).index_select(1, index.view(1))
            score.add_((picked[0] - picked[1]).squeeze())

    res = {}
    for name, fn in (("fused", fused), ("reference_torch_path", reference_path)):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(args.steps // 5, 4)
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) * 1000.0 / (steps * copies)
        del graph
    nbytes = NH * K + NH * (K // 128) * 4 + 2 * K * 2 + 2 * NH * 4 * 2 + NH * 8 + NH * 4
    us = res["fused"]
    return {"workload": "audio_head_cfg_4097x2048_fp8_1x128", "candidates": NH, "vocab": V, "copies": copies,
            "us_per_frame": round(us, 3), "launches_per_frame": 3,
            "reference_torch_path_us": round(res["reference_torch_path"], 3),
            "reference_torch_path": "bf16 head matmul + guidance + index_copy into a new -inf buffer + "
                                    "log_softmax direction_score (torch on the same GPU)",
            "speedup_vs_reference_torch_path": round(res["reference_torch_path"] / us, 2),
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (us * 1e-6) / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4), "bytes_per_launch": nbytes}}


def run_reference_prefill(args, world):
    """The reference's CPU path for the T=512 prefill layer (torch fp32 on host cores), same metric:
    each step evaluates the whole layer once."""
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    L = cpu_layer(make_prefill_layer(2000, dev))
    from oracle import cpu_port

    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(max(min(args.warmup, 1), 1)):
        cpu_port.decode_layer(L["x"], L)
    steps = max(min(args.steps, 20), 1)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_port.decode_layer(L["x"], L)
    el = time.perf_counter() - t0
    v = steps * PF_T / el
    thr = torch.get_num_threads()
    return {"impl": "reference", "metric": PF_METRIC, "value": round(v, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(el * 1000 / steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (CPU)",
            "data": "synthetic", "config": {"workload": "prefill_fp8_256_T512_zipf", "tokens": PF_T, "hidden": H,
                                            "intermediate": I, "experts": E, "top_k": TOPK,
                                            "sample": "one full T=512 layer per step (at most 20 steps)"},
            "cpu_baseline": {"value": round(v, 1), "unit": "tokens/s", "cores": thr, "kind": "port",
                             "sample": f"{steps} evaluations of one T=512 prefill layer, torch fp32 on {thr} host threads"},
            "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}


def run_reference(args, world, rank):
    """The reference's CPU path for the decode layer (torch fp32 on host cores), same metric."""
    if rank != 0:
        return None
    if args.workload == "prefill":
        return run_reference_prefill(args, world)
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    layers = [cpu_layer(make_layer(1000 + l, dev)) for l in range(2)]
    from oracle import cpu_port

    torch.set_num_threads(os.cpu_count() or 1)
    for i in range(max(args.warmup, 1)):
        L = layers[i % 2]
        cpu_port.decode_layer(L["x"], L)
    t0 = time.perf_counter()
    for i in range(args.steps):
        L = layers[i % 2]
        cpu_port.decode_layer(L["x"], L)
    el = time.perf_counter() - t0
    v = args.steps / el
    thr = torch.get_num_threads()
    return {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "layer-frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el * 1000 / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (CPU)",
            "data": "synthetic", "config": {"workload": "decode_fp8_256x40", "rows": T, "hidden": H,
                                            "intermediate": I, "experts": E, "top_k": TOPK,
                                            "sample": "one layer per step, 2 layers cycled"},
            "cpu_baseline": {"value": round(v, 3), "unit": "layer-frames/s", "cores": thr, "kind": "port",
                             "sample": f"{args.steps} layer evaluations, torch fp32 on {thr} host threads"},
            "e2e": {"value": round(v, 3), "unit": "layer-frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "speaker", "gemv", "prefill"])
    ap.add_argument("--layers", type=int, default=40)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-only", action="store_true",
                    help="default workload: skip the prefill / GEMV objects (N=1) or the NVLink objects (N>1)")
    ap.add_argument("--decode-mode", default="replicas", choices=["replicas", "sharded"],
                    help="n_gpus > 1 decode: independent replicas (weak scaling) or one frame sharded (strong)")
    ap.add_argument("--ep-placement", default="observed", choices=["observed", "balanced", "contiguous"],
                    help="expert placement of the expert-parallel prefill (n_gpus > 1)")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    parity_ok = True
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "gemv":
            line = run_gemv(args, world, rank, local)
        elif args.workload == "prefill":
            line = run_prefill(args, world, rank, local)
        else:
            line = run_decode(args, world, rank, local, speaker=args.workload == "speaker")
            if args.workload == "decode" and not args.decode_only:
                torch.cuda.empty_cache()
                if world == 1:
                    # the prompt-reading layer and the GEMV / GEMM sweep on the same GPU
                    line["prefill"] = run_prefill(args, world, rank, local)
                    torch.cuda.empty_cache()
                    line["gemv"] = run_gemv(args, world, rank, local)
                    torch.cuda.empty_cache()
                    line["gemv"]["gemm"] = run_gemm(args, world, rank, local)
                    torch.cuda.empty_cache()
                    line["gemv"]["audio_head"] = run_audio_head(args, world, rank, local)
                else:
                    # the NVLink paths, each checked against the one-GPU op first
                    line["prefill_ep"] = run_prefill_ep(args, world, rank, local)
                    torch.cuda.empty_cache()
                    line["decode_sharded"] = run_decode_sharded(args, world, rank, local)
                    parity_ok = line["prefill_ep"]["parity"]["ok"] and line["decode_sharded"]["parity"]["ok"]
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if not parity_ok:
        sys.exit("parity check of a multi-GPU path failed")


if __name__ == "__main__":
    main()
