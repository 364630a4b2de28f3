"""Generates the golden fixtures in this directory by running the reference's own code on CPU.

Run from the repository root in a checkout that has the reference tree available:

    python tests/golden/make_golden.py --reference <path to drama-3-tr>

What runs here (none of it is copied into this repository):
  * engine.fp8_block, engine.Speaker, engine.speaker_forward (engine.py:153-158, 214-237),
    imported with `soundfile` and the absent third-party `fish_speech` package stubbed. The
    stubbed `fp8_moe_forward` records the routing the reference computes and returns the
    oracle's restatement, so Speaker's own routing, bias add and rounding run unmodified.
  * fp8_linear.quantize / dequantize / FP8Linear (fp8_linear.py:30-64), including the Triton
    `_gemv` kernel executed by the Triton interpreter on CPU. Two interpreter emulation gaps are
    closed so the kernel computes what it computes on a GPU: bf16 is stored as raw uint16 bits and
    tl.dot multiplied those bits as integers (`create_dot` now widens bf16 operands to fp32), and
    fp32 -> bf16 casts truncated (they now round to nearest even, as the hardware conversion does).
    The autotuner needs a GPU benchmarker, so launches are pinned to one of the kernel's own
    configs (BN=64). The kernel source itself is unchanged.
  * fp8_linear.convert on a shared-expert MLP (the TTS_FP8 path, engine.py:201-206).

Inputs are regenerated from the seeds in tests/golden/inputs.py (torch.Generator on CPU), and each
fixture stores a float64 checksum of its generated inputs so a test notices if generation drifts.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))


def _patch_triton_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as ti

    orig = ti.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16:
            a = ti.TensorHandle(ti._convert_float(a.data, tl.bfloat16, tl.float32, None).view(np.float32), tl.float32)
        if b.dtype.scalar == tl.bfloat16:
            b = ti.TensorHandle(ti._convert_float(b.data, tl.bfloat16, tl.float32, None).view(np.float32), tl.float32)
        return orig(self, a, b, d, input_precision, max_num_imprecise_acc)

    ti.InterpreterBuilder.create_dot = create_dot

    orig_cast = ti.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            u = np.ascontiguousarray(src.data, dtype=np.float32).view(np.uint32).astype(np.uint64)
            r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            return ti.TensorHandle(r.reshape(src.data.shape), tl.bfloat16)
        return orig_cast(self, src, dst_type)

    ti.InterpreterBuilder.cast_impl = cast_impl
    ti.InterpreterBuilder.create_fp_trunc = lambda self, src, dst_type: self.cast_impl(src, dst_type)


class _OneConfig:
    """Stands in for a triton Autotuner: launches the wrapped kernel with fixed meta-parameters."""

    def __init__(self, fn, **meta):
        self.fn, self.meta = fn, meta

    def __getitem__(self, grid):
        g = grid(self.meta) if callable(grid) else grid
        return lambda *a, **k: self.fn[g](*a, **k, **self.meta)


def _stub_reference_imports(moe_impl):
    import torch

    def stub(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m
        return m

    stub("soundfile")
    for n in ["fish_speech", "fish_speech.models", "fish_speech.models.text2semantic",
              "fish_speech.models.text2semantic.fish_omni"]:
        stub(n)
    p = "fish_speech.models.text2semantic.fish_omni."

    class Any_:
        def __init__(self, *a, **k):
            pass

    stub(p + "backbone", FishOmniBackbone=Any_, backbone_name=lambda k: k, DecoderLayer=Any_)
    stub(p + "config", FishOmniConfig=Any_)
    stub(p + "layers", LayerContext=Any_)
    stub(p + "fp8_moe", fp8_moe_forward=moe_impl)
    stub(p + "generate", RAS_WINDOW_FRAMES=16, Drama3DecodeGraphs=Any_, build_drama3_prompt=None,
         ensure_drama3_caches=None)
    stub(p + "model", AUDIO_DECODER_PREFIXES=("audio_decoder.",), FishOmniModel=Any_)

    class SparseMoeBlock(torch.nn.Module):
        def forward(self, x):  # the routed path is not exercised by these fixtures
            raise NotImplementedError

    stub(p + "moe", SparseMoeBlock=SparseMoeBlock)
    stub(p + "tower", FishOmniAudioDecoder=Any_, load_audio_decoder_weights=None)


def checksum(t) -> float:
    import torch

    if t.dtype == torch.float8_e4m3fn:
        return float(t.view(torch.uint8).to(torch.float64).sum())
    return float(t.detach().to(torch.float64).sum())


def bits(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def cdiv(a, b):
    return (a + b - 1) // b


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DM3_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, args.reference)

    import torch

    import oracle
    from tests.golden import inputs

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    _patch_triton_interpreter()
    calls = []

    def fp8_moe_forward(x, ids, w, w13, s13, w2, s2):
        calls.append((ids.clone(), w.clone()))
        return oracle.moe_forward(x, ids, w, w13, s13, w2, s2, srows=128)

    _stub_reference_imports(fp8_moe_forward)
    import engine as ref_engine  # noqa: E402  (reference)
    import fp8_linear as ref_fp8  # noqa: E402  (reference)

    torch.Tensor.cuda = lambda self, *a, **k: self  # Speaker moves its tensors with .cuda()
    ref_fp8._gemv = _OneConfig(ref_fp8._gemv.fn, BN=64)

    # ------------------------------------------------------------------ fp8_block KAT
    w = inputs.block_quant_input()
    q, s = ref_engine.fp8_block(w)
    np.savez_compressed(HERE / "fp8_block.npz", q=bits(q), s=s.numpy(), in_checksum=checksum(w))

    # ------------------------------------------------------------------ fp8_linear quantize KAT
    wl = inputs.row_quant_input()
    ql, sl = ref_fp8.quantize(wl)
    deq = ref_fp8.dequantize(ql, sl)
    np.savez_compressed(HERE / "fp8_rows.npz", q=bits(ql), s=sl.numpy(), deq_checksum=checksum(deq),
                        deq_row0=deq[0].numpy(), in_checksum=checksum(wl))

    # ------------------------------------------------------------------ Triton _gemv (interpreter) + FP8Linear
    gx, gw = inputs.gemv_case()
    lin = torch.nn.Linear(gw.shape[1], gw.shape[0], bias=False, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(gw)
    f = ref_fp8.FP8Linear(lin)
    out = {}
    for m in (1, 2):
        y = torch.empty((m, f.out_features), dtype=torch.bfloat16)
        ref_fp8._gemv[(cdiv(f.out_features, 64),)](gx[:m].contiguous(), f.q, f.s, y, f.out_features,
                                                   f.in_features, M=m, MP=2)
        out[f"y_m{m}"] = bits(y)
    out["y_m3"] = bits(f(gx[:3]))  # FP8Linear rows > 2: dequantise + F.linear (fp8_linear.py:61)
    out["ref_bf16_m2"] = bits(lin(gx[:2]))
    np.savez_compressed(HERE / "gemv_ref.npz", x_checksum=checksum(gx), w_checksum=checksum(gw), **out)

    # ------------------------------------------------------------------ Speaker (engine.py:222-237)
    p = inputs.speaker_params()
    sp = ref_engine.Speaker(p)
    res = {"p_checksums": np.array([checksum(p[k]) for k in ("gate", "bias", "w13", "w2")])}
    for t in (1, 2):
        x = inputs.decode_rows(t, seed=100 + t)
        calls.clear()
        y = sp(x)
        ids, wts = calls[0]
        res[f"x{t}_checksum"] = checksum(x)
        res[f"ids_t{t}"] = ids.numpy()
        res[f"w_t{t}"] = bits(wts)
        res[f"y_t{t}"] = bits(y)
    res["s13"] = sp.s13.numpy()
    res["s2_sum"] = float(sp.s2.double().sum())
    res["w13_checksum"] = checksum(sp.w13)
    np.savez_compressed(HERE / "speaker_ref.npz", **res)

    # ------------------------------------------------------------------ speaker_forward (engine.py:153-158)
    ref_engine.OnDemandExperts.batch = 2
    shared = inputs.shared_mlp()
    sgate = inputs.shared_gate_linear()
    block = types.SimpleNamespace(experts=types.SimpleNamespace(speaker=sp), shared_expert=shared,
                                  shared_expert_gate=sgate)
    res = {}
    x = inputs.decode_rows(2, seed=202)
    res["x_checksum"] = checksum(x)
    y = ref_engine.speaker_forward(block, x[None])
    res["y_bf16_shared"] = bits(y[0])
    # the TTS_FP8 variant: fp8_linear.convert swaps the shared expert's linears (engine.py:201-206)
    shared8 = inputs.shared_mlp()
    n = ref_fp8.convert(shared8)
    block8 = types.SimpleNamespace(experts=types.SimpleNamespace(speaker=sp), shared_expert=shared8,
                                   shared_expert_gate=sgate)
    y8 = ref_engine.speaker_forward(block8, x[None])
    res["converted"] = n
    res["y_fp8_shared"] = bits(y8[0])
    np.savez_compressed(HERE / "speaker_forward_ref.npz", **res)

    # ------------------------------------------------------------------ 256-expert router (exp1_routing.py:59-60, engine.py:235)
    x = inputs.decode_rows(4, seed=303)
    gate = inputs.router256()
    lin = torch.nn.Linear(gate.shape[1], gate.shape[0], bias=False, dtype=torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(gate)
    logits = lin(x)
    probs = torch.softmax(logits.float(), dim=-1)
    wv, ids = probs.topk(8, dim=-1)
    wv = (wv / wv.sum(-1, keepdim=True)).to(torch.bfloat16)
    np.savez_compressed(HERE / "route256_ref.npz", ids=ids.numpy(), w=bits(wv), logits=bits(logits),
                        x_checksum=checksum(x), gate_checksum=checksum(gate))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
