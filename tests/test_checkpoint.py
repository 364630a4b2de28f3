"""Checkpoint readers: the speaker release file (release/convert_weights.py:14-18 layout) and the
HBM-resident expert table filled from the model checkpoint's expert keys (checkpoint.py:21-23,
:89-96) in the ExpertStore slot layout (engine.py:26-36). CPU tests check the bytes; the GPU test
runs the loaded tables through the kernels against the oracle."""

import json

import pytest
import torch
from safetensors.torch import save_file

import oracle
from tests.golden import inputs
from tests.helpers import REL_L2_TOL, rel_l2

H, I, E, L = 256, 128, 4, 2
PREFIX = "model.language_model."


def _speaker_layers(n=3, e=8, h=H, i=I):
    g = torch.Generator().manual_seed(31)
    out = []
    for _ in range(n):
        w13, s13 = oracle.fp8_block(torch.randn(e, 2 * i, h, generator=g) * 0.02)
        w2, s2 = oracle.fp8_block(torch.randn(e, h, i, generator=g) * 0.02)
        out.append({"selected": torch.randperm(64, generator=g)[:e], "gate": torch.randn(e, h, generator=g) * 0.02,
                    "bias": torch.randn(h, generator=g) * 0.02, "w13": w13, "s13": s13, "w2": w2, "s2": s2})
    return out


def _write_speaker(path, layers):
    flat = {f"layers.{i}.{k}": v.contiguous() for i, p in enumerate(layers) for k, v in p.items()}
    save_file(flat, str(path), metadata={"format": "pt", "quant": "fp8_e4m3 block 128x128"})


def test_speaker_file_round_trip(dm3, tmp_path):
    layers = _speaker_layers()
    path = tmp_path / "speaker.safetensors"
    _write_speaker(path, layers)
    back = dm3.read_speaker_file(path)
    assert len(back) == len(layers)
    for a, b in zip(back, layers):
        assert set(a) == set(b)
        for k in b:
            assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
            assert torch.equal(a[k].view(torch.uint8) if a[k].dtype == torch.float8_e4m3fn else a[k],
                               b[k].view(torch.uint8) if b[k].dtype == torch.float8_e4m3fn else b[k]), k
    torch.save(layers, tmp_path / "speaker.pt")
    assert torch.equal(dm3.read_speaker_file(tmp_path / "speaker.pt")[1]["gate"], layers[1]["gate"])


def test_speaker_file_rejects_foreign_keys_and_gaps(dm3, tmp_path):
    layers = _speaker_layers(2)
    bad = {f"layers.{i}.{k}": v.contiguous() for i, p in enumerate(layers) for k, v in p.items()}
    bad["layers.0.unknown"] = torch.zeros(2)
    save_file(bad, str(tmp_path / "a.safetensors"))
    with pytest.raises(ValueError, match="unexpected tensor"):
        dm3.read_speaker_file(tmp_path / "a.safetensors")
    gap = {f"layers.{2 * i}.{k}": v.contiguous() for i, p in enumerate(layers) for k, v in p.items()}
    save_file(gap, str(tmp_path / "b.safetensors"))
    with pytest.raises(ValueError, match="numbered"):
        dm3.read_speaker_file(tmp_path / "b.safetensors")


def _checkpoint(tmp_path, layers=L, experts=E, drop=None):
    """A two-shard synthetic checkpoint with the model's expert keys plus unrelated tensors."""
    g = torch.Generator().manual_seed(41)
    src, shards = {}, [{}, {}]
    for l in range(layers):
        for e in range(experts):
            for proj, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
                q, s = oracle.fp8_block(torch.randn(*shape, generator=g) * 0.02)
                base = f"{PREFIX}layers.{l}.mlp.experts.{e}.{proj}"
                src[(l, e, proj)] = (q, s)
                for kind, t in (("weight", q), ("weight_scale_inv", s)):
                    key = f"{base}.{kind}"
                    if key != drop:
                        shards[(l + e) % 2][key] = t.contiguous()
        shards[l % 2][f"{PREFIX}layers.{l}.self_attn.q_proj.weight"] = torch.zeros(8, 8, dtype=torch.bfloat16)
    shards[0]["lm_head.weight"] = torch.zeros(4, 8, dtype=torch.bfloat16)
    names = ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]
    wmap = {}
    for name, sh in zip(names, shards):
        save_file(sh, str(tmp_path / name))
        wmap.update({k: name for k in sh})
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wmap}))
    return src


def test_expert_table_packs_checkpoint_into_slots(dm3, tmp_path):
    src = _checkpoint(tmp_path)
    table = dm3.ExpertTable.from_checkpoint(tmp_path, L, E, H, I, device="cpu")
    assert table.missing() == []
    u8 = lambda t: t.view(torch.uint8)  # noqa: E731
    for l in range(L):
        w13, s13, w2, s2 = table.layer(l)
        assert w13.stride(0) == 3 * I * H and w2.stride(0) == 3 * I * H  # the ExpertStore slot stride
        for e in range(E):
            gq, gs = src[(l, e, "gate_proj")]
            uq, us = src[(l, e, "up_proj")]
            dq, ds = src[(l, e, "down_proj")]
            assert torch.equal(u8(w13[e, :I]), u8(gq)) and torch.equal(u8(w13[e, I:]), u8(uq))
            assert torch.equal(u8(w2[e]), u8(dq))
            assert torch.equal(s13[e], torch.cat([gs, us])) and torch.equal(s2[e], ds)
            # the slot row is [gate; up; down] bytes back to back
            row = table.buf[l, e]
            assert torch.equal(row, torch.cat([u8(gq).flatten(), u8(uq).flatten(), u8(dq).flatten()]))


def test_expert_table_reports_missing_and_misshapen_tensors(dm3, tmp_path):
    drop = f"{PREFIX}layers.1.mlp.experts.2.up_proj.weight_scale_inv"
    _checkpoint(tmp_path, drop=drop)
    with pytest.raises(ValueError, match="missing"):
        dm3.ExpertTable.from_checkpoint(tmp_path, L, E, H, I, device="cpu")
    table = dm3.ExpertTable(L, E, H, I, device="cpu")
    with pytest.raises(ValueError, match="shape"):
        table.put(0, 0, "gate_proj", "weight", torch.zeros(I, H + 128, dtype=torch.float8_e4m3fn))
    with pytest.raises(ValueError, match="outside"):
        table.put(0, E, "gate_proj", "weight", torch.zeros(I, H, dtype=torch.float8_e4m3fn))


@pytest.mark.gpu
def test_resident_experts_and_speaker_file_on_gpu(dm3, tmp_path):
    src = _checkpoint(tmp_path)
    table = dm3.ExpertTable.from_checkpoint(tmp_path, L, E, H, I, device="cuda")
    x = inputs.decode_rows(6, seed=43, h=H)
    g = torch.Generator().manual_seed(44)
    ids = torch.stack([torch.randperm(E, generator=g)[:2] for _ in range(6)])
    w = torch.softmax(torch.randn(6, 2, generator=g), -1).to(torch.bfloat16)
    for l in range(L):
        mod = dm3.ResidentExperts(l, table)
        y = mod(x.cuda(), ids.cuda(), w.cuda())
        q13 = torch.stack([torch.cat([src[(l, e, "gate_proj")][0].view(torch.uint8),
                                      src[(l, e, "up_proj")][0].view(torch.uint8)]) for e in range(E)])
        s13 = torch.stack([torch.cat([src[(l, e, "gate_proj")][1], src[(l, e, "up_proj")][1]]) for e in range(E)])
        q2 = torch.stack([src[(l, e, "down_proj")][0].view(torch.uint8) for e in range(E)])
        s2 = torch.stack([src[(l, e, "down_proj")][1] for e in range(E)])
        ref = oracle.moe_forward(x, ids, w, q13.view(torch.float8_e4m3fn), s13, q2.view(torch.float8_e4m3fn), s2)
        assert rel_l2(y, ref) < REL_L2_TOL
    # the speaker release file straight into fused Speaker objects
    layers = _speaker_layers(2, e=8, h=512, i=128)
    path = tmp_path / "speaker.safetensors"
    _write_speaker(path, layers)
    sps = dm3.speakers_from_file(path)
    xs = inputs.decode_rows(2, seed=45, h=512)
    for sp, p in zip(sps, layers):
        y, ids2, _ = sp.route_and_combine(xs.cuda())
        ry, rids, _ = oracle.speaker(xs, p)
        assert torch.equal(ids2.cpu(), rids)
        assert rel_l2(y, ry) < REL_L2_TOL
