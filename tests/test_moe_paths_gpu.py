"""The two decode-layer paths on the GPU: the default route kernel + cluster kernel against the
four-kernel chain (DM3_CLUSTER=0, read once per process, so it runs in a child process on the same
inputs), and the cluster path's determinism (its sums are 64-bit fixed-point integers, so repeated
calls give the same bits whatever order the CTAs finish in)."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.golden import inputs
from tests.helpers import rel_l2, routed_layer as _routed_layer, to_dev

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

_CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import drama3_b200 as dm3
d = torch.load(sys.argv[2])
outs = []
for x in d["xs"]:
    y, ids, w = dm3.ops.moe_layer(x.cuda(), d["gate"].cuda(), 8, True, None, d["w13"].cuda(), d["s13"].cuda(),
                                  d["w2"].cuda(), d["s2"].cuda(), d["sh_w13"].cuda(), d["sh_s13"].cuda(),
                                  d["sh_w2"].cuda(), d["sh_s2"].cuda(), d["sh_gate"].cuda(), None)
    outs.append((y.cpu(), ids.cpu(), w.cpu()))
torch.save(outs, sys.argv[3])
"""


def _layer_call(dm3, d, x):
    return dm3.ops.moe_layer(x.cuda(), d["gate"].cuda(), 8, True, None, d["w13"], d["s13"], d["w2"], d["s2"],
                             d["sh_w13"], d["sh_s13"], d["sh_w2"], d["sh_s2"], d["sh_gate"].cuda(), None)


def test_cluster_path_matches_four_kernel_chain(dm3, tmp_path):
    layer = _routed_layer(120, srows=128)
    ex, sh = layer["experts"], layer["sh"]
    d = {"gate": layer["gate"], "w13": ex["w13"], "s13": ex["s13"], "w2": ex["w2"], "s2": ex["s2"],
         "sh_w13": sh["w13"], "sh_s13": sh["s13"], "sh_w2": sh["w2"], "sh_s2": sh["s2"], "sh_gate": layer["sh_gate"],
         "xs": [inputs.decode_rows(t, seed=121 + t) for t in (1, 2, 4)]}
    torch.save(d, tmp_path / "in.pt")
    env = dict(os.environ, DM3_CLUSTER="0")
    res = subprocess.run([sys.executable, "-c", _CHILD, str(ROOT), str(tmp_path / "in.pt"), str(tmp_path / "out.pt")],
                         env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    legacy = torch.load(tmp_path / "out.pt")
    dev = to_dev({k: v for k, v in d.items() if k not in ("xs", "gate", "sh_gate")})
    dev["gate"], dev["sh_gate"] = d["gate"], d["sh_gate"]
    for x, (ly, lids, lw) in zip(d["xs"], legacy):
        y, ids, w = _layer_call(dm3, dev, x)
        assert torch.equal(ids.cpu(), lids), "the two paths selected different experts"
        assert torch.equal(w.cpu(), lw), "the two paths computed different routing weights"
        # the paths split h exactly in different groupings and sum in different orders (fp32 vs
        # exact fixed point): outputs agree to well inside the parity tolerance
        assert rel_l2(y, ly) < 5e-3


def test_cluster_path_is_deterministic(dm3):
    layer = _routed_layer(130, srows=128)
    ex, sh = to_dev(layer["experts"]), to_dev(layer["sh"])
    d = {"gate": layer["gate"], "w13": ex["w13"], "s13": ex["s13"], "w2": ex["w2"], "s2": ex["s2"],
         "sh_w13": sh["w13"], "sh_s13": sh["s13"], "sh_w2": sh["w2"], "sh_s2": sh["s2"], "sh_gate": layer["sh_gate"]}
    x = inputs.decode_rows(2, seed=131)
    first = _layer_call(dm3, d, x)[0].clone()
    for _ in range(5):
        assert torch.equal(_layer_call(dm3, d, x)[0], first)
