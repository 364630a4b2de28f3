"""Expert-parallel prefill and the sharded decode layer: the algorithm on gloo CPU ranks
(oracle.ep_oracle) against the one-process oracle, and the NVLink kernels on 2 GPUs against the
one-GPU kernels."""

import os

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from tests import ep_worker
from tests.golden import inputs
from tests.helpers import oracle_shared, rel_l2, routed_layer


def _spawn(fn, world, tmp_path):
    store = str(tmp_path / "store")
    mp.start_processes(fn, args=(world, store, str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    return [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]


@pytest.mark.parametrize("world", [2, 4])
def test_ep_algorithm_matches_single_process(tmp_path, world):
    res = _spawn(ep_worker.cpu_rank, world, tmp_path)
    h, i, e, k, t = 256, 128, 16, 4, 24
    layer = routed_layer(400, h=h, i=i, e=e)
    bias = inputs.zipf_bias(401, e=e)
    x = inputs.decode_rows(t, seed=402, h=h)
    ry, rids, rw = oracle.moe_layer(x, layer["gate"], layer["experts"], k, logits_bf16=True, logit_bias=bias,
                                    sw=oracle_shared(layer, 128), g=layer["sh_gate"])
    y = torch.cat([r["y"] for r in res])
    ids = torch.cat([r["ids"] for r in res])
    assert torch.equal(ids, rids)
    assert torch.equal(torch.cat([r["w"] for r in res]), rw)
    assert rel_l2(y, ry) < 1e-5


@pytest.mark.gpu
def test_ep_prefill_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(ep_worker.gpu_rank, 2, tmp_path)
    for r in res:
        assert r["status"] == 0, r
        assert r["fused_ids"] and r["fused_w"], r
        assert r["fused_y"], r
        assert r["split_y0"] and r["split_y1"], r
        assert r["graph_y"], r
        assert r["placed_y"], r
        assert r["decode_status"] == 0 and r["decode_ok"], r
