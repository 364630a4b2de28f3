"""The fused audio head (dm3::audio_head + dm3::direction_score) against the oracle restating
CfgGraphs.run's head lines (engine.py:423-424) and direction_score (engine.py:476-479): the GEMV
logits within tolerance, the guidance and the index_copy bit-exact from the kernel's own logits,
the vocabulary buffer untouched elsewhere, log-sum-exp and score to 1e-5, CUDA-graph replay with a
changing strength and token, and the gathered-rows variant."""

import pytest
import torch

import oracle
from tests.golden import inputs
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu

V, K, BAND0, NB, EOS = 6000, 2048, 1000, 4096, 5999


def _setup():
    g = torch.Generator().manual_seed(61)
    lm = (torch.randn(V, K, generator=g) * 0.02).to(torch.bfloat16)
    cand = torch.cat([torch.tensor([EOS]), torch.arange(BAND0, BAND0 + NB)])
    hidden = inputs.decode_rows(2, seed=62, h=K)
    return lm, cand, hidden


def _guided_from(logits, st):
    """The reference's guidance on given logits, with torch's fp32 ops."""
    L = logits.cpu()
    return L[1:] + torch.tensor(st, dtype=torch.float32) * (L[:1] - L[1:])


def test_audio_head_matches_oracle(dm3):
    lm, cand, hidden = _setup()
    head = dm3.AudioHead(lm.cuda(), cand.cuda(), V)
    st = 1.7
    strength = torch.tensor([st], dtype=torch.float32, device="cuda")
    guided, logits = head(hidden.cuda(), strength)
    torch.cuda.synchronize()
    q, s = oracle.quantize_rows(lm[cand])
    ref_logits, ref_guided = oracle.audio_head(hidden, q, s, 1, cand, V, st)
    assert rel_l2(logits, ref_logits) < 5e-3
    assert (logits.cpu().to(torch.bfloat16).float() == logits.cpu()).all()  # bf16-rounded as the reference
    assert rel_l2(guided[0, cand], ref_guided[0, cand]) < 2e-2
    # the guidance and the scatter, bit-exact from the kernel's own logits
    assert torch.equal(guided[0, cand].cpu(), _guided_from(logits, st)[0])
    mask = torch.ones(V, dtype=torch.bool)
    mask[cand] = False
    assert torch.isinf(guided[0, mask.cuda()]).all() and (guided[0, mask.cuda()] < 0).all()
    assert torch.allclose(head.lse.cpu(), torch.logsumexp(logits.cpu(), -1), atol=1e-5, rtol=0)
    score = torch.zeros((), dtype=torch.float32, device="cuda")
    for tok in (BAND0 + 17, EOS, BAND0):
        token = torch.tensor([[tok, 3]], dtype=torch.int64, device="cuda")
        before = float(score)
        head.score_into(score, token[0, 0], EOS, BAND0)
        ref = float(oracle.direction_score(logits.cpu(), tok, EOS, BAND0))
        assert abs(float(score) - before - ref) < 1e-5, tok


def test_audio_head_graph_replay_and_gather(dm3):
    lm, cand, hidden = _setup()
    dev = torch.device("cuda")
    head = dm3.AudioHead(lm.to(dev), cand.to(dev), V)
    hid = hidden.to(dev).clone()
    strength = torch.tensor([1.0], dtype=torch.float32, device=dev)
    token = torch.tensor([BAND0 + 5], dtype=torch.int64, device=dev)
    score = torch.zeros((), dtype=torch.float32, device=dev)
    head(hid, strength)
    head.score_into(score, token, EOS, BAND0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        guided, logits = head(hid, strength)
        head.score_into(score, token, EOS, BAND0)
    for rep, (st, tok) in enumerate([(2.5, BAND0 + 9), (0.5, EOS), (3.0, BAND0 + 4095)]):
        hid.copy_(inputs.decode_rows(2, seed=70 + rep, h=K).to(dev))
        strength.fill_(st)
        token.fill_(tok)
        score.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(guided[0, cand.to(dev)].cpu(), _guided_from(logits, st)[0])
        ref = float(oracle.direction_score(logits.cpu(), tok, EOS, BAND0))
        assert abs(float(score) - ref) < 1e-5
    # the head gathered in the kernel from the full quantised matrix gives the same logits
    qf, sf = dm3.quantize(lm.to(dev))
    gathered = dm3.AudioHead(None, cand.to(dev), V, q=qf, s=sf, rows=cand.to(dev))
    g2, l2 = gathered(hid, strength)
    torch.cuda.synchronize()
    assert rel_l2(l2, logits) < 1e-3
    assert torch.equal(g2[0, cand.to(dev)].cpu(), _guided_from(l2, 3.0)[0])
