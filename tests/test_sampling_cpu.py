"""Sampling: greedy equivalence, top-k / top-p supports, the temperature
distribution, and seeded reproducibility (CPU tensors)."""
import importlib

import torch

smp = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.sampling")
P = smp.SamplingParams


def test_greedy_and_top1_are_argmax():
    x = torch.randn(4, 100, generator=torch.Generator().manual_seed(0))
    want = x.argmax(-1)
    assert torch.equal(smp.sample(x, [P()] * 4), want)
    assert torch.equal(smp.sample(x, [P(temperature=1.0, top_k=1)] * 4), want)


def test_top_k_and_top_p_restrict_the_support():
    x = torch.tensor([[5.0, 4.0, 3.0, 0.0, -1.0, -2.0]])
    g = torch.Generator().manual_seed(1)
    seen_k = {int(smp.sample(x, [P(temperature=5.0, top_k=3)], [g])[0]) for _ in range(300)}
    assert seen_k == {0, 1, 2}
    # probs at T=1: ~[0.66, 0.24, 0.09, ...]: top_p=0.8 keeps exactly the first two
    seen_p = {int(smp.sample(x, [P(temperature=1.0, top_p=0.8)], [g])[0]) for _ in range(300)}
    assert seen_p == {0, 1}
    # a tiny top_p always keeps the top token
    assert {int(smp.sample(x, [P(temperature=1.0, top_p=1e-6)], [g])[0]) for _ in range(50)} == {0}


def test_temperature_matches_softmax_frequencies():
    x = torch.tensor([[1.0, 0.0, -1.0]])
    g = torch.Generator().manual_seed(2)
    n = 6000
    counts = torch.zeros(3)
    for _ in range(n):
        counts[smp.sample(x, [P(temperature=2.0)], [g])[0]] += 1
    want = torch.softmax(x[0] / 2.0, 0)
    assert torch.allclose(counts / n, want, atol=0.025), (counts / n, want)


def test_seeded_draws_reproduce():
    x = torch.randn(1, 1000, generator=torch.Generator().manual_seed(3))
    a = [int(smp.sample(x, [P(temperature=1.0)], [torch.Generator().manual_seed(7)])[0]) for _ in range(5)]
    assert len(set(a)) == 1


def test_logit_adjustments():
    samp = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.sampling")
    SP = samp.SamplingParams
    logits = torch.tensor([[2.0, -1.0, 0.5, 3.0, 0.0],
                           [1.0, 1.0, 1.0, 1.0, 1.0],
                           [0.0, 0.0, 0.0, 0.0, 9.0]])
    params = [SP(repetition_penalty=2.0), SP(presence_penalty=0.5, frequency_penalty=0.25, logit_bias=((4, 3.0),)),
              SP(min_new_tokens=3)]
    out = samp.adjust_logits(logits, params, prompts=[[0, 1], [], []], outputs=[[3], [2, 2, 0], [7]],
                             stop_ids=[(), (), (4,)])
    assert torch.equal(out[0], torch.tensor([1.0, -2.0, 0.5, 1.5, 0.0]))     # seen: 0, 1, 3 (> 0 halved, < 0 doubled)
    assert torch.allclose(out[1], torch.tensor([1 - 0.5 - 0.25, 1.0, 1 - 0.5 - 0.5, 1.0, 4.0]))
    assert out[2, 4] == float("-inf") and out[2, :4].eq(0).all()            # the stop id waits for 3 tokens
    assert torch.equal(logits[0], torch.tensor([2.0, -1.0, 0.5, 3.0, 0.0]))  # the input is left as it was
    assert SP().adjusts is False and SP(min_new_tokens=1).adjusts and SP(temperature=0.5).adjusts is False


def test_batched_distribution_matches_the_per_row_definition():
    """sample_probs (one batched pass) equals temperature -> top-k -> top-p
    applied row by row, for a mix of settings."""
    samp = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.sampling")
    SP = samp.SamplingParams
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(6, 50, generator=g) * 3
    params = [SP(1.0), SP(0.7, top_k=5), SP(1.3, top_p=0.8), SP(0.5, top_k=10, top_p=0.5), SP(2.0, top_k=50),
              SP(1.0, top_k=1000)]

    def one(row, p):
        row = row / p.temperature
        if p.top_k and p.top_k < row.numel():
            row = row.masked_fill(row < torch.topk(row, p.top_k).values[-1], float("-inf"))
        if p.top_p < 1.0:
            sv, si = torch.sort(row, descending=True)
            pr = torch.softmax(sv, 0)
            sv = sv.masked_fill(torch.cumsum(pr, 0) - pr >= p.top_p, float("-inf"))
            row = torch.full_like(row, float("-inf")).scatter(0, si, sv)
        return torch.softmax(row, 0)

    got = samp.sample_probs(logits, params)
    want = torch.stack([one(logits[i], p) for i, p in enumerate(params)])
    assert torch.allclose(got, want, atol=1e-6)
    assert int((got[1] > 0).sum()) == 5 and int((got[5] > 0).sum()) == 50


def test_rows_sharing_a_generator_draw_together_and_reproduce():
    samp = importlib.import_module("3080_mod_p2p_sglang_patch_b200.engine.sampling")
    SP = samp.SamplingParams
    logits = torch.randn(5, 30, generator=torch.Generator().manual_seed(4))
    params = [SP(1.0), SP(), SP(1.0, top_k=3), SP(1.0), SP(0.9)]

    def run():
        shared, own = torch.Generator().manual_seed(10), torch.Generator().manual_seed(11)
        return samp.sample(logits, params, [shared, None, shared, own, shared])

    a, b = run(), run()
    assert torch.equal(a, b) and a[1] == logits[1].argmax()               # greedy row untouched
    assert a[2] in torch.topk(logits[2], 3).indices
