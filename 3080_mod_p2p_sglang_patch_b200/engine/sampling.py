"""Token sampling: greedy, temperature, top-k, top-p (nucleus), seeded.

Greedy requests keep the fused path (vocab-parallel argmax, in the decode
CUDA graphs). A batch with any sampled request instead produces full logits
(the LM-head shards all-gathered across the TP ranks, so every rank holds
the same values) and calls ``sample``; every rank draws with the same seeded
generator, so all ranks pick the same token without another exchange.
"""
import dataclasses

import torch


@dataclasses.dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0  # 0 = greedy
    top_k: int = 0            # 0 = off
    top_p: float = 1.0        # 1 = off
    seed: int = None          # per-request seed (None: the engine's generator)

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1


GREEDY = SamplingParams()


def sample(logits: torch.Tensor, params, generators=None) -> torch.Tensor:
    """Next token per row of ``logits`` [B, V] (any float dtype) under
    ``params`` (one SamplingParams per row). ``generators``: one
    torch.Generator (or None) per row for the draws. Returns int64 [B]."""
    B = logits.shape[0]
    out = torch.empty(B, dtype=torch.int64, device=logits.device)
    x = logits.float()
    for i, p in enumerate(params):
        row = x[i]
        if p.greedy:
            out[i] = row.argmax()
            continue
        row = row / p.temperature
        if p.top_k and p.top_k < row.numel():
            kth = torch.topk(row, p.top_k).values[-1]
            row = row.masked_fill(row < kth, float("-inf"))
        if p.top_p < 1.0:
            sorted_vals, idx = torch.sort(row, descending=True)
            probs = torch.softmax(sorted_vals, dim=0)
            # keep the smallest prefix whose mass reaches top_p (always the top token)
            drop = torch.cumsum(probs, dim=0) - probs >= p.top_p
            sorted_vals = sorted_vals.masked_fill(drop, float("-inf"))
            row = torch.full_like(row, float("-inf")).scatter(0, idx, sorted_vals)
        probs = torch.softmax(row, dim=0)
        g = generators[i] if generators is not None else None
        out[i] = torch.multinomial(probs, 1, generator=g)[0]
    return out
