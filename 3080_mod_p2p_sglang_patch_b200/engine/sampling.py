"""Token selection: greedy, temperature, top-k, top-p (nucleus), seeded; and
the logit adjustments applied before it (presence / frequency / repetition
penalties, logit bias, minimum tokens before a stop id).

Plain greedy requests keep the fused path (vocab-parallel argmax, in the
decode CUDA graphs). A batch with any request that samples, adjusts logits or
asks for logprobs instead produces full logits (the LM-head shards
all-gathered across the TP ranks, so every rank holds the same values),
applies ``adjust_logits`` and calls ``sample``; every rank draws with the same
seeded generator, so all ranks pick the same token without another exchange.
"""
import dataclasses

import torch


@dataclasses.dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0  # 0 = greedy
    top_k: int = 0            # 0 = off
    top_p: float = 1.0        # 1 = off
    seed: int = None          # per-request seed (None: the engine's generator)
    # logit adjustments, applied before the choice (greedy or sampled)
    presence_penalty: float = 0.0     # OpenAI: minus this once for every token already generated
    frequency_penalty: float = 0.0    # OpenAI: minus this times each generated token's count
    repetition_penalty: float = 1.0   # HF: prompt + generated tokens' logits divided (> 0) or multiplied (< 0)
    logit_bias: tuple = ()            # ((token id, bias), ...)
    min_new_tokens: int = 0           # stop ids masked until this many tokens exist

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1

    @property
    def adjusts(self) -> bool:
        """Logits are changed before the choice (needs the full logits)."""
        return bool(self.presence_penalty or self.frequency_penalty or self.repetition_penalty != 1.0 or
                    self.logit_bias or self.min_new_tokens)


GREEDY = SamplingParams()


def adjust_logits(logits: torch.Tensor, params, prompts, outputs, stop_ids) -> torch.Tensor:
    """Apply each row's penalties, biases and min-token mask (in place on an
    fp32 copy). ``prompts`` / ``outputs`` / ``stop_ids``: per row, the
    request's prompt ids, generated ids so far and stop ids."""
    x = logits.float().clone()
    V = x.shape[1]
    for i, p in enumerate(params):
        if p is None or not p.adjusts:
            continue
        row = x[i]
        if p.repetition_penalty != 1.0:
            seen = torch.tensor(sorted(set(prompts[i]) | set(outputs[i])), dtype=torch.long, device=x.device)
            seen = seen[seen < V]
            vals = row[seen]
            row[seen] = torch.where(vals > 0, vals / p.repetition_penalty, vals * p.repetition_penalty)
        if (p.presence_penalty or p.frequency_penalty) and outputs[i]:
            ids = torch.tensor(outputs[i], dtype=torch.long, device=x.device)
            counts = torch.bincount(ids[ids < V], minlength=V).float()
            row -= p.frequency_penalty * counts + p.presence_penalty * (counts > 0).float()
        for tok, bias in p.logit_bias:
            if 0 <= tok < V:
                row[tok] += bias
        if p.min_new_tokens and len(outputs[i]) < p.min_new_tokens and stop_ids[i]:
            stops = torch.tensor([t for t in stop_ids[i] if 0 <= t < V], dtype=torch.long, device=x.device)
            row[stops] = float("-inf")
    return x


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
