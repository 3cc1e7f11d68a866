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


def sample_probs(logits: torch.Tensor, params) -> torch.Tensor:
    """The sampling distribution of every row of ``logits`` [n, V] under its
    SamplingParams (none greedy): temperature, then top-k, then top-p (the
    smallest prefix of the sorted distribution whose mass reaches top_p,
    always the top token), in one batched pass. fp32 [n, V]."""
    x = logits.float()
    n, V = x.shape
    dev = x.device
    x = x / torch.tensor([p.temperature for p in params], device=dev)[:, None]
    ks = [p.top_k if 0 < p.top_k < V else 0 for p in params]
    if any(ks):
        kmax = max(ks)
        top = torch.topk(x, kmax, dim=-1).values                          # [n, kmax], sorted
        pick = torch.tensor([max(k, 1) - 1 for k in ks], device=dev)
        kth = top.gather(1, pick[:, None])
        kth = torch.where(torch.tensor(ks, device=dev)[:, None] > 0, kth, torch.full_like(kth, float("-inf")))
        x = x.masked_fill(x < kth, float("-inf"))                         # ties with the k-th stay
    tops = [p.top_p for p in params]
    if any(t < 1.0 for t in tops):
        sv, si = torch.sort(x, descending=True, dim=-1)
        pr = torch.softmax(sv, dim=-1)
        drop = torch.cumsum(pr, dim=-1) - pr >= torch.tensor(tops, device=dev)[:, None]
        sv = sv.masked_fill(drop, float("-inf"))
        x = torch.full_like(x, float("-inf")).scatter(1, si, sv)
    return torch.softmax(x, dim=-1)


def sample(logits: torch.Tensor, params, generators=None) -> torch.Tensor:
    """Next token per row of ``logits`` [B, V] (any float dtype) under
    ``params`` (one SamplingParams per row). ``generators``: one
    torch.Generator (or None) per row for the draws; rows that share a
    generator draw in one batched call, in row order. Returns int64 [B]."""
    out = logits.float().argmax(-1)                                        # greedy rows
    idx = [i for i, p in enumerate(params) if not p.greedy]
    if not idx:
        return out
    rows = torch.tensor(idx, device=logits.device)
    probs = sample_probs(logits.index_select(0, rows), [params[i] for i in idx])
    gens = [generators[i] if generators is not None else None for i in idx]
    groups = {}
    for j, g in enumerate(gens):                                           # by generator, first-use order
        groups.setdefault(id(g), (g, []))[1].append(j)
    for g, js in groups.values():
        sel = torch.tensor(js, device=logits.device)
        draws = torch.multinomial(probs.index_select(0, sel), 1, generator=g)[:, 0]
        out[rows.index_select(0, sel)] = draws
    return out
