"""Per-request sampling: temperature, top-k, top-p (nucleus) and per-request seeds.

Greedy requests (``temperature == 0``, the default) keep the argmax the
decode graph computes; a step with sampled requests draws their tokens from
the step's logits afterwards, on the device, in one batched pass:

* logits / temperature, then the top-k and top-p masks (ties at the k-th
  value are kept, as a sort-based mask does);
* a draw by the exponential race ``argmax(p_i / E_i)`` with ``E_i ~ Exp(1)``,
  which selects token i with probability ``p_i`` -- the noise comes from the
  engine's generator, or from the request's own when it carries a seed, so a
  seeded request reproduces its tokens whatever else is in the batch.

Penalties run before all of that, on the logits, with vLLM's meanings:
``presence_penalty`` subtracts a constant from every token already generated,
``frequency_penalty`` subtracts it once per occurrence, and
``repetition_penalty`` divides positive logits (multiplies negative ones) of
every token seen in the prompt or the output.

The reference takes these parameters through vLLM's sampler; the field names
and meanings follow the OpenAI completions API it serves.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0  # 0: greedy
    top_k: int = 0  # 0: off
    top_p: float = 1.0
    seed: int | None = None
    # generation also ends at these tokens (and at the model's EOS unless ignore_eos)
    stop_token_ids: tuple[int, ...] = ()
    ignore_eos: bool = False
    # per generated token: its log-probability under the model, and the ``logprobs`` most likely tokens
    logprobs: int | None = None
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0  # 1: off
    # stop tokens (EOS included) cannot end generation, and are not sampled, before this many tokens
    min_tokens: int = 0
    # OpenAI logit_bias: (token id, bias added to its logit) pairs, bias in [-100, 100]
    logit_bias: tuple[tuple[int, float], ...] = ()

    def __post_init__(self) -> None:
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if self.logprobs is not None and not 0 <= self.logprobs <= 20:
            raise ValueError("logprobs must be in [0, 20]")
        if not -2.0 <= self.presence_penalty <= 2.0 or not -2.0 <= self.frequency_penalty <= 2.0:
            raise ValueError("presence_penalty and frequency_penalty must be in [-2, 2]")
        if self.repetition_penalty <= 0.0:
            raise ValueError("repetition_penalty must be > 0")
        if self.min_tokens < 0:
            raise ValueError("min_tokens must be >= 0")
        if any(not -100.0 <= b <= 100.0 for _, b in self.logit_bias):
            raise ValueError("logit_bias values must be in [-100, 100]")

    @property
    def penalized(self) -> bool:
        """The logits are adjusted before the choice (penalties or a logit bias)."""
        return (self.presence_penalty != 0.0 or self.frequency_penalty != 0.0 or self.repetition_penalty != 1.0
                or bool(self.logit_bias))

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0 or self.top_k == 1


GREEDY = SamplingParams()


def make_generator(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def _token_counts(seqs: list[list[int]], V: int, device) -> torch.Tensor:
    """``[n, V]`` occurrence counts of each row's tokens."""
    width = max((len(t) for t in seqs), default=0)
    counts = torch.zeros(len(seqs), V + 1, device=device)
    if width:
        ids = torch.full((len(seqs), width), V, dtype=torch.long)
        for i, t in enumerate(seqs):
            if t:
                ids[i, : len(t)] = torch.tensor(t, dtype=torch.long).clamp_(0, V)
        counts.scatter_add_(1, ids.to(device), torch.ones(ids.shape, device=device))
    return counts[:, :V]


def apply_penalties(logits: torch.Tensor, params: list[SamplingParams], prompts: list[list[int]],
                    outputs: list[list[int]]) -> torch.Tensor:
    """Penalised fp32 copy of ``logits [n, V]``; rows without penalties are unchanged."""
    x = logits.float().clone()
    rows = [i for i, p in enumerate(params) if p.penalized]
    if not rows:
        return x
    dev, V = x.device, x.shape[1]
    idx = torch.tensor(rows, device=dev)
    sub = x.index_select(0, idx)
    out_counts = _token_counts([outputs[i] for i in rows], V, dev)
    rep = torch.tensor([params[i].repetition_penalty for i in rows], device=dev).unsqueeze(1)
    seen = (out_counts + _token_counts([prompts[i] for i in rows], V, dev)) > 0
    sub = torch.where(seen, torch.where(sub > 0, sub / rep, sub * rep), sub)
    freq = torch.tensor([params[i].frequency_penalty for i in rows], device=dev).unsqueeze(1)
    pres = torch.tensor([params[i].presence_penalty for i in rows], device=dev).unsqueeze(1)
    sub = sub - freq * out_counts - pres * (out_counts > 0).float()
    for j, i in enumerate(rows):
        for tok, bias in params[i].logit_bias:
            if 0 <= tok < V:
                sub[j, tok] += bias
    x[idx] = sub
    return x


def mask_tokens(logits: torch.Tensor, banned: list[list[int]]) -> torch.Tensor:
    """``logits`` with each row's ``banned`` tokens set to -inf (in place on an fp32 copy the caller owns)."""
    rows = [(i, t) for i, ts in enumerate(banned) for t in ts if 0 <= t < logits.shape[1]]
    if rows:
        r, c = zip(*rows)
        logits[torch.tensor(r, device=logits.device), torch.tensor(c, device=logits.device)] = float("-inf")
    return logits


def _on_device(values: list, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A small host list as a device tensor without a stream synchronisation: a copy from pageable
    memory waits for the stream's queued work, one from pinned memory is only ordered after it."""
    t = torch.tensor(values, dtype=dtype, pin_memory=device.type == "cuda")
    return t.to(device, non_blocking=True)


def filtered_probs(logits: torch.Tensor, params: list[SamplingParams]) -> torch.Tensor:
    """Row-wise probabilities after temperature, top-k and top-p; ``logits [n, V]``.  Enqueues device
    work only (no host read-back), so a step launched ahead of its predecessor's read-back can sample."""
    x = logits.float()
    dev = x.device
    temp = _on_device([max(p.temperature, 1e-6) for p in params], torch.float32, dev).unsqueeze(1)
    x = x / temp
    V = x.shape[1]
    ks = [p.top_k if 0 < p.top_k < V else 0 for p in params]
    need_sort = any(ks) or any(p.top_p < 1.0 for p in params)
    if need_sort:
        sorted_x, _ = x.sort(dim=-1, descending=True)
        if any(ks):
            kk = _on_device([k if k else V for k in ks], torch.int64, dev)
            kth = sorted_x.gather(1, (kk - 1).unsqueeze(1))
            x = x.masked_fill(x < kth, float("-inf"))
            sorted_x = sorted_x.masked_fill(torch.arange(V, device=dev)[None, :] >= kk[:, None], float("-inf"))
        top_p = _on_device([p.top_p for p in params], torch.float32, dev).unsqueeze(1)
        if any(p.top_p < 1.0 for p in params):
            sp = torch.softmax(sorted_x, dim=-1)
            # keep the smallest prefix whose mass reaches top_p (the first token always stays)
            before = sp.cumsum(dim=-1) - sp
            keep_sorted = before < top_p
            n_keep = keep_sorted.sum(dim=-1, keepdim=True).clamp_min(1)
            cutoff = sorted_x.gather(1, n_keep - 1)
            x = x.masked_fill(x < cutoff, float("-inf"))
    return torch.softmax(x, dim=-1)


def sample(logits: torch.Tensor, params: list[SamplingParams], generators: list[torch.Generator | None],
           default_generator: torch.Generator | None = None) -> torch.Tensor:
    """One token per row of ``logits [n, V]`` (int32); greedy rows take the argmax."""
    out = torch.argmax(logits.float(), dim=-1).to(torch.int32)
    rows = [i for i, p in enumerate(params) if not p.greedy]
    if not rows:
        return out
    idx = _on_device(rows, torch.int64, logits.device)
    probs = filtered_probs(logits.index_select(0, idx), [params[i] for i in rows])
    noise = torch.empty_like(probs)
    shared = [j for j, i in enumerate(rows) if generators[i] is None]
    if shared:
        sel = _on_device(shared, torch.int64, logits.device)
        noise[sel] = torch.empty(len(shared), probs.shape[1], device=probs.device).exponential_(
            generator=default_generator)
    for j, i in enumerate(rows):
        if generators[i] is not None:
            noise[j].exponential_(generator=generators[i])
    drawn = torch.argmax(probs / noise.clamp_min(1e-30), dim=-1).to(torch.int32)
    out[idx] = drawn
    return out


def token_logprobs(logits: torch.Tensor, tokens: torch.Tensor, top_n: int) -> tuple[list[float], list[list]]:
    """Log-probabilities (of the raw model distribution) of ``tokens`` per row, and each row's
    ``top_n`` most likely ``(token, logprob)`` pairs."""
    lp = torch.log_softmax(logits.float(), dim=-1)
    chosen = lp.gather(1, tokens.long().view(-1, 1)).view(-1).tolist()
    if top_n <= 0:
        return chosen, [[] for _ in chosen]
    v, i = lp.topk(top_n, dim=-1)
    return chosen, [list(zip(ii, vv)) for ii, vv in zip(i.tolist(), v.tolist())]


__all__ = ["GREEDY", "SamplingParams", "filtered_probs", "make_generator", "sample", "token_logprobs"]
