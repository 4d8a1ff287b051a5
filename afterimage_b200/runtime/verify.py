"""Speculative verification of a draft chain -- drop-in for the reference's
afterimage/runtime/verify.py (sample_categorical :29-30, temperature_probs
:32-50, speculative_sample_step :53-103).

Standard chain speculation: draft token i is accepted with probability
min(1, p_target / p_draft); the first rejection is replaced by a sample from
the normalised residual max(p_target - p_draft, 0); if every draft token is
accepted a bonus token is drawn from the target's next distribution. At
temperature <= 0 both distributions are one-hot, so the procedure emits
exactly the target's greedy tokens for any draft.
"""
from __future__ import annotations

import torch


def sample_categorical(p: torch.Tensor, generator: torch.Generator | None = None) -> int:
    return int(torch.multinomial(p, 1, generator=generator).item())


def temperature_probs(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """softmax(logits / T), or one-hot at the argmax when T <= 0, in the
    logits' own dtype (BF16 logits give BF16 probabilities, as in the
    reference), so a seeded generator samples the same tokens."""
    if temperature <= 0:
        probs = torch.zeros_like(logits)
        probs.scatter_(-1, logits.argmax(dim=-1, keepdim=True), 1.0)
        return probs
    return torch.softmax(logits / temperature, dim=-1)


def speculative_sample_step(draft_probs: list[torch.Tensor], target_probs: list[torch.Tensor],
                            draft_tokens: list[int], bonus_target_probs: torch.Tensor,
                            generator: torch.Generator | None = None) -> tuple[list[int], int]:
    """Returns (tokens, n_accepted_from_draft); tokens holds the accepted
    draft prefix plus exactly one correction or bonus token."""
    accepted: list[int] = []
    dev = generator.device if generator is not None else None
    for i, x in enumerate(draft_tokens):
        p = float(target_probs[i][x])
        q = float(draft_probs[i][x])
        u = float(torch.rand(1, generator=generator, device=dev))
        if u <= min(1.0, p / max(q, 1e-12)):
            accepted.append(x)
            continue
        residual = torch.clamp(target_probs[i] - draft_probs[i], min=0.0)
        total = float(residual.sum())
        # q dominating p everywhere: sample the target itself
        dist = residual / total if total > 1e-12 else target_probs[i]
        accepted.append(sample_categorical(dist, generator))
        return accepted, i
    accepted.append(sample_categorical(bonus_target_probs, generator))
    return accepted, len(draft_tokens)
