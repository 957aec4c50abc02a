"""CPU restatement of the reference sampler (model/sampling.py).

``sample_logits`` follows sample_logits_stateless's CPU branch
(model/sampling.py:127-225): repetition penalty where the seen mask is set
(:55-65), greedy first-argmax for temperature 0 (:183-187), otherwise
``_cpu_sample_row`` (:68-95) on ``prepared[row] / temperature[row]``: top-k
with k <= 0 meaning the whole vocabulary, softmax over the top-k values,
top-p dropping ranks whose exclusive cumulative mass exceeds top_p and
renormalising, then ``torch.multinomial`` with a private generator seeded by
``(seed + 0x9E3779B97F4A7C15 * offset) mod 2**63``.

``row_details`` exposes the intermediate filtered probabilities (rank order)
and the Exp(1) noise the same generator yields, for the GPU parity entry:
torch's CPU multinomial(p, 1) is argmax(p / Exp(1)) with that noise.
Test infrastructure only (see the package docstring).
"""

from __future__ import annotations

import torch

GOLDEN_RATIO_64 = 0x9E3779B97F4A7C15


def mixed_seed(seed: int, offset: int) -> int:
    return (int(seed) + GOLDEN_RATIO_64 * int(offset)) & ((1 << 63) - 1)


def apply_penalty(logits: torch.Tensor, penalty: torch.Tensor, seen: torch.Tensor | None) -> torch.Tensor:
    if seen is None:
        return logits
    adjusted = torch.where(logits > 0, logits / penalty.unsqueeze(1), logits * penalty.unsqueeze(1))
    return torch.where(seen, adjusted, logits)


def filtered_probs(scaled_row: torch.Tensor, top_k: int, top_p: float):
    """(probabilities in top-k rank order, token ids of the ranks)."""

    vocab = scaled_row.shape[0]
    k_eff = vocab if top_k <= 0 else min(top_k, vocab)
    values, indices = torch.topk(scaled_row.float(), k_eff)
    probs = torch.softmax(values, dim=-1)
    if top_p < 1.0:
        order = torch.argsort(probs, descending=True)
        ordered = probs[order]
        remove = ordered.cumsum(dim=-1) - ordered > top_p
        ordered = ordered.masked_fill(remove, 0)
        probs = torch.zeros_like(probs).scatter(0, order, ordered)
        probs = probs / probs.sum().clamp_min(torch.finfo(probs.dtype).tiny)
    return probs, indices


def sample_row(scaled_row: torch.Tensor, top_k: int, top_p: float, seed: int, offset: int) -> int:
    probs, indices = filtered_probs(scaled_row, top_k, top_p)
    generator = torch.Generator(device="cpu")
    generator.manual_seed(mixed_seed(seed, offset))
    pick = torch.multinomial(probs, 1, generator=generator)
    return int(indices[pick].item())


def row_noise(length: int, seed: int, offset: int) -> torch.Tensor:
    """The Exp(1) draws multinomial(p, 1) consumes for a length-`length` p."""

    generator = torch.Generator(device="cpu")
    generator.manual_seed(mixed_seed(seed, offset))
    return torch.empty(length, dtype=torch.float32).exponential_(1, generator=generator)


def scaled_rows(logits, temperature, repetition_penalty=None, seen_token_mask=None) -> list[torch.Tensor | None]:
    """prepared[row] / temperature[row] with the reference's dtype rules (None for greedy rows)."""

    if repetition_penalty is None:
        repetition_penalty = torch.ones_like(temperature)
    prepared = apply_penalty(logits, repetition_penalty, seen_token_mask)
    out: list[torch.Tensor | None] = []
    for row in range(logits.shape[0]):
        if float(temperature[row]) == 0.0:
            out.append(None)
        else:
            out.append(prepared[row] / temperature[row])
    return out


def sample_logits(logits, temperature, top_k, top_p, seed, offset, *, repetition_penalty=None,
                  seen_token_mask=None) -> torch.Tensor:
    """Tokens int64 [rows], CPU semantics of sample_logits_stateless."""

    if repetition_penalty is None:
        repetition_penalty = torch.ones_like(temperature)
    prepared = apply_penalty(logits, repetition_penalty, seen_token_mask)
    tokens = prepared.argmax(dim=-1).to(torch.long)
    for row, scaled in enumerate(scaled_rows(logits, temperature, repetition_penalty, seen_token_mask)):
        if scaled is None:
            continue
        tokens[row] = sample_row(scaled, int(top_k[row]), float(top_p[row]), int(seed[row]), int(offset[row]))
    return tokens


def row_details(logits, temperature, top_k, top_p, seed, offset, *, repetition_penalty=None, seen_token_mask=None):
    """Per row: (k_eff, probs [k_eff] rank order, ids [k_eff], noise [k_eff], token) or None for greedy rows."""

    details = []
    for row, scaled in enumerate(scaled_rows(logits, temperature, repetition_penalty, seen_token_mask)):
        if scaled is None:
            details.append(None)
            continue
        probs, ids = filtered_probs(scaled, int(top_k[row]), float(top_p[row]))
        noise = row_noise(probs.shape[0], int(seed[row]), int(offset[row]))
        token = int(ids[torch.argmax(probs / noise)].item())
        details.append((probs.shape[0], probs, ids, noise, token))
    return details
