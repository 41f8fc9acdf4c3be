"""Legal-masked softmax and inverse-CDF sampling on the device.

Reference: cardgym/rl/ppo.py:75-94 (``masked_probabilities``, ``sample_rows``), run by
``sample_decisions`` (cardgym/rl/selfplay.py:532-567) on the host in numpy float32 with
one ``game.rng.random()`` uniform per decision. Here the host supplies those same
uniforms (float64) and the device returns the probabilities and the draws.
"""

from __future__ import annotations

import torch

from . import _native as nat


def masked_sample(logits: torch.Tensor, mask: torch.Tensor, uniforms: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(probabilities fp32 [R, A], actions int64 [R]) for logits [R, A], mask bool [R, A], uniforms f64 [R]."""

    rows, width = logits.shape
    logits = logits.float().contiguous()
    mask = mask.to(torch.uint8).contiguous()
    probs = torch.empty_like(logits)
    actions = torch.empty(rows, dtype=torch.int64, device=logits.device)
    nat.call("cg_masked_sample", nat.ptr(logits), nat.ptr(mask), nat.ptr(uniforms.to(torch.float64).contiguous()),
             rows, width, nat.ptr(probs), nat.ptr(actions), nat.stream_handle(logits.device))
    return probs, actions


def masked_probabilities(logits: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """Softmax over legal entries only; illegal entries get exactly zero."""

    zeros = torch.zeros(logits.shape[0], dtype=torch.float64, device=logits.device)
    return masked_sample(logits, mask, zeros)[0]


def sample_rows(logits: torch.Tensor, mask: torch.Tensor, uniforms: torch.Tensor) -> torch.Tensor:
    """One legal index per row, drawn by inverse CDF from the masked softmax of ``logits``."""

    return masked_sample(logits, mask, uniforms)[1]
