"""Rummy candidate pointer head on the device.

Reference: cardgym/games/rummy/model.py:292-357 (``CandidateScorer.forward``), called by
``RummyActor.policy_logits`` (391-399) with the candidate features that
cardgym/games/rummy/selfplay.py:28-50 builds: per candidate its kind, the cards it moves
(``cards``), a lay-off's target meld (``target``), NO_CARD-padded to MAX_MELD_CARDS, and for
draw decisions the counts of each card type it takes from the pile (``taken``).
"""

from __future__ import annotations

import torch

from . import _native as nat

NUM_CARDS = 52
NO_CARD = NUM_CARDS
MAX_MELD_CARDS = 13


class CandidateScorer:
    """``CandidateScorer.forward(hidden, grid, kind, cards, target, taken=None) -> logits fp32 [N, K]``.

    Built from the reference module's parameters (``prefix + "query.weight"`` etc., as in a
    RummyActor ``state_dict`` with prefix ``"scorer."``). fp32 arithmetic.
    """

    NAMES = ("query.weight", "query.bias", "card.weight", "target.weight", "taken.weight", "card_id.weight",
             "target_id.weight", "taken_id.weight", "kind.weight", "size.weight", "norm.weight", "norm.bias",
             "hidden.weight", "hidden.bias", "out.weight", "out.bias")

    def __init__(self, state: dict, prefix: str = "", device: torch.device | str = "cuda"):
        self.params = {
            name: torch.as_tensor(state[prefix + name]).detach().to(device=device, dtype=torch.float32).contiguous()
            for name in self.NAMES
        }
        p = self.params
        dim, d = p["query.weight"].shape
        self.weights = nat.CandidateScorerWeights(
            d, p["card.weight"].shape[1], dim, p["card_id.weight"].shape[0], p["kind.weight"].shape[0],
            p["size.weight"].shape[0], *[nat.ptr(p[name]) for name in self.NAMES],
        )

    def __call__(self, hidden: torch.Tensor, grid: torch.Tensor, kind: torch.Tensor, cards: torch.Tensor,
                 target: torch.Tensor, taken: torch.Tensor | None = None) -> torch.Tensor:
        count, candidates = kind.shape
        if cards.shape[-1] != target.shape[-1]:
            raise ValueError("cards and target lists must have the same length (the reference's slot layout)")
        hidden = hidden.float().contiguous()
        if grid.dtype not in nat.DTYPE_CODES:
            grid = grid.float()
        grid = grid.contiguous()
        kind = kind.long().contiguous()
        cards = cards.long().contiguous()
        target = target.long().contiguous()
        if taken is not None:
            taken = taken.float().contiguous()
        logits = torch.empty((count, candidates), dtype=torch.float32, device=hidden.device)
        nat.call("cg_candidate_scorer", self.weights, nat.ptr(hidden), count, candidates, cards.shape[-1],
                 nat.ptr(grid), nat.DTYPE_CODES[grid.dtype], nat.ptr(kind), nat.ptr(cards), nat.ptr(target),
                 nat.ptr(taken), nat.ptr(logits), nat.stream_handle(hidden.device))
        return logits
