"""Numpy restatement of the rummy candidate pointer head (oracle only).

Restates cardgym/games/rummy/model.py:292-357 (``CandidateScorer.forward``) literally: the
per-slot card counts (NO_CARD entries add zero), their product with the grid, the
concatenated projections and identity tables, the kind and size embeddings, then
LayerNorm, the hidden layer, exact GELU and the output layer, in float64.
"""

from __future__ import annotations

import numpy as np

from .numerics import gelu, layer_norm

NUM_CARDS = 52
NO_CARD = NUM_CARDS


def candidate_scorer(hidden, grid, kind, cards, target, taken, w: dict) -> np.ndarray:
    rows, width = kind.shape
    slots = 2 if taken is None else 3
    f = lambda name: w[name].astype(np.float64)  # noqa: E731
    ids = np.concatenate([cards, target], axis=-1).astype(np.int64)
    present = ids != NO_CARD
    offsets = np.repeat(np.arange(2), cards.shape[-1]) * NUM_CARDS
    counts = np.zeros((rows, width, slots * NUM_CARDS))
    index = np.where(present, ids + offsets, 0)
    for r in range(rows):
        for c in range(width):
            np.add.at(counts[r, c], index[r, c], present[r, c].astype(np.float64))
    if taken is not None:
        counts[..., 2 * NUM_CARDS:] = taken
    summed = np.matmul(counts.reshape(rows, width * slots, NUM_CARDS), grid.astype(np.float64)).reshape(rows, width, -1)
    projections = np.concatenate([f("card.weight"), f("target.weight"), f("taken.weight")][:slots], axis=1)
    identities = np.concatenate([f("card_id.weight"), f("target_id.weight"), f("taken_id.weight")][:slots], axis=0)
    sizes = present[..., : cards.shape[-1]].sum(-1)
    candidate = summed @ projections.T + counts @ identities + f("kind.weight")[kind] + f("size.weight")[sizes]
    query = hidden.astype(np.float64) @ f("query.weight").T + f("query.bias")
    mixed = layer_norm(query[:, None, :] + candidate, f("norm.weight"), f("norm.bias"))
    hid = gelu(mixed @ f("hidden.weight").T + f("hidden.bias"))
    return (hid @ f("out.weight").T + f("out.bias"))[..., 0]
