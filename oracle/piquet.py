"""Numpy restatement of the piquet field lookup (oracle only).

Restates cardgym/games/piquet/model.py: ``_onehot_bags`` 255-264 (every table's field sums
as one GEMM of one-hot token rows against the tables side by side, in the autocast dtype
or the tables' own) and the field part of ``PiquetEmbedding.forward`` 323-345 (ids =
tokens[..., :NUM_FIELDS] + the per-field row offsets); ``CardScorer.forward`` 348-363. The field vocabularies restate
cardgym/games/piquet/tokens.py:108-128 independently of the product's copy.
"""

from __future__ import annotations

import numpy as np

from .numerics import gelu, layer_norm, round_to

NUM_FIELDS = 32
CARD_START = NUM_FIELDS
FIELD_VOCAB = (8, 4, 3, 2, 33, 9, 9, 4, 4, 9, 76, 9, 3, 4, 64, 5, 3, 13, 3, 5, 13, 13, 100, 100, 141, 141, 6, 2,
               9, 16, 4, 149)
OFFSETS = np.concatenate([[0], np.cumsum(FIELD_VOCAB)[:-1]]).astype(np.int64)
ROWS = int(sum(FIELD_VOCAB))


def onehot_bags(ids: np.ndarray, tables: list[np.ndarray], storage: str = "fp32") -> list[np.ndarray]:
    """``_onehot_bags``: ids [..., F] (row ids), tables [rows, w_i] -> sums [..., w_i].

    ``zeros(N, rows).scatter_(1, ids, 1.0)`` marks each distinct row once; the product with
    the tables (rounded to ``storage`` first) is taken exactly (float64) and rounded once to
    ``storage``, which is what an fp32-accumulating GEMM computes up to its summation order.
    """

    flat = ids.reshape(-1, ids.shape[-1]).astype(np.int64)
    rows = tables[0].shape[0]
    if flat.size and (flat.min() < 0 or flat.max() >= rows):
        raise IndexError("field id outside the table")
    table = round_to(np.concatenate(tables, axis=1), storage)
    hot = np.zeros((flat.shape[0], rows), dtype=np.float64)
    np.put_along_axis(hot, flat, 1.0, axis=1)
    sums = round_to(hot @ table, storage)
    widths = [t.shape[1] for t in tables]
    parts = np.split(sums, np.cumsum(widths)[:-1], axis=1)
    return [p.reshape(*ids.shape[:-1], w) for p, w in zip(parts, widths)]


def field_sums(tokens: np.ndarray, tables: list[np.ndarray], storage: str = "fp32") -> list[np.ndarray]:
    """The field sums of ``PiquetEmbedding.forward`` (without the card-grid summary)."""

    ids = tokens[..., :NUM_FIELDS].astype(np.int64) + OFFSETS
    return onehot_bags(ids, tables, storage)


def card_scorer(hidden: np.ndarray, grid: np.ndarray, w: dict) -> np.ndarray:
    """``CardScorer.forward`` in float64: out(GELU(hidden(LayerNorm(query(h)[:, None] + card(grid) + card_id))))."""

    h = hidden.astype(np.float64)
    g = grid.astype(np.float64)
    query = h @ w["query.weight"].T.astype(np.float64) + w["query.bias"]
    mixed = query[:, None, :] + g @ w["card.weight"].T.astype(np.float64) + w["card_id.weight"].astype(np.float64)
    normed = layer_norm(mixed, w["norm.weight"].astype(np.float64), w["norm.bias"].astype(np.float64))
    hid = gelu(normed @ w["hidden.weight"].T.astype(np.float64) + w["hidden.bias"])
    return (hid @ w["out.weight"].T.astype(np.float64) + w["out.bias"])[..., 0]
