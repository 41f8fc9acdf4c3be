"""Numpy restatement of the piquet field lookup (oracle only).

Restates cardgym/games/piquet/model.py: ``_onehot_bags`` 255-264 (every table's field sums
as one GEMM of one-hot token rows against the tables side by side, in the autocast dtype
or the tables' own) and the field part of ``PiquetEmbedding.forward`` 323-345 (ids =
tokens[..., :NUM_FIELDS] + the per-field row offsets); ``CardScorer.forward`` 348-363;
``CardGrid`` 180-240 with ``GridBlock`` 129-177 and ``GridNorm`` 118-126. The field vocabularies restate
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


NUM_SUITS, NUM_RANKS = 4, 8
CARD_RANKS = np.arange(NUM_SUITS * NUM_RANKS) % NUM_RANKS  # card = suit * 8 + rank (piquet/cards.py)


def grid_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """GridNorm: RMSNorm over the card width with a gain (fp32 statistics in the reference)."""

    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * weight


def card_grid(codes: np.ndarray, w: dict, blocks: int = 2, kernel: int = 3, storage: str = "fp32",
              ranks: int = NUM_RANKS, circular: bool = False):
    """``CardGrid.forward``: card codes [N, 32] -> (cards [N, 32, width], summary [N, d]).

    ``storage="bf16"`` rounds where the reference's bf16 autocast does: every Linear / matmul
    output (the rank convolution with its bias, the suit mean, the across-suit projection,
    the output layer with its bias), their sum and the GELU; the residual grid, the norms and
    the final features stay fp32. The summary projection is left to the caller's GEMM.

    ``ranks=13, kernel=5, circular=True`` is rummy's ledger grid (cardgym/games/rummy/model.py:
    112-225): 52 cards, a circular convolution along the ranks."""

    f = lambda name: w[name].astype(np.float64)  # noqa: E731
    rnd = (lambda x: round_to(x, "bf16")) if storage == "bf16" else (lambda x: x)  # noqa: E731
    count = codes.shape[0]
    card_ranks = np.arange(NUM_SUITS * ranks) % ranks
    grid = f("code.weight")[codes.astype(np.int64)] + f("rank.weight")[card_ranks]
    width = grid.shape[-1]
    grid = grid.reshape(count, NUM_SUITS, ranks, width)
    half = kernel // 2
    for b in range(blocks):
        p = f"blocks.{b}."
        rows = rnd(grid_norm(grid, f(p + "norm.weight")))  # autocast casts the GEMM input
        conv = rnd(f(p + "along_rank.weight"))  # [hidden, width, kernel]
        hidden = conv.shape[0]
        along = np.zeros((count, NUM_SUITS, ranks, hidden))
        for tap in range(kernel):
            for o in range(ranks):
                i = o + tap - half
                if circular:
                    i %= ranks
                if 0 <= i < ranks:
                    along[:, :, o, :] += rows[:, :, i, :] @ conv[:, :, tap].T
        along = rnd(along + rnd(f(p + "along_rank.bias")))
        pooled = rnd(rows.mean(axis=1))  # [N, ranks, width]
        across = rnd(pooled @ rnd(f(p + "across_suits.weight")).T)  # [N, ranks, hidden]
        mixed = rnd(along + across[:, None])
        out = rnd(rnd(gelu(mixed)) @ rnd(f(p + "out.weight")).T + rnd(f(p + "out.bias")))
        grid = grid + out
    cards = grid_norm(grid, f("norm.weight")).reshape(count, NUM_SUITS * ranks, width)
    if "summary.weight" not in w:
        return cards, None
    summary = cards.reshape(count, -1) @ f("summary.weight").T
    return cards, summary
