"""Numpy restatement of the plump embedder and actor heads (oracle only).

Restates cardgym/games/plump/model.py: ``_bag`` 94-101, ``PlumpEmbedding.__init__``
104-133 and ``forward`` 135-167, ``PlumpActor.card_logits`` 204-207,
``policy_logits`` 209-214, ``player_values`` 216-217 (``value_mlp`` of
cardgym/nn/model.py:12-17). The schema numbers restate
cardgym/games/plump/tokens.py:45-93 and 121-214 independently of the product's
copy, so a test can hold the two against each other.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .numerics import gelu, layer_norm
from .trunk import Precision, Trunk, TrunkShape, TrunkWeights, value_layers

NUM_CARDS, NUM_SUITS, NUM_RANKS = 52, 4, 13
SLOT_TYPE, SLOT_RANK, SLOT_SUIT, SLOT_CARD = 0, 2, 3, 4
SLOT_REMAINING_HAND, SLOT_NA_PATTERN = 16, 25
TOKEN_TRICK_WIN = 5
FIELDS = tuple(slot for slot in range(16) if slot != SLOT_CARD)


def schema_tables(max_players: int = 5, max_hand_size: int = 10):
    """(vocabulary sizes, NA ids) per base slot: tokens.py:183-214."""

    p, n = max_players, max_hand_size
    sizes = (7, p + 1, NUM_RANKS + 1, NUM_SUITS + 1, NUM_CARDS + 1, n + 2, n + 1, p + 1,
             n + 1, p + 1, p + 1, 3, p + 2, p * n + 2, p * n + 2, p + 2)
    na = (None, p, NUM_RANKS, NUM_SUITS, NUM_CARDS, n + 1, n, p, None, None, p, 0,
          p + 1, p * n + 1, p * n + 1, p + 1)
    return sizes, na


@dataclass
class Embedding:
    offsets: np.ndarray  # per summed field
    na_ids: np.ndarray  # -1: always present
    rank_offset: int
    suit_offset: int
    tables: list[tuple[np.ndarray, np.ndarray] | None]  # (fields, na_pattern) for d, ple, value

    @classmethod
    def from_state(cls, state: dict, max_players: int = 5, max_hand_size: int = 10) -> "Embedding":
        sizes, na = schema_tables(max_players, max_hand_size)
        field_sizes = [sizes[slot] for slot in FIELDS]
        offsets = np.array([sum(field_sizes[:i]) for i in range(len(field_sizes))], dtype=np.int64)
        na_ids = np.array([-1 if na[slot] is None else na[slot] for slot in FIELDS], dtype=np.int64)
        tables = []
        for name in ("", "ple_", "value_"):
            key = f"embedding.{name}fields.weight"
            if key in state:
                tables.append(
                    (np.asarray(state[key], np.float64), np.asarray(state[f"embedding.{name}na_pattern.weight"], np.float64))
                )
            else:
                tables.append(None)
        return cls(
            offsets=offsets,
            na_ids=na_ids,
            rank_offset=int(offsets[FIELDS.index(SLOT_RANK)]),
            suit_offset=int(offsets[FIELDS.index(SLOT_SUIT)]),
            tables=tables,
        )

    def forward(self, tokens: np.ndarray, dtype=np.float64):
        """Sum of present field rows + the NA-pattern row (+ remaining-hand rank/suit rows on TRICK_WIN).

        Summation order follows the reference: the 15 field rows in field order,
        then the pattern row, then (TRICK_WIN rows) the hand bag (rank, suit) per
        card in slot order, added last as one bag.
        """

        tokens = np.asarray(tokens, dtype=np.int64)
        fields = tokens[..., list(FIELDS)]
        ids = fields + self.offsets
        valid = (self.na_ids < 0) | (fields != self.na_ids)
        pattern = tokens[..., SLOT_NA_PATTERN]
        trick_win = tokens[..., SLOT_TYPE] == TOKEN_TRICK_WIN
        remaining = tokens[..., SLOT_REMAINING_HAND:SLOT_NA_PATTERN]
        card_valid = remaining < NUM_CARDS
        safe = np.minimum(remaining, NUM_CARDS - 1)
        ranks = safe % NUM_RANKS + self.rank_offset
        suits = safe // NUM_RANKS + self.suit_offset

        outputs = []
        for entry in self.tables:
            if entry is None:
                outputs.append(None)
                continue
            table, na_table = (t.astype(dtype) for t in entry)
            out = np.zeros((*tokens.shape[:-1], table.shape[1]), dtype=dtype)
            for f in range(ids.shape[-1]):
                out = out + table[ids[..., f]] * valid[..., f, None]
            out = out + na_table[pattern]
            hand = np.zeros_like(out)
            for c in range(remaining.shape[-1]):
                hand = hand + table[ranks[..., c]] * card_valid[..., c, None]
                hand = hand + table[suits[..., c]] * card_valid[..., c, None]
            out = np.where(trick_win[..., None], out + hand, out)
            outputs.append(out)
        return tuple(outputs)


@dataclass
class Heads:
    bid_w: np.ndarray
    bid_b: np.ndarray
    card_w: np.ndarray  # [52, d] = rank[r] + suit[s]
    card_b: np.ndarray
    value_w1: np.ndarray
    value_b1: np.ndarray
    value_w2: np.ndarray
    value_b2: np.ndarray

    @classmethod
    def from_state(cls, state: dict) -> "Heads":
        get = lambda k: np.asarray(state[k], np.float64)  # noqa: E731
        cards = np.arange(NUM_CARDS)
        ranks, suits = cards % NUM_RANKS, cards // NUM_RANKS
        # The reference sums the two rows in float32 (model.py:205-206).
        card_w = (np.asarray(state["card_rank.weight"], np.float32)[ranks]
                  + np.asarray(state["card_suit.weight"], np.float32)[suits]).astype(np.float64)
        card_b = (np.asarray(state["card_rank_bias"], np.float32)[ranks]
                  + np.asarray(state["card_suit_bias"], np.float32)[suits]).astype(np.float64)
        return cls(get("bid_head.weight"), get("bid_head.bias"), card_w, card_b,
                   get("value_head.0.weight"), get("value_head.0.bias"),
                   get("value_head.2.weight"), get("value_head.2.bias"))

    def policy_logits(self, hidden: np.ndarray, head: str) -> np.ndarray:
        if head == "bid":
            return hidden @ self.bid_w.T + self.bid_b
        if head == "play":
            return hidden @ self.card_w.T + self.card_b
        raise ValueError(f"Unknown plump policy head {head!r}.")

    def player_values(self, hidden: np.ndarray) -> np.ndarray:
        return gelu(hidden @ self.value_w1.T + self.value_b1) @ self.value_w2.T + self.value_b2


class PlumpActor:
    """Embedder + trunk + heads over a reference-named state dict."""

    def __init__(self, state: dict, config: dict, prec: Precision | None = None) -> None:
        n_layers = config["n_layers"]
        shape = TrunkShape(
            d_model=config["d_model"], n_layers=n_layers, n_heads=config["n_heads"],
            n_kv_heads=config["n_kv_heads"], d_ff=config["d_ff"], per_layer_dim=config["per_layer_dim"],
            value_layers=value_layers(n_layers, config["value_embeddings"]),
        )
        self.prec = prec or Precision()
        self.embedding = Embedding.from_state(state, config.get("max_players", 5), config.get("max_hand_size", 10))
        self.trunk = Trunk(TrunkWeights.from_state(state, shape), self.prec)
        self.heads = Heads.from_state(state)

    def prepare(self, tokens: np.ndarray):
        return self.trunk.condition(*self.embedding.forward(tokens, self.prec.dtype))

    def forward_hidden(self, tokens: np.ndarray) -> np.ndarray:
        return self.trunk.forward(*self.prepare(tokens))

    def forward_prefill(self, tokens, cache, rows):
        return self.trunk.forward_prefill(*self.prepare(tokens), cache, rows)

    def forward_ragged(self, tokens, positions, cache, readout_offsets, span=None, rows=None):
        return self.trunk.forward_ragged(*self.prepare(tokens), cache, positions, readout_offsets, span, rows)

    def new_cache(self, capacity: int, max_len: int):
        from .trunk import Cache

        s = self.trunk.s
        return Cache(s.n_layers, capacity, s.n_kv_heads, max_len, s.head_dim, self.prec)

    def final_norm(self, x: np.ndarray) -> np.ndarray:
        return layer_norm(x, self.trunk.w.final_w, self.trunk.w.final_b)
