"""Plump token schema constants the field-lookup kernel needs.

Mirrors the v6 token layout of the reference (cardgym/games/plump/tokens.py:45-93 for
the slots, :121-214 for the NA ids and vocabulary sizes) and the embedder's field list
(cardgym/games/plump/model.py:55-56, 104-133). Only the numbers the B200 lookup uses
live here; the game rules stay with the reference's host engine.
"""

from __future__ import annotations

from dataclasses import dataclass

NUM_CARDS = 52
NUM_SUITS = 4
NUM_RANKS = 13

SLOT_TYPE = 0
SLOT_RANK = 2
SLOT_SUIT = 3
SLOT_CARD = 4
BASE_WIDTH = 16
REMAINING_HAND_SLOTS = 9
SLOT_REMAINING_HAND = BASE_WIDTH
SLOT_NA_PATTERN = SLOT_REMAINING_HAND + REMAINING_HAND_SLOTS
TOKEN_WIDTH = SLOT_NA_PATTERN + 1
TOKEN_TRICK_WIN = 5
NUM_TOKEN_TYPES = 7
NUM_NA_PATTERNS = 12

# Base fields the embedder sums: every base slot but the exact card id.
FIELDS = tuple(slot for slot in range(BASE_WIDTH) if slot != SLOT_CARD)


@dataclass(frozen=True)
class PlumpSchema:
    """Vocabulary limits; every NA id and table size derives from these two."""

    max_players: int = 5
    max_hand_size: int = 10

    @property
    def bid_count(self) -> int:
        return self.max_hand_size + 1

    @property
    def base_na_ids(self) -> tuple[int | None, ...]:
        p, n = self.max_players, self.max_hand_size
        bids_made_na = p + 1
        bid_sum_na = p * n + 1
        return (
            None, p, NUM_RANKS, NUM_SUITS, NUM_CARDS, n + 1, n, p,
            None, None, p, 0, bids_made_na, bid_sum_na, bid_sum_na, bids_made_na,
        )

    @property
    def base_vocab_sizes(self) -> tuple[int, ...]:
        p, n = self.max_players, self.max_hand_size
        return (
            NUM_TOKEN_TYPES, p + 1, NUM_RANKS + 1, NUM_SUITS + 1, NUM_CARDS + 1,
            n + 2, n + 1, p + 1, n + 1, p + 1, p + 1, 3,
            p + 2, p * n + 2, p * n + 2, p + 2,
        )

    def field_offsets(self) -> list[int]:
        sizes = [self.base_vocab_sizes[slot] for slot in FIELDS]
        return [sum(sizes[:i]) for i in range(len(sizes))]

    def field_rows(self) -> int:
        return sum(self.base_vocab_sizes[slot] for slot in FIELDS)

    def field_na_ids(self) -> list[int]:
        """Per summed field, the id that marks it absent (-1: always present)."""

        return [-1 if self.base_na_ids[slot] is None else self.base_na_ids[slot] for slot in FIELDS]

    @property
    def rank_offset(self) -> int:
        return self.field_offsets()[FIELDS.index(SLOT_RANK)]

    @property
    def suit_offset(self) -> int:
        return self.field_offsets()[FIELDS.index(SLOT_SUIT)]
