"""Test-only CPU restatement of the continuous collector's wave packing.

Test infrastructure: only tests may import this module. It restates, entry by entry, how
cardgym/rl/continuous.py:316-331 (``ContinuousCollector._launch``) lays out one decode wave,
to check the vectorised ``card_playing_gym_b200.continuous.pack_wave`` against. Parity is
pinned by the reference's own semantics read from that code: rows bucketed to a multiple of
64, padding rows at position 0 of the scratch row with zero tokens, a short block padded by
repeating its last token, span rounded up to a multiple of 32.
"""

from __future__ import annotations

import numpy as np


def round_up(value: int, multiple: int) -> int:
    return -(-value // multiple) * multiple


def pack_wave(entries, scratch: int, row_bucket: int = 64, span_bucket: int = 32):
    """(tokens, positions, offsets, cache_rows, span) for (row, position, block) entries."""

    run = max(len(block) for _, _, block in entries)
    count = len(entries)
    rows = round_up(count, row_bucket)
    width = entries[0][2].shape[1]
    tokens = np.zeros((rows, run, width), dtype=np.int64)
    cache_rows = np.full(rows, scratch, dtype=np.int64)
    positions = np.zeros(rows, dtype=np.int64)
    offsets = np.zeros(rows, dtype=np.int64)
    for index, (row, position, block) in enumerate(entries):
        tokens[index, : len(block)] = block
        tokens[index, len(block):] = block[-1]
        cache_rows[index] = row
        positions[index] = position
        offsets[index] = len(block) - 1
    span = round_up(int(positions.max()) + run, span_bucket)
    return tokens, positions, offsets, cache_rows, span
