"""Batch self-play collector: deal a batch of games together and decode until the last one ends.

Reference: cardgym/rl/selfplay.py:208-484 (``SelfPlayCollector``). Games are ordered longest
expected lifetime first and run in chunks of at most ``max_rows`` cache rows, split into
``cohorts`` that take turns (the host steps one cohort's games while the device decodes the
other's). Each cohort prefills every prefix (rows sharing a prefix length share one
``forward_prefill``), then repeats one wave per decision: sample, step every live game, slide the
surviving games' cache rows down so that the live rows stay a dense prefix of the pool
(``KVCache.copy_rows``, counted in ``stats.compactions``), and append every observer's new tokens
with one ragged forward over that prefix, padded to a multiple of ``ROW_BUCKET`` rows.

On the device, as in ``continuous.ContinuousCollector``: each launch scores its readouts and
samples them there (``continuous.launch_decisions``), with each game's ``rng.random()`` drawn when
its decision is launched (after ``decision()``, before the next ``step()``, as
``sample_decisions`` draws it); only probabilities, actions and values come back to the host.
Pointer heads get the readout token's grid cards from the model's ``pop_context``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .continuous import (CollectionStats, LiveGame, Trajectory, _pinned, _Wave, launch_decisions, record_decisions,
                         restart_contexts, round_up)

_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


@dataclass
class _Cohort:
    cache: object
    live: list[tuple[int, LiveGame]]
    waves: list[_Wave] = field(default_factory=list)  # launched, not yet received


class SelfPlayCollector:
    ROW_BUCKET = 64
    SPAN_BUCKET = 32

    def __init__(self, model, *, device: torch.device | str = "cuda", precision: str | None = None,
                 kv_dtype: str | torch.dtype = "fp16", max_rows: int, max_length: int, cohorts: int = 1,
                 record_values: bool = False) -> None:
        if precision is not None and precision != getattr(model, "precision", precision):
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.device = torch.device(device)
        self.kv_dtype = _DTYPES[kv_dtype] if isinstance(kv_dtype, str) else kv_dtype
        self.max_rows = max_rows
        self.cohorts = max(1, cohorts)
        self.record_values = record_values
        # One spare position past the longest stream absorbs ragged padding.
        self.cache_length = max_length + 1
        self._caches: dict[int, object] = {}
        self.stats = CollectionStats()

    def release(self) -> None:
        """Drop the cached KV pools."""

        self._caches = {}

    @torch.no_grad()
    def collect(self, games: list, version: int = 0) -> list[Trajectory]:
        started = time.perf_counter()
        self.stats = CollectionStats(games=len(games))
        order = sorted(range(len(games)), key=lambda i: -getattr(games[i], "lifetime", lambda: 0)())
        results: dict[int, Trajectory] = {}
        chunk: list[int] = []
        rows = 0
        for index in order:
            players = games[index].num_players
            if chunk and rows + players > self.max_rows:
                self._run(chunk, games, results, version)
                chunk, rows = [], 0
            chunk.append(index)
            rows += players
        if chunk:
            self._run(chunk, games, results, version)
        self.stats.collect_sec = time.perf_counter() - started
        return [results[index] for index in range(len(games))]

    # ------------------------------------------------------------------

    def _ensure_cache(self, slot: int, rows: int):
        cache = self._caches.get(slot)
        if cache is None or cache.capacity < rows:
            self._caches.pop(slot, None)
            capacity = max(rows, min(self.max_rows, rows + rows // 4))
            cache = self.model.new_cache(capacity, self.cache_length, self.kv_dtype)
            self._caches[slot] = cache
        return cache

    def _run(self, indices: list[int], games: list, results: dict[int, Trajectory], version: int) -> None:
        count = min(self.cohorts, len(indices))
        cohorts: list[_Cohort] = []
        total_rows = 0
        for slot in range(count):
            members = indices[slot::count]  # interleaved: each cohort keeps lifetimes descending
            rows = sum(games[index].num_players for index in members)
            total_rows += rows
            live, row = [], 0
            for index in members:
                game = games[index]
                live.append((index, LiveGame(game=game, base=row, lengths=[0] * game.num_players,
                                             blocks=[[] for _ in range(game.num_players)])))
                row += game.num_players
            cohorts.append(_Cohort(cache=self._ensure_cache(slot, rows), live=live))
        self.stats.peak_rows = max(self.stats.peak_rows, total_rows)
        for cohort in cohorts:
            self._prefill(cohort)
        while any(cohort.live for cohort in cohorts):
            for cohort in cohorts:
                if cohort.live:
                    self._wave(cohort, results, version)

    def _launch(self, cohort: _Cohort, hidden: torch.Tensor, context: torch.Tensor | None,
                states: list[LiveGame]) -> None:
        uniforms = [state.game.rng.random() for state in states]
        cohort.waves.append(launch_decisions(self.model, hidden, context, states, uniforms,
                                             values=self.record_values))

    def _context(self, rows: torch.Tensor, positions: torch.Tensor) -> torch.Tensor | None:
        pop = getattr(self.model, "pop_context", None)
        context = pop() if pop is not None else None
        return None if context is None else context[rows, positions]

    def _prefill(self, cohort: _Cohort) -> None:
        """Encode every prefix; rows sharing a prefix length share one forward (selfplay.py:376-404)."""

        started = time.perf_counter()
        groups: dict[int, list[tuple[LiveGame, int, np.ndarray]]] = {}
        for _, state in cohort.live:
            state.pending = state.game.decision()
            for seat, prefix in enumerate(state.game.prefix_tokens()):
                groups.setdefault(prefix.shape[0], []).append((state, seat, prefix))
                state.blocks[seat].append(prefix)
                state.lengths[seat] = prefix.shape[0]
        for length, entries in groups.items():
            tokens = _pinned(np.stack([prefix for _, _, prefix in entries]).astype(np.int64), self.device)
            rows = _pinned(np.asarray([state.base + seat for state, seat, _ in entries], dtype=np.int64), self.device)
            hidden = self.model.forward_prefill(tokens, cohort.cache, rows)
            readout = [(position, state) for position, (state, seat, _) in enumerate(entries)
                       if state.pending.seat == seat]
            for position, state in readout:
                state.readout = entries[position][2][-1]
            self.stats.forward_rows += len(entries) * length
            if readout:
                index = _pinned(np.asarray([p for p, _ in readout], dtype=np.int64), self.device)
                context = self._context(index, torch.full_like(index, length - 1))
                self._launch(cohort, hidden.index_select(0, index), context, [state for _, state in readout])
            elif getattr(self.model, "pop_context", None) is not None:
                self.model.pop_context()
        self.stats.forward_sec += time.perf_counter() - started

    def _receive(self, cohort: _Cohort, version: int) -> None:
        started = time.perf_counter()
        for wave in cohort.waves:
            if wave.fence is not None:
                wave.fence.synchronize()
        self.stats.wait_sec += time.perf_counter() - started
        for wave in cohort.waves:
            self.stats.decisions += record_decisions(wave, version)
        cohort.waves = []

    def _wave(self, cohort: _Cohort, results: dict[int, Trajectory], version: int) -> None:
        """Receive one cohort's decisions, act in every live game, launch the next decode
        (selfplay.py:304-334)."""

        self.stats.waves += 1
        t0 = time.perf_counter()
        self._receive(cohort, version)
        t1 = time.perf_counter()
        appends: list[tuple[LiveGame, list[np.ndarray]]] = []
        survivors: list[tuple[int, LiveGame]] = []
        for index, state in cohort.live:
            blocks = state.game.step(state.decisions[-1].action)
            for seat, block in enumerate(blocks):
                if len(block):
                    state.blocks[seat].append(block)
            if state.game.done():
                results[index] = self._finish(state)
            else:
                appends.append((state, restart_contexts(state, blocks)))
                survivors.append((index, state))
        self.stats.sample_sec += t1 - t0
        self.stats.step_sec += time.perf_counter() - t1
        if len(survivors) != len(cohort.live):
            self._compact(cohort, [state for _, state in survivors])
        cohort.live = survivors
        if appends:
            self._append(cohort, appends)

    @staticmethod
    def _finish(state: LiveGame) -> Trajectory:
        streams = [np.concatenate(blocks, axis=0) for blocks in state.blocks]
        return Trajectory(game=state.game, streams=streams, decisions=state.decisions,
                          returns=np.asarray(state.game.returns(), dtype=np.float64))

    def _compact(self, cohort: _Cohort, survivors: list[LiveGame]) -> None:
        """Slide survivors down so live rows stay a dense prefix of the pool (selfplay.py:351-372)."""

        sources: list[int] = []
        targets: list[int] = []
        length = 0
        row = 0
        for state in survivors:
            if state.base != row:
                for seat in range(state.game.num_players):
                    sources.append(state.base + seat)
                    targets.append(row + seat)
                length = max(length, max(state.lengths))
                state.base = row
            row += state.game.num_players
        if sources:
            self.stats.compactions += 1
            cohort.cache.copy_rows(_pinned(np.asarray(sources, dtype=np.int64), self.device),
                                   _pinned(np.asarray(targets, dtype=np.int64), self.device), length)

    def _append(self, cohort: _Cohort, appends: list[tuple[LiveGame, list[np.ndarray]]]) -> None:
        """One ragged forward over the live prefix of the pool (selfplay.py:406-459)."""

        started = time.perf_counter()
        run = max(len(block) for _, blocks in appends for block in blocks)
        live_rows = appends[-1][0].base + appends[-1][0].game.num_players
        rows = max(live_rows, min(round_up(live_rows, self.ROW_BUCKET), cohort.cache.capacity))
        width = next(block.shape[1] for _, blocks in appends for block in blocks if len(block))
        # Rows past the live prefix are shape padding: zeros, written at position 0.
        tokens = np.zeros((rows, run, width), dtype=np.int64)
        positions = np.zeros(rows, dtype=np.int64)
        offsets = np.zeros(rows, dtype=np.int64)
        readout_rows: list[int] = []
        states: list[LiveGame] = []
        longest = 0
        for state, blocks in appends:
            for seat, block in enumerate(blocks):
                row = state.base + seat
                count = len(block)
                positions[row] = state.lengths[seat]
                if count:
                    tokens[row, :count] = block
                    tokens[row, count:] = block[-1]  # padding repeats the last token; its output is dropped
                    offsets[row] = count - 1
                state.lengths[seat] += count
            longest = max(longest, max(state.lengths))
            state.pending = state.game.decision()
            if not len(blocks[state.pending.seat]):
                raise AssertionError("The next actor's stream received no readout token.")
            state.readout = blocks[state.pending.seat][-1]
            readout_rows.append(state.base + state.pending.seat)
            states.append(state)
        if longest >= self.cache_length:
            raise RuntimeError("A stream outgrew the model's maximum sequence length.")
        span = min(round_up(int(positions.max()) + run, self.SPAN_BUCKET), cohort.cache.max_len)
        hidden = self.model.forward_ragged(_pinned(tokens, self.device), _pinned(positions, self.device),
                                           cohort.cache, _pinned(offsets, self.device), span=span)
        self.stats.forward_rows += rows * run
        self.stats.padded_rows += rows * run - sum(len(block) for _, blocks in appends for block in blocks)
        index = _pinned(np.asarray(readout_rows, dtype=np.int64), self.device)
        context = self._context(index, _pinned(offsets[readout_rows], self.device))
        self._launch(cohort, hidden.index_select(0, index), context, states)
        self.stats.forward_sec += time.perf_counter() - started
