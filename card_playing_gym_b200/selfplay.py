"""Batch self-play collector: a list of games played together until the last one ends.

Drop-in for cardgym/rl/selfplay.py:208-484 (``SelfPlayCollector(model, ...).collect(games)``),
with its schedule: games ordered longest expected ``lifetime()`` first, played in chunks of at
most ``max_rows`` KV rows, each chunk's games dealt round-robin into ``cohorts`` that take turns
on the device; every game's decisions drawn from its own ``rng``.

It runs on ``rollout.RolloutEngine``, the continuous collector's engine, without refills: a
chunk's games get their rows once, their prefixes go out as the first wave (a ragged append from
position 0, one entry per observer), and each cohort then alternates one wave and one host step
of its games until none is left. Waves decode gathered rows, so the rows of finished games are
simply left out of later waves; there is no compaction step (``stats.compactions`` stays 0).
"""

from __future__ import annotations

import time
from collections import deque

import numpy as np
import torch

from .continuous import KV_DTYPES, _fewer_gc_passes
from .rollout import (ROW_BUCKET, SPAN_BUCKET, CollectionStats, GameTrace, RolloutEngine, Trajectory, expect_decision,
                      queue_after_step)


class SelfPlayCollector:
    ROW_BUCKET = ROW_BUCKET
    SPAN_BUCKET = SPAN_BUCKET

    def __init__(self, model, *, device: torch.device | str = "cuda", precision: str | None = None,
                 kv_dtype: str | torch.dtype = "fp16", max_rows: int, max_length: int, cohorts: int = 1,
                 record_values: bool = False, half_factory=None) -> None:
        if precision is not None and precision != getattr(model, "precision", precision):
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.device = torch.device(device)
        self.kv_dtype = KV_DTYPES[kv_dtype] if isinstance(kv_dtype, str) else kv_dtype
        self.max_rows = max_rows
        self.max_length = max_length
        self.cohorts = max(1, cohorts)
        self.record_values = record_values
        self.half_factory = half_factory
        self.engine: RolloutEngine | None = None
        self.stats = CollectionStats()

    def release(self) -> None:
        """Drop the KV pool; it is dead weight during the update's backward."""

        self.engine = None

    @torch.no_grad()
    def collect(self, games: list, version: int = 0) -> list[Trajectory]:
        started = time.perf_counter()
        self.stats = CollectionStats(games=len(games))
        if self.engine is None:
            self.engine = RolloutEngine(self.model, device=self.device, kv_dtype=self.kv_dtype,
                                        max_length=self.max_length, record_values=self.record_values,
                                        half_factory=self.half_factory)
        results: list[Trajectory | None] = [None] * len(games)
        with _fewer_gc_passes():
            for chunk in self._chunks(games):
                self._play(chunk, games, results, version)
        self.stats.collect_sec = time.perf_counter() - started
        return results

    def _chunks(self, games: list):
        """Game indices, longest expected lifetime first (ties keep list order), cut into the longest runs
        whose rows fit in ``max_rows`` (a game larger than that runs alone)."""

        lifetimes = np.array([getattr(game, "lifetime", lambda: 0)() for game in games], dtype=np.float64)
        order = np.argsort(-lifetimes, kind="stable")
        ends = np.cumsum([games[i].num_players for i in order])
        first, used = 0, 0
        while first < len(order):
            last = max(int(np.searchsorted(ends, used + self.max_rows, side="right")), first + 1)
            yield order[first:last].tolist()
            used = int(ends[last - 1])
            first = last

    def _play(self, chunk: list[int], games: list, results: list, version: int) -> None:
        engine, stats = self.engine, self.stats
        rows = sum(games[index].num_players for index in chunk)
        engine.reserve(rows)
        stats.peak_rows = max(stats.peak_rows, rows)
        count = min(self.cohorts, len(chunk))
        cohorts: list[list[tuple[int, GameTrace]]] = []
        base = 0
        for cohort in range(count):
            members = []
            for index in chunk[cohort::count]:  # every cohort keeps lifetimes descending
                trace = GameTrace(games[index], base)
                engine.start(trace, games[index].prefix_tokens())
                expect_decision(trace)
                members.append((index, trace))
                base += games[index].num_players
            cohorts.append(members)
        flights: deque = deque()
        for cohort, members in enumerate(cohorts):
            self._send(cohort, members, flights)
        while flights:
            cohort, wave = flights.popleft()
            t0 = time.perf_counter()
            wave.wait()
            t1 = time.perf_counter()
            stats.decisions += engine.land(wave, version)
            t2 = time.perf_counter()
            survivors = []
            for index, trace in cohorts[cohort]:
                blocks = trace.game.step(trace.records[-1].action)
                trace.observe(blocks)
                if trace.game.done():
                    results[index] = trace.trajectory()
                else:
                    queue_after_step(trace, engine.table, blocks)
                    expect_decision(trace)
                    survivors.append((index, trace))
            cohorts[cohort] = survivors
            stats.wait_sec += t1 - t0
            stats.sample_sec += t2 - t1
            stats.step_sec += time.perf_counter() - t2
            self._send(cohort, survivors, flights)

    def _send(self, cohort: int, members, flights: deque) -> None:
        if not members:
            return
        started = time.perf_counter()
        wave = self.engine.launch([trace for _, trace in members], self.stats)
        self.stats.forward_sec += time.perf_counter() - started
        if wave is not None:
            flights.append((cohort, wave))
