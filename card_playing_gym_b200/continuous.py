"""Continuous self-play collector: a fixed set of game slots kept full, refilled as games end.

Drop-in for cardgym/rl/continuous.py:55-408 (``Lane``, ``split_lanes``,
``ContinuousCollector(model, ...).collect(lanes, rng, version=)``). Each lane keeps
``in_flight`` games running; every game owns one KV row per seat for its whole life; a
collection returns each lane's ``quota`` of finished games (or, without a quota, every game its
source deals) and carries the games still running, with their rows, into the next call.

The work runs on ``rollout.RolloutEngine``: slots are split into ``cohorts`` that take turns,
so that the host steps one cohort's games while the device decodes and samples the other's
wave. The schedule is a queue of waves in flight: the oldest lands (its decisions are
recorded, its games stepped, finished games replaced), and its cohort's next wave is sent
while the lanes still want games.
"""

from __future__ import annotations

import gc
import random
import time
from collections import deque
from collections.abc import Callable
from contextlib import contextmanager
from dataclasses import dataclass, field, replace

import numpy as np
import torch

from .rollout import (ROW_BUCKET, SPAN_BUCKET, CollectionStats, Decision, DecisionRecord, EagerHalf, GameTrace,
                      GraphedHalf, PackedWave, RolloutEngine, RowTable, Trajectory, WaveInFlight, expect_decision,
                      pack_columns, pack_wave, queue_after_step, round_up, stack_features)

__all__ = [
    "ROW_BUCKET", "SPAN_BUCKET", "CollectionStats", "ContinuousCollector", "Decision", "DecisionRecord", "EagerHalf",
    "GraphedHalf", "Lane", "PackedWave", "RowTable", "Trajectory", "WaveInFlight", "pack_columns", "pack_wave",
    "round_up", "split_lanes", "stack_features",
]

KV_DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


@dataclass(frozen=True)
class Lane:
    """One kind of game kept running.

    ``deal(rng)`` returns a fresh game, or None once a finite source is spent. With ``quota = None``
    the lane runs until its source is spent and every game has ended; otherwise each collection
    returns exactly ``quota`` finished games from it.
    """

    name: str
    players: int  # cache rows per game
    in_flight: int
    quota: int | None
    deal: Callable[[random.Random], object | None] = field(compare=False)


def _share(total: int, index: int, count: int) -> int:
    """Worker ``index`` of ``count``'s part of ``total`` when parts differ by at most one, larger first."""

    whole, extra = divmod(total, count)
    return whole + (1 if index < extra else 0)


def split_lanes(lanes: list[Lane], index: int, count: int) -> list[Lane]:
    """Worker ``index`` of ``count``'s share of every lane: its part of the quota and of the games in
    flight (at least one), lanes whose quota share is empty left out (cardgym/rl/continuous.py:73-89)."""

    if any(lane.quota is None for lane in lanes):
        raise ValueError("Only lanes with a quota can be split between workers.")
    shares = [(lane, _share(lane.quota, index, count), _share(lane.in_flight, index, count)) for lane in lanes]
    return [replace(lane, quota=quota, in_flight=max(1, games)) for lane, quota, games in shares if quota > 0]


@contextmanager
def _fewer_gc_passes():
    """A wave allocates a few objects per decision (records, blocks), almost none in cycles; at the default
    young-generation threshold the cyclic collector rescans every game in flight every few hundred
    decisions. It runs far less often while a collection lasts."""

    saved = gc.get_threshold()
    gc.set_threshold(max(saved[0], 100_000), *saved[1:])
    try:
        yield
    finally:
        gc.set_threshold(*saved)


@dataclass
class _Slot:
    lane: int
    base: int  # first cache row
    cohort: int
    trace: GameTrace | None = None


class ContinuousCollector:
    """Keeps every lane's ``in_flight`` games running; ``collect`` returns each lane's quota of finished
    games. ``stats.policy_lag`` reports how many versions old the returned decisions are."""

    ROW_BUCKET = ROW_BUCKET
    SPAN_BUCKET = SPAN_BUCKET

    def __init__(self, model, *, device: torch.device | str = "cuda", precision: str | None = None,
                 kv_dtype: str | torch.dtype = "fp16", max_length: int, cohorts: int = 1, record_values: bool = False,
                 half_factory=None) -> None:
        if precision is not None and precision != getattr(model, "precision", precision):
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.device = torch.device(device)
        self.kv_dtype = KV_DTYPES[kv_dtype] if isinstance(kv_dtype, str) else kv_dtype
        self.max_length = max_length
        self.cohorts = max(1, cohorts)
        self.record_values = record_values
        self.half_factory = half_factory
        self.stats = CollectionStats()
        self.reset()

    def reset(self) -> None:
        """Drop every game in flight, every banked result and the KV pool."""

        self._shape: tuple | None = None
        self._slots: list[_Slot] = []
        self._banks: dict[str, deque[Trajectory]] = {}
        self._live: list[int] = []
        self.engine: RolloutEngine | None = None

    def release(self) -> None:
        """Nothing to free between updates: the pool holds the games in flight."""

    @property
    def in_flight(self) -> int:
        return sum(self._live)

    @torch.no_grad()
    def collect(self, lanes: list[Lane], rng: random.Random, *, version: int = 0) -> list[Trajectory]:
        started = time.perf_counter()
        self.stats = stats = CollectionStats()
        self._arrange(lanes)
        with _fewer_gc_passes():
            for slot in self._slots:
                if slot.trace is None:
                    self._refill(slot, lanes, rng)
            flights: deque[tuple[int, WaveInFlight]] = deque()
            for cohort in range(self.cohorts):
                self._send(cohort, flights, lanes)
            while flights:
                cohort, wave = flights.popleft()
                self._settle(cohort, wave, lanes, rng, version)
                self._send(cohort, flights, lanes)
        results = []
        for lane in lanes:
            bank = self._banks[lane.name]
            take = len(bank) if lane.quota is None else min(lane.quota, len(bank))
            results.extend(bank.popleft() for _ in range(take))
        versions = [record.version for trajectory in results for record in trajectory.decisions]
        stats.games = len(results)
        stats.in_flight = self.in_flight
        stats.policy_lag = float(version - np.mean(versions)) if versions else 0.0
        stats.collect_sec = time.perf_counter() - started
        return results

    # ------------------------------------------------------------------------------------------------
    def _arrange(self, lanes: list[Lane]) -> None:
        """Slots for the lanes' games in flight; a new layout starts from nothing."""

        shape = tuple((lane.name, lane.players, lane.in_flight) for lane in lanes)
        if shape == self._shape:
            return
        self.reset()
        self._shape = shape
        bases = np.cumsum([0] + [lane.players for lane in lanes for _ in range(lane.in_flight)])
        kinds = [index for index, lane in enumerate(lanes) for _ in range(lane.in_flight)]
        self._slots = [_Slot(lane=kind, base=int(bases[i]), cohort=i % self.cohorts) for i, kind in enumerate(kinds)]
        self._banks = {lane.name: deque() for lane in lanes}
        self._live = [0] * len(lanes)
        self.engine = RolloutEngine(self.model, device=self.device, kv_dtype=self.kv_dtype, max_length=self.max_length,
                                    record_values=self.record_values, half_factory=self.half_factory)
        self.engine.reserve(int(bases[-1]))

    def _wanted(self, lanes: list[Lane]) -> bool:
        """Whether some lane still needs games: a quota not yet met, or a quota-less lane with games running."""

        for index, lane in enumerate(lanes):
            if self._live[index] if lane.quota is None else len(self._banks[lane.name]) < lane.quota:
                return True
        return False

    def _refill(self, slot: _Slot, lanes: list[Lane], rng: random.Random) -> None:
        """Deal the slot a game; games over before their first decision are banked at once. A lane whose
        bank already covers its quota deals nothing."""

        lane = lanes[slot.lane]
        bank = self._banks[lane.name]
        while lane.quota is None or len(bank) < lane.quota:
            game = lane.deal(rng)
            if game is None:
                return
            trace = GameTrace(game, slot.base)
            self.engine.start(trace, game.prefix_tokens())
            if game.done():
                bank.append(trace.trajectory())
                continue
            expect_decision(trace)
            slot.trace = trace
            self._live[slot.lane] += 1
            return

    def _send(self, cohort: int, flights: deque, lanes: list[Lane]) -> None:
        if not self._wanted(lanes):
            return
        started = time.perf_counter()
        traces = [slot.trace for slot in self._slots if slot.cohort == cohort and slot.trace is not None]
        wave = self.engine.launch(traces, self.stats) if traces else None
        self.stats.forward_sec += time.perf_counter() - started
        if wave is not None:
            flights.append((cohort, wave))

    def _settle(self, cohort: int, wave: WaveInFlight, lanes: list[Lane], rng: random.Random, version: int) -> None:
        """Land the cohort's wave, step its games with the sampled actions, bank and replace finished games."""

        stats = self.stats
        t0 = time.perf_counter()
        wave.wait()
        t1 = time.perf_counter()
        stats.decisions += self.engine.land(wave, version)
        t2 = time.perf_counter()
        table = self.engine.table
        for slot in self._slots:
            trace = slot.trace
            if trace is None or slot.cohort != cohort:
                continue
            blocks = trace.game.step(trace.records[-1].action)
            trace.observe(blocks)
            if trace.game.done():
                self._banks[lanes[slot.lane].name].append(trace.trajectory())
                slot.trace = None
                self._live[slot.lane] -= 1
                self._refill(slot, lanes, rng)
            else:
                queue_after_step(trace, table, blocks)
                expect_decision(trace)
        stats.wait_sec += t1 - t0
        stats.sample_sec += t2 - t1
        stats.step_sec += time.perf_counter() - t2
