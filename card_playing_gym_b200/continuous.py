"""Continuous self-play collector: a fixed pool of games in flight, refilled as games end.

Reference: cardgym/rl/continuous.py:55-408 (``Lane``, ``split_lanes``, ``ContinuousCollector``)
and the helpers it takes from cardgym/rl/selfplay.py (``restart_contexts`` 172-190,
``sample_decisions`` 532-567, ``_round_up`` 204-205). The host side keeps the reference's
protocol: games implement ``SelfPlayGame`` (``prefix_tokens``, ``decision``, ``step``,
``done``, ``returns``, ``context_starts``, a per-game ``rng``), each game owns one cache row
per seat, a wave decodes only the rows that received tokens (gathered by index, padded to a
multiple of ``ROW_BUCKET`` with entries that write a scratch row past every game's rows), and
``cohorts = 2`` lets the host step one group of games while the device decodes the other's.

What runs where. One wave is, on the device and in stream order: the host-packed inputs
uploaded from pinned memory, one ``DecodeGraphs`` replay (field lookup, the ragged trunk
decode into the KV pool, every head's logits and the per-seat values), a gather of the
readout rows, legal-masked softmax and inverse-CDF sampling for each head group
(``sampling.masked_sample``) and the copy of only the readouts' probabilities, actions and
values back to pinned host memory, closed by one event. The host never sees logits.

Uniforms. ``sample_decisions`` draws one ``game.rng.random()`` per decision after the wave's
logits arrive. Here it is drawn when the wave is launched, which is after the game's
``decision()`` and before its next ``step()`` exactly as there; every game owns its ``rng``
(cardgym/games/*/selfplay.py seed ``^ 0x5EED``) and nothing else draws from it in between,
so each game sees the same sequence of uniforms.
"""

from __future__ import annotations

import gc
import random
import time
from collections import deque
from collections.abc import Callable
from dataclasses import dataclass, field, replace

import numpy as np
import torch

ROW_BUCKET = 64
SPAN_BUCKET = 32


def round_up(value: int, multiple: int) -> int:
    return -(-value // multiple) * multiple


@dataclass
class Decision:
    """What the acting seat must choose now (selfplay.py:51-59)."""

    seat: int
    head: str
    legal: np.ndarray  # bool [actions]; actions index the head's output
    features: dict[str, np.ndarray] | None = None


@dataclass
class DecisionRecord:
    """One sampled decision (selfplay.py:113-124)."""

    seat: int
    head: str
    position: int  # readout index in the seat's own stream
    action: int
    probs: np.ndarray  # masked behaviour policy, float32 [actions]
    features: dict[str, np.ndarray] | None = None
    version: int = 0
    value: np.ndarray | None = None


@dataclass
class Trajectory:
    game: object
    streams: list[np.ndarray]  # per absolute seat, [length, width]
    decisions: list[DecisionRecord]
    returns: np.ndarray


@dataclass
class CollectionStats:
    """The reference's counters (selfplay.py:134-150)."""

    games: int = 0
    decisions: int = 0
    waves: int = 0
    forward_rows: int = 0
    padded_rows: int = 0
    peak_rows: int = 0
    compactions: int = 0
    collect_sec: float = 0.0
    forward_sec: float = 0.0  # host time preparing and launching device work
    wait_sec: float = 0.0  # host time blocked on the device
    sample_sec: float = 0.0
    step_sec: float = 0.0
    in_flight: int = 0
    policy_lag: float = 0.0


@dataclass(frozen=True)
class Lane:
    """One kind of game kept running (continuous.py:55-70).

    ``deal(rng)`` returns a fresh game, or None once a finite source is spent. With
    ``quota = None`` the lane runs until its source is spent and every game has ended;
    otherwise each collection returns exactly ``quota`` finished games from it.
    """

    name: str
    players: int  # cache rows per game
    in_flight: int
    quota: int | None
    deal: Callable[[random.Random], object | None] = field(compare=False)


def split_lanes(lanes: list[Lane], index: int, count: int) -> list[Lane]:
    """Worker ``index`` of ``count``'s share of each lane's quota and games in flight
    (continuous.py:73-89); shares differ by at most one game, empty shares are left out."""

    shares = []
    for lane in lanes:
        if lane.quota is None:
            raise ValueError("Only lanes with a quota can be split between workers.")
        quota = lane.quota // count + (index < lane.quota % count)
        in_flight = lane.in_flight // count + (index < lane.in_flight % count)
        if quota > 0:
            shares.append(replace(lane, quota=quota, in_flight=max(1, in_flight)))
    return shares


@dataclass
class LiveGame:
    """A game in flight (selfplay.py:153-169)."""

    game: object
    base: int  # first cache row
    lengths: list[int]  # per observer cached tokens (Python ints: the collector's inner loops index them)
    blocks: list[list[np.ndarray]]  # per observer recorded blocks
    decisions: list[DecisionRecord] = field(default_factory=list)
    pending: Decision | None = None
    readout: np.ndarray | None = None  # the pending actor's last token
    offsets: list[int] | None = None  # per observer, stream tokens before its current context

    def __post_init__(self) -> None:
        if self.offsets is None:
            self.offsets = [0] * len(self.lengths)


def restart_contexts(state: LiveGame, blocks: list[np.ndarray]) -> list[np.ndarray]:
    """Apply the game's context restarts after a step; returns the blocks to decode
    (selfplay.py:172-190). A restarted observer's cached length drops to zero: the new
    context is written from position 0 and causal attention never reaches the stale keys."""

    starts = state.game.context_starts()
    if starts is None:
        return blocks
    decoded = list(blocks)
    for seat, start in enumerate(starts):
        if start is None:
            continue
        state.offsets[seat] += state.lengths[seat] + start
        state.lengths[seat] = 0
        decoded[seat] = blocks[seat][start:]
    return decoded


@dataclass
class PackedWave:
    tokens: np.ndarray  # int64 [rows, run, width]
    positions: np.ndarray  # int64 [rows]
    offsets: np.ndarray  # int64 [rows], each row's last real token
    cache_rows: np.ndarray  # int64 [rows]
    span: int
    count: int  # real entries; the rest write the scratch row
    real_tokens: int = 0  # tokens of the real entries (the rest of rows x run is padding)


def pack_wave(entries: list[tuple[int, int, np.ndarray]], scratch: int, row_bucket: int = ROW_BUCKET,
              span_bucket: int = SPAN_BUCKET) -> PackedWave:
    """Pack (cache row, position, token block) entries into one wave (continuous.py:316-331).

    Rows are padded to a multiple of ``row_bucket`` with zero tokens at position 0 of the
    scratch row; a block shorter than the wave's run repeats its last token; the span is the
    furthest position written, rounded up to ``span_bucket``. One gather over the
    concatenated blocks replaces the reference's per-entry copy loop.
    """

    return pack_columns([row for row, _, _ in entries], [position for _, position, _ in entries],
                        [block for _, _, block in entries], scratch, row_bucket, span_bucket)


def pack_columns(cache_rows: list[int], positions: list[int], blocks: list[np.ndarray], scratch: int,
                 row_bucket: int = ROW_BUCKET, span_bucket: int = SPAN_BUCKET) -> PackedWave:
    """``pack_wave`` over the entries' three columns, as the collector gathers them."""

    count = len(blocks)
    lengths = np.fromiter(map(len, blocks), dtype=np.int64, count=count)
    if count == 0 or lengths.min() < 1:
        raise ValueError("every entry needs at least one token")
    run = int(lengths.max())
    rows = round_up(count, row_bucket)
    width = blocks[0].shape[1]
    flat = np.concatenate(blocks, axis=0)
    tokens = np.zeros((rows, run, width), dtype=np.int64)
    if run == 1:
        tokens[:count, 0] = flat
    else:
        starts = np.cumsum(lengths) - lengths
        tokens[:count] = flat[starts[:, None] + np.minimum(np.arange(run)[None, :], lengths[:, None] - 1)]
    packed_rows = np.full(rows, scratch, dtype=np.int64)
    packed_rows[:count] = cache_rows
    packed_positions = np.zeros(rows, dtype=np.int64)
    packed_positions[:count] = positions
    offsets = np.zeros(rows, dtype=np.int64)
    offsets[:count] = lengths - 1
    span = round_up(int(packed_positions.max()) + run, span_bucket)
    return PackedWave(tokens, packed_positions, offsets, packed_rows, span, count, int(lengths.sum()))


@dataclass
class _Readout:
    """One head group's sampled decisions on their way to the host."""

    states: list[LiveGame]
    probs: torch.Tensor  # pinned fp32 [n, head width]
    actions: torch.Tensor  # pinned int64 [n]
    values: torch.Tensor | None  # pinned fp32 [n, seats]


@dataclass
class _Wave:
    readouts: list[_Readout] = field(default_factory=list)
    fence: torch.cuda.Event | None = None


def _pinned(array: np.ndarray, device: torch.device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(array)).pin_memory().to(device, non_blocking=True)


class DeviceWaves:
    """A wave's device half: graph replay, readout gather, masked sampling, readout copy-back.

    ``launch`` enqueues everything on the current stream and returns at once; ``receive``
    waits on the wave's event and hands every state its sampled decision.
    """

    def __init__(self, model, cache, *, values: bool) -> None:
        from .graphs import DecodeGraphs

        self.graphs = DecodeGraphs(model, cache, values=values)
        self.values = values
        self.device = cache.device

    def launch(self, wave: PackedWave, readouts: list[tuple[int, LiveGame, float]]) -> _Wave:
        from .sampling import masked_sample

        output = self.graphs.run(wave.tokens, wave.positions, wave.offsets, wave.cache_rows, wave.span)
        columns = self.graphs.columns
        groups: dict[str, list[tuple[int, LiveGame, float]]] = {}
        for entry in readouts:
            groups.setdefault(entry[1].pending.head, []).append(entry)
        result = _Wave()
        for head, group in groups.items():
            head_columns = columns[head]
            width = head_columns.stop - head_columns.start
            masks = [state.pending.legal for _, state, _ in group]
            sizes = set(map(len, masks))
            if max(sizes) > width:
                raise ValueError(f"head {head!r} has {width} actions, a decision offers {max(sizes)}")
            if sizes == {width}:
                legal = np.stack(masks).astype(np.uint8, copy=False)
            else:
                legal = np.zeros((len(group), width), dtype=np.uint8)
                for row, mask in enumerate(masks):
                    legal[row, : mask.shape[0]] = mask
            index = _pinned(np.fromiter((entry for entry, _, _ in group), dtype=np.int64, count=len(group)),
                            self.device)
            uniforms = _pinned(np.fromiter((u for _, _, u in group), dtype=np.float64, count=len(group)),
                               self.device)
            selected = output.index_select(0, index)
            probs, actions = masked_sample(selected[:, head_columns], _pinned(legal, self.device), uniforms)
            values = selected[:, columns["values"]].to("cpu", non_blocking=True) if self.values else None
            result.readouts.append(_Readout([state for _, state, _ in group], probs.to("cpu", non_blocking=True),
                                            actions.to("cpu", non_blocking=True), values))
        result.fence = torch.cuda.Event()
        result.fence.record()
        return result

    @staticmethod
    def wait(wave: _Wave) -> None:
        if wave.fence is not None:
            wave.fence.synchronize()


def stack_features(features: list[dict[str, np.ndarray]]) -> dict[str, np.ndarray]:
    """Per-decision candidate features padded with zeros along the candidate axis and stacked
    (selfplay.py:570-587, ``_stack_features`` without the shape bucket)."""

    count = max(next(iter(entry.values())).shape[0] for entry in features)
    stacked = {}
    for key, first in features[0].items():
        array = np.zeros((len(features), count, *first.shape[1:]), dtype=first.dtype)
        for row, entry in enumerate(features):
            value = entry[key]
            array[row, : value.shape[0]] = value
        stacked[key] = array
    return stacked


def launch_decisions(model, hidden: torch.Tensor, context: torch.Tensor | None, states: list[LiveGame],
                     uniforms: list[float], *, values: bool) -> _Wave:
    """Score and sample every state's pending decision on the device (selfplay.py:486-567).

    ``hidden`` [N, d] (and ``context`` [N, ...] or None) are the states' readouts in order.
    Per head group: the candidate features stacked and uploaded (heads that take them), the
    head's logits, legal-masked softmax and inverse-CDF sampling with the states' uniforms, and
    the probabilities, actions and (with ``values``) player values copied to pinned host memory.
    """

    from .sampling import masked_sample

    device = hidden.device
    groups: dict[str, list[int]] = {}
    for position, state in enumerate(states):
        groups.setdefault(state.pending.head, []).append(position)
    result = _Wave()
    for head, positions in groups.items():
        index = _pinned(np.asarray(positions, dtype=np.int64), device)
        head_hidden = hidden.index_select(0, index)
        head_context = None if context is None else context.index_select(0, index)
        decisions = [states[p].pending for p in positions]
        features = None
        if decisions[0].features is not None:
            features = {k: _pinned(v, device) for k, v in stack_features([d.features for d in decisions]).items()}
        logits = model.policy_logits(head_hidden, head, features, None, head_context).float()
        width = logits.shape[1]
        if max(d.legal.shape[0] for d in decisions) > width:
            raise ValueError(f"head {head!r} scored {width} actions, a decision offers more")
        legal = np.zeros((len(positions), width), dtype=np.uint8)
        for row, decision in enumerate(decisions):
            legal[row, : decision.legal.shape[0]] = decision.legal
        draws = _pinned(np.asarray([uniforms[p] for p in positions], dtype=np.float64), device)
        probs, actions = masked_sample(logits, _pinned(legal, device), draws)
        head_values = model.player_values(head_hidden).float().to("cpu", non_blocking=True) if values else None
        result.readouts.append(_Readout([states[p] for p in positions], probs.to("cpu", non_blocking=True),
                                        actions.to("cpu", non_blocking=True), head_values))
    result.fence = torch.cuda.Event()
    result.fence.record()
    return result


def record_decisions(wave: _Wave, version: int) -> int:
    """Hand each state its sampled decision as a ``DecisionRecord`` (selfplay.py:549-566), once
    the wave's fence has passed; returns the count."""

    count = 0
    for readout in wave.readouts:
        probs = readout.probs.numpy()
        actions = readout.actions.numpy()
        values = None if readout.values is None else readout.values.numpy()
        for row, state in enumerate(readout.states):
            decision = state.pending
            width = decision.legal.shape[0]
            state.decisions.append(DecisionRecord(
                seat=decision.seat, head=decision.head,
                position=state.offsets[decision.seat] + state.lengths[decision.seat] - 1,
                action=int(actions[row]), probs=probs[row, :width].astype(np.float32),
                features=decision.features, version=version,
                value=None if values is None else values[row].copy()))
            state.pending = None
            count += 1
    return count


class EagerWaves(DeviceWaves):
    """The device half for models whose heads take per-decision candidate features (rummy): the
    wave's launches are issued eagerly (continuous.py:333-353), each head group's features are
    stacked and uploaded, and the head's logits go straight into masked sampling on the device.
    """

    def __init__(self, model, cache, *, values: bool) -> None:
        self.model = model
        self.cache = cache
        self.values = values
        self.device = cache.device

    def launch(self, wave: PackedWave, readouts: list[tuple[int, LiveGame, float]]) -> _Wave:
        model = self.model
        tokens, positions, offsets, cache_rows = (
            _pinned(a, self.device) for a in (wave.tokens, wave.positions, wave.offsets, wave.cache_rows))
        hidden = model.forward_ragged(tokens, positions, self.cache, offsets, span=min(wave.span, self.cache.max_len),
                                      rows=cache_rows)
        pop = getattr(model, "pop_context", None)
        context = pop() if pop is not None else None
        entries = np.fromiter((entry for entry, _, _ in readouts), dtype=np.int64, count=len(readouts))
        index = _pinned(entries, self.device)
        if context is not None:
            context = context[index, _pinned(wave.offsets[entries], self.device)]
        return launch_decisions(model, hidden.index_select(0, index), context, [state for _, state, _ in readouts],
                                [u for _, _, u in readouts], values=self.values)


class ContinuousCollector:
    """Keeps every lane's ``in_flight`` games running; ``collect`` returns each lane's quota
    of finished games (continuous.py:115-408). Games still running carry over, with their
    cache rows, into the next call. ``policy_lag`` in the stats reports how many versions old
    the returned decisions are."""

    ROW_BUCKET = ROW_BUCKET
    SPAN_BUCKET = SPAN_BUCKET

    def __init__(self, model, *, device: torch.device | str = "cuda", precision: str | None = None,
                 kv_dtype: str | torch.dtype = "fp16", max_length: int, cohorts: int = 1,
                 record_values: bool = False, waves_factory=None) -> None:
        if precision is not None and precision != getattr(model, "precision", precision):
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.device = torch.device(device)
        self.record_values = record_values
        dtypes = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}
        self.kv_dtype = dtypes[kv_dtype] if isinstance(kv_dtype, str) else kv_dtype
        self.cohorts = max(1, cohorts)
        # One spare position past the longest stream absorbs ragged padding.
        self.cache_length = max_length + 1
        self.stats = CollectionStats()
        # Graph-captured waves for models whose heads read only the readout (plump, piquet), as
        # the reference's graphs_enabled decides (graphs.py:49-56); eager waves otherwise.
        kind = DeviceWaves if getattr(model, "graphable_heads", False) else EagerWaves
        self._waves_factory = waves_factory or (lambda cache: kind(model, cache, values=record_values))
        self.reset()

    def reset(self) -> None:
        """Drop every game in flight, every banked result and the cache."""

        self._layout: tuple | None = None
        self._slots: list[_Slot] = []
        self._finished: dict[str, deque[Trajectory]] = {}
        self._cache = None
        self._device_waves = None
        self._scratch = 0
        self._waves = [_Wave() for _ in range(self.cohorts)]
        self._width: int | None = None

    def release(self) -> None:
        """Nothing to free between updates: the pool holds the games in flight."""

    @property
    def in_flight(self) -> int:
        return sum(slot.state is not None for slot in self._slots)

    @torch.no_grad()
    def collect(self, lanes: list[Lane], rng: random.Random, *, version: int = 0) -> list[Trajectory]:
        started = time.perf_counter()
        self.stats = CollectionStats()
        self._configure(lanes)
        # Every wave allocates a few objects per decision (records, entries, blocks) and almost
        # none form cycles; at the default young-generation threshold the cyclic collector runs
        # every few hundred decisions and rescans the games in flight, about a third of the
        # collector's host time. It runs less often for the collection's duration.
        thresholds = gc.get_threshold()
        gc.set_threshold(max(thresholds[0], 100_000), *thresholds[1:])
        try:
            for slot in self._slots:
                if slot.state is None:
                    self._deal(slot, lanes, rng)
            pending = [False] * self.cohorts
            while True:
                for cohort in range(self.cohorts):
                    if pending[cohort]:
                        self._receive(cohort)
                        self._act(cohort, lanes, rng, version)
                        pending[cohort] = False
                    if not self._satisfied(lanes) and self.in_flight:
                        pending[cohort] = self._launch(cohort)
                if not any(pending):
                    break
        finally:
            gc.set_threshold(*thresholds)
        results: list[Trajectory] = []
        for lane in lanes:
            bank = self._finished[lane.name]
            count = len(bank) if lane.quota is None else min(lane.quota, len(bank))
            results.extend(bank.popleft() for _ in range(count))
        versions = [record.version for trajectory in results for record in trajectory.decisions]
        self.stats.games = len(results)
        self.stats.in_flight = self.in_flight
        self.stats.policy_lag = float(version - np.mean(versions)) if versions else 0.0
        self.stats.collect_sec = time.perf_counter() - started
        return results

    # ------------------------------------------------------------------

    def _configure(self, lanes: list[Lane]) -> None:
        layout = tuple((lane.name, lane.players, lane.in_flight) for lane in lanes)
        if layout == self._layout:
            return
        self.reset()
        self._layout = layout
        row = 0
        for index, lane in enumerate(lanes):
            self._finished[lane.name] = deque()
            for _ in range(lane.in_flight):
                self._slots.append(_Slot(lane=index, base=row, cohort=len(self._slots) % self.cohorts))
                row += lane.players
        self._scratch = row
        self._cache = self.model.new_cache(row + 1, self.cache_length, self.kv_dtype)
        self._device_waves = self._waves_factory(self._cache)

    def _satisfied(self, lanes: list[Lane]) -> bool:
        for index, lane in enumerate(lanes):
            if lane.quota is None:
                if any(slot.state is not None for slot in self._slots if slot.lane == index):
                    return False
            elif len(self._finished[lane.name]) < lane.quota:
                return False
        return True

    def _deal(self, slot: _Slot, lanes: list[Lane], rng: random.Random) -> None:
        """Fill an empty slot; games that end before any decision finish at once. A lane
        whose finished games already cover its quota deals nothing (continuous.py:224-255)."""

        lane = lanes[slot.lane]
        if lane.quota is not None and len(self._finished[lane.name]) >= lane.quota:
            return
        while True:
            game = lane.deal(rng)
            if game is None:
                return
            state = LiveGame(game=game, base=slot.base, lengths=[0] * game.num_players,
                             blocks=[[] for _ in range(game.num_players)])
            queued = self._record(state, game.prefix_tokens())
            if game.done():
                self._finished[lane.name].append(self._finish(state))
                continue
            slot.state = state
            slot.queued = queued
            self._expect_readout(state, queued)
            return

    def _record(self, state: LiveGame, blocks: list[np.ndarray], restart: bool = False) -> list[tuple[int, np.ndarray]]:
        """Record every observer's new tokens; returns those to decode (after any restart)."""

        queued = []
        for seat, block in enumerate(blocks):
            if len(block):
                state.blocks[seat].append(block)
                queued.append((seat, block))
        if queued:
            self._width = queued[-1][1].shape[1]
        if restart:
            decoded = restart_contexts(state, blocks)
            if decoded is not blocks:
                return [(seat, block) for seat, block in enumerate(decoded) if len(block)]
        return queued

    @staticmethod
    def _expect_readout(state: LiveGame, queued: list[tuple[int, np.ndarray]]) -> None:
        state.pending = state.game.decision()
        seat = state.pending.seat
        blocks = [block for queued_seat, block in queued if queued_seat == seat]
        if not blocks:
            raise AssertionError("The next actor's stream received no readout token.")
        state.readout = blocks[-1][-1]

    def _finish(self, state: LiveGame) -> Trajectory:
        width = self._width or 0
        streams = [np.concatenate(blocks, axis=0) if blocks else np.zeros((0, width), dtype=np.int16)
                   for blocks in state.blocks]
        return Trajectory(game=state.game, streams=streams, decisions=state.decisions,
                          returns=np.asarray(state.game.returns(), dtype=np.float64))

    def _launch(self, cohort: int) -> bool:
        """Decode the cohort's queued blocks and sample its pending decisions on the device
        (continuous.py:299-353). Returns whether anything was launched."""

        started = time.perf_counter()
        cache_rows: list[int] = []  # the entries, as three columns: cache row, position, block
        positions: list[int] = []
        blocks: list[np.ndarray] = []
        readouts: list[tuple[int, LiveGame, float]] = []  # (entry, state, uniform)
        limit = self.cache_length
        for slot in self._slots:
            state = slot.state
            if state is None or slot.cohort != cohort:
                continue
            actor = state.pending.seat
            lengths = state.lengths
            for seat, block in slot.queued:
                if seat == actor:
                    readouts.append((len(blocks), state, state.game.rng.random()))
                length = lengths[seat]
                cache_rows.append(slot.base + seat)
                positions.append(length)
                blocks.append(block)
                length += len(block)
                lengths[seat] = length
                if length >= limit:
                    raise RuntimeError("A stream outgrew the model's maximum sequence length.")
            slot.queued = []
        if not blocks:
            return False
        wave = pack_columns(cache_rows, positions, blocks, self._scratch, self.ROW_BUCKET, self.SPAN_BUCKET)
        self._waves[cohort] = self._device_waves.launch(wave, readouts)
        rows, run = wave.tokens.shape[:2]
        self.stats.waves += 1
        self.stats.forward_rows += rows * run
        self.stats.padded_rows += rows * run - wave.real_tokens
        self.stats.peak_rows = max(self.stats.peak_rows, wave.count)
        self.stats.forward_sec += time.perf_counter() - started
        return True

    def _receive(self, cohort: int) -> None:
        started = time.perf_counter()
        self._device_waves.wait(self._waves[cohort])
        self.stats.wait_sec += time.perf_counter() - started

    def _act(self, cohort: int, lanes: list[Lane], rng: random.Random, version: int) -> None:
        """Record the cohort's sampled decisions and step their games; retire and replace
        finished games (continuous.py:383-408, selfplay.py:532-567)."""

        t0 = time.perf_counter()
        wave = self._waves[cohort]
        self._waves[cohort] = _Wave()
        self.stats.decisions += record_decisions(wave, version)
        t1 = time.perf_counter()
        for slot in self._slots:
            state = slot.state
            if state is None or slot.cohort != cohort:
                continue
            queued = self._record(state, state.game.step(state.decisions[-1].action), restart=True)
            if state.game.done():
                self._finished[lanes[slot.lane].name].append(self._finish(state))
                slot.state = None
                self._deal(slot, lanes, rng)
            else:
                slot.queued = queued
                self._expect_readout(state, queued)
        self.stats.sample_sec += t1 - t0
        self.stats.step_sec += time.perf_counter() - t1


@dataclass
class _Slot:
    lane: int
    base: int  # first cache row
    cohort: int = 0
    state: LiveGame | None = None
    queued: list[tuple[int, np.ndarray]] = field(default_factory=list)  # (seat, block) not yet decoded
