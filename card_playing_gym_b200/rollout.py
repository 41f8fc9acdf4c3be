"""The rollout engine shared by both self-play collectors: a KV pool of per-game rows, the
bookkeeping of what each row holds, wave assembly, and the device half that decodes a wave and
samples its decisions.

The collectors keep the reference's protocol and data formats (cardgym/rl/selfplay.py:48-150:
``SelfPlayGame`` with ``prefix_tokens``, ``decision``, ``step``, ``done``, ``returns``,
``context_starts`` and a per-game ``rng``; ``Decision``, ``DecisionRecord``, ``Trajectory``,
``CollectionStats``) and its scheduling rules, but run them on one engine built for these
kernels:

* Every wave decodes gathered rows. The trunk kernels take a row index per wave entry at no
  cost (the attention reads each row's keys where they are; the dense layers work on the
  wave's row-tokens), so a game keeps its rows for its whole life and nothing is ever
  compacted: a finished game's rows simply stop appearing in waves. The reference's batch
  collector instead slides survivors down (cardgym/rl/selfplay.py:351-372) so that its
  attention can read a dense prefix of the pool.
* What a row holds is two integer arrays over the pool, ``cached`` (its KV context length)
  and ``shift`` (stream tokens before that context, advanced by context restarts), updated
  for a whole wave at once; positions, limits and record positions come from them by
  indexing.
* A wave's device half is one CUDA graph replay (graphs.DecodeGraphs) or, for heads that
  take per-decision candidate features, eager launches; either way the readouts are
  gathered, masked and sampled on the device and only probabilities, actions and values
  return to pinned host memory, behind one event.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

ROW_BUCKET = 64  # wave entries are padded to a multiple of this (the reference's bucket)
SPAN_BUCKET = 32  # attention spans are rounded up to a multiple of this


def round_up(value: int, multiple: int) -> int:
    return -(-value // multiple) * multiple


# -- the reference's data formats (cardgym/rl/selfplay.py:48-150) ------------------------------------------
@dataclass
class Decision:
    """What the acting seat must choose now."""

    seat: int
    head: str
    legal: np.ndarray  # bool [actions]; actions index the head's output
    features: dict[str, np.ndarray] | None = None  # candidate features of pointer heads


@dataclass
class DecisionRecord:
    """One sampled decision."""

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
    games: int = 0
    decisions: int = 0
    waves: int = 0
    forward_rows: int = 0
    padded_rows: int = 0
    peak_rows: int = 0
    compactions: int = 0  # always 0 here: rows stay where their game was dealt
    collect_sec: float = 0.0
    forward_sec: float = 0.0  # host time preparing and launching device work
    wait_sec: float = 0.0  # host time blocked on the device
    sample_sec: float = 0.0  # host time turning sampled decisions into records
    step_sec: float = 0.0  # host time in the games' rules
    in_flight: int = 0
    policy_lag: float = 0.0


# -- wave packing ---------------------------------------------------------------------------------------------
@dataclass
class PackedWave:
    tokens: np.ndarray  # int64 [rows, run, width]
    positions: np.ndarray  # int64 [rows]
    offsets: np.ndarray  # int64 [rows], each entry's last real token
    cache_rows: np.ndarray  # int64 [rows]
    span: int
    count: int  # real entries; the rest write the scratch row
    real_tokens: int = 0  # tokens of the real entries (the rest of rows x run is padding)


def pack_columns(cache_rows, positions, blocks: list[np.ndarray], scratch: int, row_bucket: int = ROW_BUCKET,
                 span_bucket: int = SPAN_BUCKET) -> PackedWave:
    """Lay out one wave from its entries' three columns (cache row, write position, token block).

    Entries are padded to a multiple of ``row_bucket`` with zero tokens written at position 0 of
    the ``scratch`` row; a block shorter than the wave's run repeats its last token (its outputs
    are never read); the span is the furthest position written, rounded up to ``span_bucket``.
    One gather over the concatenated blocks fills the token array (the reference copies entry
    by entry, cardgym/rl/continuous.py:316-331).
    """

    count = len(blocks)
    lengths = np.fromiter(map(len, blocks), dtype=np.int64, count=count)
    if count == 0 or lengths.min() < 1:
        raise ValueError("every wave entry needs at least one token")
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


def pack_wave(entries: list[tuple[int, int, np.ndarray]], scratch: int, row_bucket: int = ROW_BUCKET,
              span_bucket: int = SPAN_BUCKET) -> PackedWave:
    """``pack_columns`` over (cache row, position, block) entries."""

    return pack_columns([e[0] for e in entries], [e[1] for e in entries], [e[2] for e in entries], scratch,
                        row_bucket, span_bucket)


def stack_features(features: list[dict[str, np.ndarray]]) -> dict[str, np.ndarray]:
    """Per-decision candidate features stacked, zero-padded along the candidate axis to the longest list
    (the padding of cardgym/rl/selfplay.py:570-587 without its shape bucket)."""

    longest = max(next(iter(entry.values())).shape[0] for entry in features)
    stacked = {}
    for key, first in features[0].items():
        out = np.zeros((len(features), longest, *first.shape[1:]), dtype=first.dtype)
        for index, entry in enumerate(features):
            value = entry[key]
            out[index, : value.shape[0]] = value
        stacked[key] = out
    return stacked


def upload(array: np.ndarray, device: torch.device) -> torch.Tensor:
    """A host array on the device through pinned memory, without blocking the host."""

    return torch.from_numpy(np.ascontiguousarray(array)).pin_memory().to(device, non_blocking=True)


# -- games in flight and the rows they own -----------------------------------------------------------------------
class GameTrace:
    """One game in flight: its rows, what it has produced, and what its next wave must decode."""

    __slots__ = ("game", "base", "blocks", "records", "pending", "queue", "token_width")

    def __init__(self, game, base: int) -> None:
        self.game = game
        self.base = base  # first cache row; seat s owns row base + s
        self.blocks: list[list[np.ndarray]] = [[] for _ in range(game.num_players)]
        self.records: list[DecisionRecord] = []
        self.pending: Decision | None = None
        self.queue: list[tuple[int, np.ndarray]] = []  # (seat, block) not yet decoded
        self.token_width = 0

    def observe(self, blocks: list[np.ndarray]) -> None:
        """Keep every non-empty block for the trajectory."""

        for seat, block in enumerate(blocks):
            if len(block):
                self.blocks[seat].append(block)
                self.token_width = block.shape[1]

    def trajectory(self) -> Trajectory:
        streams = [np.concatenate(seat, axis=0) if seat else np.zeros((0, self.token_width), dtype=np.int16)
                   for seat in self.blocks]
        return Trajectory(game=self.game, streams=streams, decisions=self.records,
                          returns=np.asarray(self.game.returns(), dtype=np.float64))


class RowTable:
    """What every row of the KV pool holds: ``cached`` tokens of the current context, after ``shift``
    tokens of the stream that came before it (a context restart moves the boundary,
    cardgym/rl/selfplay.py:172-190)."""

    def __init__(self, rows: int) -> None:
        self.cached = np.zeros(rows, dtype=np.int64)
        self.shift = np.zeros(rows, dtype=np.int64)

    def clear(self, base: int, count: int) -> None:
        self.cached[base:base + count] = 0
        self.shift[base:base + count] = 0

    def restart(self, row: int, start: int) -> None:
        """The stream's context begins again at ``start`` tokens into the block just returned: the row's
        KV is rewritten from position 0 and causal attention never reaches the stale keys beyond."""

        self.shift[row] += self.cached[row] + start
        self.cached[row] = 0


def queue_after_step(trace: GameTrace, table: RowTable, blocks: list[np.ndarray]) -> None:
    """Queue a step's blocks for decoding, after any context restart the game asks for."""

    starts = trace.game.context_starts()
    queue = []
    for seat, block in enumerate(blocks):
        start = None if starts is None else starts[seat]
        if start is not None:
            table.restart(trace.base + seat, start)
            block = block[start:]
        if len(block):
            queue.append((seat, block))
    trace.queue = queue


def expect_decision(trace: GameTrace) -> None:
    """Ask the game for its next decision; the acting seat must have a token to read out."""

    trace.pending = trace.game.decision()
    if not any(seat == trace.pending.seat for seat, _ in trace.queue):
        raise AssertionError(f"seat {trace.pending.seat} must act but no new token of its stream is queued")


# -- the device half of a wave ------------------------------------------------------------------------------------
@dataclass
class SampledGroup:
    """One head's sampled decisions of a wave, on their way to pinned host memory."""

    traces: list[GameTrace]
    probs: torch.Tensor  # fp32 [n, width]
    actions: torch.Tensor  # int64 [n]
    values: torch.Tensor | None  # fp32 [n, seats]


@dataclass
class WaveInFlight:
    groups: list[SampledGroup] = field(default_factory=list)
    fence: torch.cuda.Event | None = None

    def wait(self) -> None:
        if self.fence is not None:
            self.fence.synchronize()


def _by_head(readouts: list[tuple[int, GameTrace, float]]) -> list[tuple[str, list[tuple[int, GameTrace, float]]]]:
    groups: dict[str, list] = {}
    for readout in readouts:
        groups.setdefault(readout[1].pending.head, []).append(readout)
    return list(groups.items())


def _legal_matrix(traces: list[GameTrace], width: int) -> np.ndarray:
    masks = [trace.pending.legal for trace in traces]
    if all(mask.shape[0] == width for mask in masks):
        return np.stack(masks).astype(np.uint8, copy=False)
    legal = np.zeros((len(masks), width), dtype=np.uint8)
    for row, mask in enumerate(masks):
        legal[row, : mask.shape[0]] = mask
    return legal


def _sample_group(logits: torch.Tensor, group, device, values: torch.Tensor | None) -> SampledGroup:
    """Masked softmax and inverse-CDF draws of one head's decisions on the device.

    The reference samples a head's decisions as rows as wide as the group's longest legal vector
    (cardgym/rl/selfplay.py:532-545), and the kernel's sums follow numpy's order over that row
    length, so the logits are cut to it: the draws are then bit-identical to the reference's.
    """

    from .sampling import masked_sample

    traces = [trace for _, trace, _ in group]
    width = max(trace.pending.legal.shape[0] for trace in traces)
    if width > logits.shape[1]:
        raise ValueError(f"head {traces[0].pending.head!r} scores {logits.shape[1]} actions, a decision offers {width}")
    uniforms = upload(np.fromiter((u for _, _, u in group), dtype=np.float64, count=len(group)), device)
    probs, actions = masked_sample(logits[:, :width], upload(_legal_matrix(traces, width), device), uniforms)
    return SampledGroup(traces, probs.to("cpu", non_blocking=True), actions.to("cpu", non_blocking=True),
                        None if values is None else values.to("cpu", non_blocking=True))


class GraphedHalf:
    """Heads that read only the readout state (plump, piquet): each wave is one DecodeGraphs replay, then
    one gather of every readout row and one masked draw per head."""

    def __init__(self, model, cache, *, values: bool) -> None:
        from .graphs import DecodeGraphs

        self.graphs = DecodeGraphs(model, cache, values=values)
        self.values = values
        self.device = cache.device

    def launch(self, wave: PackedWave, readouts) -> WaveInFlight:
        output = self.graphs.run(wave.tokens, wave.positions, wave.offsets, wave.cache_rows, wave.span)
        groups = _by_head(readouts)
        order = np.fromiter((entry for _, group in groups for entry, _, _ in group), dtype=np.int64,
                            count=len(readouts))
        selected = output.index_select(0, upload(order, self.device))
        columns = self.graphs.columns
        result = WaveInFlight()
        at = 0
        for head, group in groups:
            part = selected[at:at + len(group)]
            at += len(group)
            values = part[:, columns["values"]] if self.values else None
            result.groups.append(_sample_group(part[:, columns[head]], group, self.device, values))
        result.fence = torch.cuda.Event()
        result.fence.record()
        return result


class EagerHalf:
    """Heads that take per-decision candidate features (rummy): the wave's launches are issued directly, each
    head group's features stacked and uploaded, its logits sampled on the device as they come."""

    def __init__(self, model, cache, *, values: bool) -> None:
        self.model = model
        self.cache = cache
        self.values = values
        self.device = cache.device

    def launch(self, wave: PackedWave, readouts) -> WaveInFlight:
        model, device = self.model, self.device
        hidden = model.forward_ragged(upload(wave.tokens, device), upload(wave.positions, device), self.cache,
                                      upload(wave.offsets, device), span=min(wave.span, self.cache.max_len),
                                      rows=upload(wave.cache_rows, device))
        pop = getattr(model, "pop_context", None)
        context = pop() if pop is not None else None
        result = WaveInFlight()
        for head, group in _by_head(readouts):
            entries = np.fromiter((entry for entry, _, _ in group), dtype=np.int64, count=len(group))
            index = upload(entries, device)
            head_hidden = hidden.index_select(0, index)
            head_context = None if context is None else context[index, upload(wave.offsets[entries], device)]
            decisions = [trace.pending for _, trace, _ in group]
            features = None
            if decisions[0].features is not None:
                stacked = stack_features([decision.features for decision in decisions])
                features = {key: upload(value, device) for key, value in stacked.items()}
            logits = model.policy_logits(head_hidden, head, features, None, head_context).float()
            values = model.player_values(head_hidden).float() if self.values else None
            result.groups.append(_sample_group(logits, group, device, values))
        result.fence = torch.cuda.Event()
        result.fence.record()
        return result


def default_half(model):
    """The reference's choice (cardgym/rl/graphs.py:49-56): graphs for models whose heads need no features."""

    kind = GraphedHalf if getattr(model, "graphable_heads", False) else EagerHalf
    return lambda cache, values: kind(model, cache, values=values)


# -- the engine -----------------------------------------------------------------------------------------------------
class RolloutEngine:
    """A KV pool of per-game rows, what each row holds, and the device half that decodes waves over them.

    ``reserve(rows)`` sizes the pool (plus one scratch row that padding entries write to);
    ``launch(traces)`` decodes every queued block of those games and samples their pending decisions;
    ``land(wave, version)`` waits for a launched wave and turns its draws into ``DecisionRecord`` s.
    """

    def __init__(self, model, *, device, kv_dtype: torch.dtype, max_length: int, record_values: bool,
                 half_factory=None) -> None:
        self.model = model
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        self.cache_length = max_length + 1  # one spare position past the longest stream takes padding
        self.record_values = record_values
        self.half_factory = half_factory or default_half(model)
        self.cache = None
        self.half = None
        self.table = RowTable(0)
        self.scratch = 0

    def reserve(self, rows: int) -> None:
        """A pool of at least ``rows`` game rows; a new pool (and device half) only when it must grow."""

        if self.cache is not None and self.scratch >= rows:
            return
        self.cache = None
        self.half = None
        self.cache = self.model.new_cache(rows + 1, self.cache_length, self.kv_dtype)
        self.half = self.half_factory(self.cache, self.record_values)
        self.table = RowTable(rows + 1)
        self.scratch = rows

    def launch(self, traces, stats: CollectionStats) -> WaveInFlight | None:
        """One wave over the queued blocks of ``traces``; None when none is queued.

        Each game's uniform is drawn from its own ``rng`` here, after its ``decision()`` and before its
        next ``step()``, where the reference's ``sample_decisions`` draws it (cardgym/rl/selfplay.py:547).
        """

        rows: list[int] = []
        blocks: list[np.ndarray] = []
        readouts: list[tuple[int, GameTrace, float]] = []
        for trace in traces:
            actor = trace.pending.seat
            for seat, block in trace.queue:
                if seat == actor:
                    readouts.append((len(rows), trace, trace.game.rng.random()))
                rows.append(trace.base + seat)
                blocks.append(block)
            trace.queue = []
        if not rows:
            return None
        row_index = np.asarray(rows, dtype=np.int64)
        positions = self.table.cached[row_index]
        grown = positions + np.fromiter(map(len, blocks), dtype=np.int64, count=len(blocks))
        if int(grown.max()) >= self.cache_length:
            raise RuntimeError("A stream outgrew the model's maximum sequence length.")
        self.table.cached[row_index] = grown
        wave = pack_columns(row_index, positions, blocks, self.scratch)
        in_flight = self.half.launch(wave, readouts)
        entries, run = wave.tokens.shape[:2]
        stats.waves += 1
        stats.forward_rows += entries * run
        stats.padded_rows += entries * run - wave.real_tokens
        stats.peak_rows = max(stats.peak_rows, wave.count)
        return in_flight

    def land(self, wave: WaveInFlight, version: int) -> int:
        """Wait for ``wave`` and append one ``DecisionRecord`` per sampled decision; returns the count."""

        wave.wait()
        count = 0
        cached, shift = self.table.cached, self.table.shift
        for group in wave.groups:
            probs = group.probs.numpy()
            actions = group.actions.numpy().tolist()
            values = None if group.values is None else group.values.numpy()
            rows = np.fromiter((t.base + t.pending.seat for t in group.traces), dtype=np.int64,
                               count=len(group.traces))
            positions = (shift[rows] + cached[rows] - 1).tolist()
            for index, trace in enumerate(group.traces):
                decision = trace.pending
                trace.records.append(DecisionRecord(
                    seat=decision.seat, head=decision.head, position=positions[index], action=actions[index],
                    probs=probs[index, : decision.legal.shape[0]].copy(), features=decision.features,
                    version=version, value=None if values is None else values[index].copy()))
                trace.pending = None
            count += len(group.traces)
        return count

    def start(self, trace: GameTrace, blocks: list[np.ndarray]) -> None:
        """A newly dealt game's prefix: its rows start empty and the prefix is queued for decoding."""

        self.table.clear(trace.base, trace.game.num_players)
        trace.observe(blocks)
        trace.queue = [(seat, block) for seat, block in enumerate(blocks) if len(block)]
