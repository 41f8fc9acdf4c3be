"""The continuous self-play collector (cardgym/rl/continuous.py:55-408).

CPU: ``pack_wave`` against the oracle's entry-by-entry restatement of the reference's packing;
``split_lanes`` and ``restart_contexts``; the collector's host logic with a stand-in device
half (uniform probabilities, the oracle's inverse CDF): quotas, slot refills, games that end
before any decision, context restarts, cohorts, that every KV row is appended in order with no
gaps and no two entries of a wave share a row, and that each game's decisions consume its own
``rng`` in the reference's order. GPU: the real device half (``DecodeGraphs`` replay, readout
gather, masked sampling on the device) on a small plump actor, each recorded decision's
probabilities against an eager prefill of the same context and the oracle's softmax.
"""

from __future__ import annotations

import random
from dataclasses import replace

import numpy as np
import pytest
import torch

from card_playing_gym_b200 import continuous as cont
from card_playing_gym_b200 import rollout
from oracle import continuous as ocont
from oracle import ppo as oppo
from tests.conftest import load_golden

BID, PLAY = 11, 52


class ScriptedGame:
    """A 4-seat game over real plump tokens, its course set by ``seed``.

    Every observer sees one or two new tokens per step, so the next actor always receives its
    readout token; the first four decisions use the bid head, the rest the play head. With
    ``restart`` the game asks for a fresh context at that step for seats 0 and 2. The game logs,
    per decision, the acting seat, where its current context starts in its stream and the
    stream's length, which is what an eager recomputation needs.
    """

    players = 4

    def __init__(self, seed: int, pool: np.ndarray, *, restart: int | None = None, max_steps: int = 7):
        self.seed = seed
        self.rng = random.Random(seed ^ 0x5EED)
        self._script = random.Random(seed)
        self.num_players = self.players
        self.pool = pool
        self.steps_left = self._script.randint(0, max_steps)
        self.turn = 0
        self.restart = restart
        self.streams = [[] for _ in range(self.players)]
        self.context_base = [0] * self.players
        self._starts = None
        self.log = []  # (seat, head, legal, context base, stream length)
        self.actions = []
        self._prefix = self._blocks(1, 3)  # dealt with the game: decision() may come first

    def head(self) -> tuple[str, int]:
        return ("bid", BID) if self.turn < 4 else ("play", PLAY)

    def _blocks(self, low: int, high: int):
        blocks = []
        for seat in range(self.players):
            count = self._script.randint(low, high)
            rows = [self._script.randrange(len(self.pool)) for _ in range(count)]
            block = self.pool[rows].astype(np.int16)
            self.streams[seat].extend(block)
            blocks.append(block)
        return blocks

    def prefix_tokens(self):
        return self._prefix

    def decision(self):
        seat = self.turn % self.players
        head, width = self.head()
        legal = np.array([self._script.random() < 0.5 for _ in range(width)])
        legal[self._script.randrange(width)] = True
        self.log.append((seat, head, legal, self.context_base[seat], len(self.streams[seat])))
        return cont.Decision(seat=seat, head=head, legal=legal)

    def step(self, action: int):
        seat, head, legal, _, _ = self.log[-1]
        assert legal[action], "an illegal action was sampled"
        self.actions.append(action)
        self.turn += 1
        self.steps_left -= 1
        before = [len(stream) for stream in self.streams]
        blocks = self._blocks(1, 2)
        self._starts = None
        if self.restart is not None and self.turn == self.restart and not self.done():
            starts = [None] * self.players
            for restarted in range(0, self.players, 2):
                starts[restarted] = len(blocks[restarted]) - 1
                self.context_base[restarted] = before[restarted] + starts[restarted]
            self._starts = starts
        return blocks

    def done(self) -> bool:
        return self.steps_left <= 0

    def returns(self):
        score = np.array([self._script.uniform(-1, 1) for _ in range(self.players)])
        return score - score.mean()

    def context_starts(self):
        return self._starts


class ScriptedRummy(ScriptedGame):
    """Three seats, rummy tokens and rummy's candidate heads: each decision offers 1-9
    candidates with their features (kind, cards, target; taken counts for draws)."""

    players = 3

    def decision(self):
        seat = self.turn % self.players
        head = "draw" if self.turn % 2 == 0 else "play"
        count = self._script.randint(1, 9)
        features = {"kind": np.array([self._script.randrange(7) for _ in range(count)], dtype=np.int64),
                    "cards": np.full((count, 13), 52, dtype=np.int64), "target": np.full((count, 13), 52, dtype=np.int64)}
        for c in range(count):
            n = self._script.randint(0, 4)
            features["cards"][c, :n] = [self._script.randrange(52) for _ in range(n)]
        if head == "draw":
            features["taken"] = np.array([[self._script.randrange(3) if self._script.random() < 0.1 else 0
                                           for _ in range(52)] for _ in range(count)], dtype=np.int64)
        legal = np.array([self._script.random() < 0.6 for _ in range(count)])
        legal[self._script.randrange(count)] = True
        self.log.append((seat, head, legal, self.context_base[seat], len(self.streams[seat])))
        self.features.append(features)
        return cont.Decision(seat=seat, head=head, legal=legal, features=features)

    def __init__(self, *args, **kwargs):
        self.features = []
        super().__init__(*args, **kwargs)


class ScriptedPiquet(ScriptedGame):
    """The same script with two seats, piquet tokens and piquet's heads: exchange (32 cards +
    stop), declare (2), play (32 cards)."""

    players = 2

    def head(self) -> tuple[str, int]:
        return (("exchange", 33), ("declare", 2), ("play", 32))[min(self.turn // 2, 2)]


def _pool() -> np.ndarray:
    data = load_golden("plump_streams")
    rows = [data["tokens"][i, : data["lengths"][i]] for i in range(data["tokens"].shape[0])]
    return np.concatenate(rows, axis=0).astype(np.int64)


class _FakeCache:
    def __init__(self, rows: int, length: int):
        self.rows, self.length = rows, length


class _FakeModel:
    precision = "bf16"

    def new_cache(self, rows, length, dtype):
        return _FakeCache(rows, length)


class FakeHalf:
    """The device half's contract, on the host: uniform probabilities over the legal actions, the oracle's
    inverse CDF. Checks every wave's entries against the KV lengths it has seen."""

    def __init__(self, cache):
        self.cache = cache
        self.lengths = np.zeros(cache.rows, dtype=np.int64)
        self.waves = []

    def launch(self, wave, readouts):
        self.waves.append(wave)
        real = wave.cache_rows[: wave.count]
        assert len(set(real.tolist())) == wave.count, "two entries of one wave share a cache row"
        assert (wave.cache_rows[wave.count:] == self.cache.rows - 1).all()
        assert wave.tokens.shape[0] % cont.ROW_BUCKET == 0 and wave.span % cont.SPAN_BUCKET == 0
        for index in range(wave.count):
            row, position = int(wave.cache_rows[index]), int(wave.positions[index])
            assert position in (0, self.lengths[row]), (row, position, self.lengths[row])
            self.lengths[row] = position + int(wave.offsets[index]) + 1
            assert self.lengths[row] < self.cache.length
        result = cont.WaveInFlight()
        groups = {}
        for entry, trace, uniform in readouts:
            groups.setdefault(trace.pending.head, []).append((trace, uniform))
        for head, group in groups.items():
            width = max(trace.pending.legal.shape[0] for trace, _ in group)
            mask = np.zeros((len(group), width), dtype=bool)
            for row, (trace, _) in enumerate(group):
                mask[row, : trace.pending.legal.shape[0]] = trace.pending.legal
            probs = oppo.masked_probabilities(np.zeros(mask.shape, np.float32), mask)
            actions = oppo.sample_rows(probs, mask, np.array([u for _, u in group]))
            result.groups.append(rollout.SampledGroup([trace for trace, _ in group], torch.from_numpy(probs),
                                                      torch.from_numpy(actions.astype(np.int64)), None))
        return result


def test_pack_wave_matches_the_reference_packing():
    rng = np.random.default_rng(5)
    for count, max_run in ((1, 1), (63, 3), (64, 1), (65, 5), (200, 9)):
        entries = []
        for row in rng.permutation(1000)[:count]:
            length = int(rng.integers(1, max_run + 1))
            entries.append((int(row), int(rng.integers(0, 300)), rng.integers(0, 90, size=(length, 26))))
        got = cont.pack_wave(entries, scratch=1000)
        want = ocont.pack_wave(entries, scratch=1000)
        for a, b in zip((got.tokens, got.positions, got.offsets, got.cache_rows, got.span), want):
            assert np.array_equal(a, b)
        assert got.count == count
    with pytest.raises(ValueError):
        cont.pack_wave([(0, 0, np.zeros((0, 26), np.int64))], scratch=1)


def test_split_lanes_shares_quota_and_games():
    lanes = [cont.Lane("plump", 4, 10, 7, deal=None), cont.Lane("piquet", 2, 3, 2, deal=None)]
    shares = [cont.split_lanes(lanes, index, 3) for index in range(3)]
    for name, lane in (("plump", lanes[0]), ("piquet", lanes[1])):
        parts = [s for share in shares for s in share if s.name == name]
        assert sum(p.quota for p in parts) == lane.quota
        assert max(p.quota for p in parts) - min(p.quota for p in parts) <= 1
        assert all(p.in_flight >= 1 for p in parts)
    assert [s.name for s in shares[2]] == ["plump"]  # piquet's 2 games go to workers 0 and 1
    with pytest.raises(ValueError):
        cont.split_lanes([replace(lanes[0], quota=None)], 0, 2)


def test_context_restart_rewrites_the_row_from_position_zero():
    """selfplay.py:172-190: a restarted observer's row length drops to zero, the stream tokens before the new
    context move into its shift, and only the block's tail from the start index is decoded."""

    class Game:
        num_players = 2

        def context_starts(self):
            return [None, 1]

    table = rollout.RowTable(4)
    table.cached[2:4] = [5, 7]
    trace = rollout.GameTrace(Game(), base=2)
    blocks = [np.zeros((2, 3)), np.arange(9).reshape(3, 3)]
    rollout.queue_after_step(trace, table, blocks)
    assert trace.queue[0][1] is blocks[0] and np.array_equal(trace.queue[1][1], blocks[1][1:])
    assert table.cached[2:4].tolist() == [5, 0] and table.shift[2:4].tolist() == [0, 8]


@pytest.mark.parametrize("cohorts", (1, 2))
def test_collector_host_logic(cohorts):
    pool = _pool()
    dealt = []

    def deal(rng):
        seed = rng.randrange(1 << 30)
        game = ScriptedGame(seed, pool, restart=2 if seed % 3 == 0 else None)
        dealt.append(game)
        return game

    lanes = [cont.Lane("plump", 4, 37, 50, deal=deal)]
    fakes = []
    collector = cont.ContinuousCollector(
        _FakeModel(), device="cpu", max_length=64, cohorts=cohorts,
        half_factory=lambda cache, values: fakes.append(FakeHalf(cache)) or fakes[-1])
    rng = random.Random(1)
    first = collector.collect(lanes, rng, version=0)
    assert len(first) == 50 and collector.in_flight > 0
    second = collector.collect(lanes, rng, version=1)
    assert len(second) == 50 and len(fakes) == 1  # the pool and its rows carry over
    assert collector.stats.policy_lag >= 0.0
    fake = fakes[0]
    assert fake.cache.rows == 37 * 4 + 1
    for wave in fake.waves:
        want = ocont.pack_wave([(int(r), int(p), wave.tokens[i, : int(o) + 1])
                                for i, (r, p, o) in enumerate(zip(wave.cache_rows, wave.positions, wave.offsets))
                                if i < wave.count], scratch=37 * 4)
        assert np.array_equal(wave.tokens, want[0]) and np.array_equal(wave.cache_rows, want[3])
    assert any(game.steps_left <= 0 and not game.actions for game in dealt)  # some ended at the deal
    assert any(game.restart is not None and game.turn > game.restart for game in dealt)
    for trajectory in first + second:
        game = trajectory.game
        assert game.done()
        assert [record.action for record in trajectory.decisions] == game.actions
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            assert (record.seat, record.head) == (seat, head)
            assert record.position == length - 1
            probs = oppo.masked_probabilities(np.zeros(legal.shape, np.float32)[None], legal[None])
            want = oppo.sample_rows(probs, legal[None], np.array([replay.random()]))[0]
            assert record.action == want
            assert np.array_equal(record.probs, probs[0])
        for seat in range(4):
            assert np.array_equal(trajectory.streams[seat], np.asarray(game.streams[seat]))
        assert abs(trajectory.returns.sum()) < 1e-12


@pytest.mark.gpu
def test_collector_decisions_match_an_eager_prefill():
    import dataclasses

    from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    config = dataclasses.replace(RL_V6, n_layers=2)
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=4), precision="fp32")
    assert tuple(actor.heads_desc.width[:2]) == (BID, PLAY)
    pool = _pool()

    def deal(rng):
        seed = rng.randrange(1 << 30)
        return ScriptedGame(seed, pool, restart=2 if seed % 2 else None)

    lanes = [cont.Lane("plump", 4, 24, 40, deal=deal)]
    collector = cont.ContinuousCollector(actor, max_length=48, cohorts=2, kv_dtype="fp32", record_values=True)
    results = collector.collect(lanes, random.Random(7))
    assert len(results) == 40
    checked = 0
    cache = actor.new_cache(1, 48, torch.float32)
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            context = trajectory.streams[seat][base:length].astype(np.int64)
            hidden = actor.forward_prefill(torch.from_numpy(context[None]).cuda(), cache, rows=None)
            logits = actor.policy_logits(hidden, head).float().cpu().numpy()
            probs = oppo.masked_probabilities(logits, legal[None])[0]
            np.testing.assert_allclose(record.probs, probs, rtol=0, atol=2e-5)
            values = actor.player_values(hidden).float().cpu().numpy()[0]
            np.testing.assert_allclose(record.value, values, rtol=0, atol=2e-4)
            u = replay.random()
            assert record.action == oppo.sample_rows(record.probs[None], legal[None], np.array([u]))[0]
            checked += 1
    assert checked > 100
    assert collector.stats.waves > 0 and collector.stats.peak_rows > 0


@pytest.mark.gpu
def test_collector_runs_piquet_pointer_heads():
    """The collector over a piquet actor: the card scorers read each readout token's grid cards
    through ``pop_context`` inside the graphed wave; every recorded decision against an eager
    prefill of its context with the same context cards (fp32)."""

    from card_playing_gym_b200.piquet import PiquetActor, PiquetModelConfig

    data = load_golden("piquet_actor")
    config = PiquetModelConfig(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    actor = PiquetActor(config, {k[2:]: v for k, v in data.items() if k.startswith("w_")}, precision="fp32")
    pool = data["tokens"].reshape(-1, data["tokens"].shape[-1]).astype(np.int64)

    def deal(rng):
        seed = rng.randrange(1 << 30)
        return ScriptedPiquet(seed, pool, restart=3 if seed % 2 else None)

    lanes = [cont.Lane("piquet", 2, 20, 30, deal=deal)]
    collector = cont.ContinuousCollector(actor, max_length=48, cohorts=2, kv_dtype="fp32", record_values=True)
    results = collector.collect(lanes, random.Random(11))
    assert len(results) == 30
    cache = actor.new_cache(1, 48, torch.float32)
    checked = set()
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            context = trajectory.streams[seat][base:length].astype(np.int64)
            hidden = actor.forward_prefill(torch.from_numpy(context[None]).cuda(), cache, rows=None)
            cards = actor.pop_context()[:, -1]
            logits = actor.policy_logits(hidden, head, None, None, cards).cpu().numpy()
            probs = oppo.masked_probabilities(logits, legal[None])[0]
            np.testing.assert_allclose(record.probs, probs, rtol=0, atol=2e-5)
            np.testing.assert_allclose(record.value, actor.player_values(hidden).cpu().numpy()[0], rtol=0, atol=2e-4)
            assert record.action == oppo.sample_rows(record.probs[None], legal[None], np.array([replay.random()]))[0]
            checked.add(head)
    assert checked == {"exchange", "declare", "play"}


@pytest.mark.gpu
def test_collector_runs_rummy_candidate_heads():
    """The collector over a rummy actor (heads with per-decision candidate features, so eager
    waves as in the reference): every recorded decision against an eager prefill of its context,
    its ledger cards and its candidates (fp32)."""

    from card_playing_gym_b200.rummy import RummyActor, RummyModelConfig

    data = load_golden("rummy_actor")
    config = RummyModelConfig(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    actor = RummyActor(config, {k[2:]: v for k, v in data.items() if k.startswith("w_")}, precision="fp32")
    pool = data["tokens"].reshape(-1, data["tokens"].shape[-1]).astype(np.int64)

    def deal(rng):
        seed = rng.randrange(1 << 30)
        return ScriptedRummy(seed, pool, restart=2 if seed % 2 else None)

    lanes = [cont.Lane("rummy", 3, 16, 24, deal=deal)]
    collector = cont.ContinuousCollector(actor, max_length=48, cohorts=2, kv_dtype="fp32", record_values=True)
    results = collector.collect(lanes, random.Random(13))
    assert isinstance(collector.engine.half, cont.EagerHalf)
    assert len(results) == 24
    cache = actor.new_cache(1, 48, torch.float32)
    heads = set()
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length), features in zip(trajectory.decisions, game.log, game.features):
            context = trajectory.streams[seat][base:length].astype(np.int64)
            hidden = actor.forward_prefill(torch.from_numpy(context[None]).cuda(), cache, rows=None)
            cards = actor.pop_context()[:, -1]
            feats = {k: torch.from_numpy(v[None]).cuda() for k, v in features.items()}
            logits = actor.policy_logits(hidden, head, feats, None, cards).cpu().numpy()
            probs = oppo.masked_probabilities(logits, legal[None])[0]
            assert record.probs.shape == legal.shape
            np.testing.assert_allclose(record.probs, probs, rtol=0, atol=2e-5)
            np.testing.assert_allclose(record.value, actor.player_values(hidden).cpu().numpy()[0], rtol=0, atol=2e-4)
            assert record.action == oppo.sample_rows(record.probs[None], legal[None], np.array([replay.random()]))[0]
            heads.add(head)
    assert heads == {"draw", "play"}


def test_stack_features_pads_the_candidate_axis_with_zeros():
    """selfplay.py:570-587: each key stacked over decisions, zero-padded to the longest list."""

    a = {"kind": np.array([3, 1]), "cards": np.full((2, 13), 52)}
    b = {"kind": np.array([5, 6, 2]), "cards": np.arange(39).reshape(3, 13)}
    stacked = cont.stack_features([a, b])
    assert stacked["kind"].tolist() == [[3, 1, 0], [5, 6, 2]]
    assert stacked["cards"].shape == (2, 3, 13) and not stacked["cards"][0, 2].any()
    assert np.array_equal(stacked["cards"][1], b["cards"]) and stacked["cards"].dtype == b["cards"].dtype


@pytest.mark.gpu
def test_continuous_collector_probabilities_match_the_oracle():
    """Every decision the continuous collector records for a plump actor (graphed waves, context restarts, slot
    refills), against the CPU oracle (numpy float64): the oracle prefills the decision's context and scores
    the head; the reference's numpy sampler turns its logits into probabilities and a draw. fp32, fp32 KV."""

    import dataclasses

    from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor
    from oracle import plump as oplump
    from oracle.trunk import Precision

    config = dataclasses.replace(RL_V6, n_layers=2)
    state = synthetic_plump_actor_state(config, seed=6)
    actor = PlumpActor(config, state, precision="fp32")
    oracle = oplump.PlumpActor(state, {k: getattr(config, k) for k in (
        "d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff", "per_layer_dim", "value_embeddings", "max_players",
        "max_hand_size")}, Precision())
    pool = _pool()

    def deal(rng):
        seed = rng.randrange(1 << 30)
        return ScriptedGame(seed, pool, restart=2 if seed % 2 else None)

    collector = cont.ContinuousCollector(actor, max_length=48, cohorts=2, kv_dtype="fp32", record_values=True)
    # The first 24 games to finish (short ones come first): enough decisions of both heads to check.
    results = collector.collect([cont.Lane("plump", 4, 8, 24, deal=deal)], random.Random(41))
    checked = 0
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            context = trajectory.streams[seat][base:length].astype(np.int64)[None]
            hidden = oracle.forward_prefill(context, oracle.new_cache(1, context.shape[1] + 1), None)
            probs = oppo.masked_probabilities(oracle.heads.policy_logits(hidden, head).astype(np.float32), legal[None])
            np.testing.assert_allclose(record.probs, probs[0], rtol=1e-5, atol=1e-7)
            np.testing.assert_allclose(record.value, oracle.heads.player_values(hidden)[0], rtol=1e-5, atol=2e-6)
            u = replay.random()
            near = np.abs(np.cumsum(probs[0]).astype(np.float64) - u).min() < 1e-5
            assert record.action == oppo.sample_rows(probs, legal[None], np.array([u]))[0] or near
            checked += 1
    assert checked > 20
