"""The batch self-play collector (cardgym/rl/selfplay.py:208-484). CPU: its host bookkeeping
against a model whose KV rows hold the tokens written to them. GPU: scripted games over
the plump, piquet and rummy actors, in chunks of at most ``max_rows`` rows and two cohorts, so
that games end mid-chunk while the others keep their rows. Every recorded decision is checked
against an eager prefill of its context (fp32): probabilities, values, and the action the game's
own ``rng`` draws."""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from oracle import ppo as oppo
from tests.conftest import load_golden
from tests.test_continuous import ScriptedGame, ScriptedPiquet, ScriptedRummy, _pool


def _actor(kind: str):
    if kind == "plump":
        import dataclasses

        from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
        from card_playing_gym_b200.plump import PlumpActor

        config = dataclasses.replace(RL_V6, n_layers=2)
        return PlumpActor(config, synthetic_plump_actor_state(config, seed=4), precision="fp32"), ScriptedGame, _pool()
    from card_playing_gym_b200 import piquet, rummy

    module, game = (piquet, ScriptedPiquet) if kind == "piquet" else (rummy, ScriptedRummy)
    data = load_golden(f"{kind}_actor")
    config_cls = piquet.PiquetModelConfig if kind == "piquet" else rummy.RummyModelConfig
    config = config_cls(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    actor_cls = piquet.PiquetActor if kind == "piquet" else rummy.RummyActor
    actor = actor_cls(config, {k[2:]: v for k, v in data.items() if k.startswith("w_")}, precision="fp32")
    return actor, game, data["tokens"].reshape(-1, data["tokens"].shape[-1]).astype(np.int64)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ("plump", "piquet", "rummy"))
def test_batch_collector_decisions_match_an_eager_prefill(kind):
    from card_playing_gym_b200.selfplay import SelfPlayCollector

    actor, game_cls, pool = _actor(kind)
    rng = random.Random(17)
    games = [game_cls(rng.randrange(1 << 30), pool, restart=2 if i % 3 == 0 else None) for i in range(30)]
    players = games[0].num_players
    collector = SelfPlayCollector(actor, max_rows=12 * players, max_length=48, cohorts=2, kv_dtype="fp32",
                                  record_values=True)
    results = collector.collect(games)
    assert [t.game for t in results] == games
    assert collector.stats.decisions == sum(len(g.actions) for g in games)
    cache = actor.new_cache(1, 48, torch.float32)
    checked = 0
    for trajectory in results:
        game = trajectory.game
        assert [record.action for record in trajectory.decisions] == game.actions
        replay = random.Random(game.seed ^ 0x5EED)
        features_log = getattr(game, "features", [None] * len(game.log))
        for record, (seat, head, legal, base, length), features in zip(trajectory.decisions, game.log, features_log):
            assert record.position == length - 1
            context = trajectory.streams[seat][base:length].astype(np.int64)
            hidden = actor.forward_prefill(torch.from_numpy(context[None]).cuda(), cache, rows=None)
            pop = getattr(actor, "pop_context", None)
            cards = pop()[:, -1] if pop is not None else None
            feats = None if features is None else {k: torch.from_numpy(v[None]).cuda() for k, v in features.items()}
            logits = actor.policy_logits(hidden, head, feats, None, cards).float().cpu().numpy()
            probs = oppo.masked_probabilities(logits[:, : legal.shape[0]], legal[None])[0]
            np.testing.assert_allclose(record.probs, probs, rtol=0, atol=2e-5)
            np.testing.assert_allclose(record.value, actor.player_values(hidden).float().cpu().numpy()[0],
                                       rtol=0, atol=2e-4)
            assert record.action == oppo.sample_rows(record.probs[None], legal[None], np.array([replay.random()]))[0]
            checked += 1
    assert checked > 50


class _TokenCache:
    """A KV pool whose rows hold the token written at each position, as the decode kernels write it: every
    entry writes its whole padded run, positions clamped to the pool's last slot (the spare padding slot)."""

    def __init__(self, capacity: int, length: int):
        self.capacity, self.max_len = capacity, length
        self.rows = [[None] * length for _ in range(capacity)]

    def write(self, row: int, position: int, run) -> None:
        for step, token in enumerate(run):
            self.rows[row][min(position + step, self.max_len - 1)] = tuple(token)


class _TokenModel:
    precision = "bf16"

    def __init__(self):
        self.caches = []

    def new_cache(self, capacity, length, dtype):
        self.caches.append(_TokenCache(capacity, length))
        return self.caches[-1]


class _TokenHalf:
    """Writes each wave into the token pool, then checks every game in the wave: the first ``cached`` slots
    of each of its rows hold exactly that observer's current context; samples uniformly over the legal
    actions with each game's uniform (the oracle's inverse CDF)."""

    def __init__(self, cache, engine_of):
        self.cache, self.engine_of = cache, engine_of
        self.waves = 0

    def launch(self, wave, readouts):
        from card_playing_gym_b200 import rollout

        self.waves += 1
        assert (wave.cache_rows[wave.count:] == self.cache.capacity - 1).all()  # padding: the scratch row only
        for entry in range(wave.tokens.shape[0]):
            self.cache.write(int(wave.cache_rows[entry]), int(wave.positions[entry]), wave.tokens[entry])
        table = self.engine_of().table
        for _, trace, _ in readouts:
            for seat in range(trace.game.num_players):
                row = trace.base + seat
                start, length = int(table.shift[row]), int(table.cached[row])
                context = [tuple(t) for t in np.asarray(trace.game.streams[seat])[start:start + length]]
                assert self.cache.rows[row][:length] == context, (row, seat)
        result = rollout.WaveInFlight()
        for _, trace, u in readouts:
            legal = trace.pending.legal
            probs = oppo.masked_probabilities(np.zeros((1, legal.shape[0]), np.float32), legal[None])
            action = oppo.sample_rows(probs, legal[None], np.array([u]))
            result.groups.append(rollout.SampledGroup([trace], torch.from_numpy(probs), torch.from_numpy(action), None))
        return result


@pytest.mark.parametrize("cohorts", (1, 2))
def test_batch_collector_keeps_every_stream_in_its_rows(cohorts):
    """Host logic without a GPU: after every wave's writes (padding included), each game's rows hold exactly
    its observers' current contexts (prefixes, appends, context restarts, games ending mid-chunk), padding
    entries write only the scratch row, and decisions replay each game's own rng."""

    from card_playing_gym_b200 import selfplay

    model = _TokenModel()
    halves = []
    pool = _pool()
    rng = random.Random(23)
    games = [ScriptedGame(rng.randrange(1 << 30), pool, restart=2 if i % 3 == 0 else None) for i in range(25)]
    collector = selfplay.SelfPlayCollector(
        model, device="cpu", max_rows=40, max_length=64, cohorts=cohorts,
        half_factory=lambda cache, values: halves.append(_TokenHalf(cache, lambda: collector.engine)) or halves[-1])
    results = collector.collect(games)
    assert [t.game for t in results] == games and collector.stats.compactions == 0
    assert sum(half.waves for half in halves) == collector.stats.waves > 10
    assert collector.stats.peak_rows <= 40
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            assert record.position == length - 1
            probs = oppo.masked_probabilities(np.zeros((1, legal.shape[0]), np.float32), legal[None])
            assert record.action == oppo.sample_rows(probs, legal[None], np.array([replay.random()]))[0]
        assert [r.action for r in trajectory.decisions] == game.actions
        for seat in range(game.num_players):
            assert np.array_equal(trajectory.streams[seat], np.asarray(game.streams[seat]))


@pytest.mark.gpu
def test_batch_collector_probabilities_match_the_oracle():
    """Every decision the batch collector records for a plump actor, against the CPU oracle (numpy float64):
    the oracle prefills the decision's context, scores the head, and the reference's numpy sampler turns
    its logits into probabilities and a draw with the game's own uniform. fp32 mode, fp32 KV."""

    import dataclasses

    from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor
    from card_playing_gym_b200.selfplay import SelfPlayCollector
    from oracle import plump as oplump
    from oracle.trunk import Precision

    config = dataclasses.replace(RL_V6, n_layers=2)
    state = synthetic_plump_actor_state(config, seed=4)
    actor = PlumpActor(config, state, precision="fp32")
    oracle = oplump.PlumpActor(state, {k: getattr(config, k) for k in (
        "d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff", "per_layer_dim", "value_embeddings", "max_players",
        "max_hand_size")}, Precision())
    pool = _pool()
    rng = random.Random(29)
    games = [ScriptedGame(rng.randrange(1 << 30), pool, restart=2 if i % 3 == 0 else None) for i in range(16)]
    collector = SelfPlayCollector(actor, max_rows=32, max_length=48, cohorts=2, kv_dtype="fp32", record_values=True)
    results = collector.collect(games)
    checked = boundary = 0
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            context = trajectory.streams[seat][base:length].astype(np.int64)[None]
            ocache = oracle.new_cache(1, context.shape[1] + 1)
            hidden = oracle.forward_prefill(context, ocache, None)
            logits = oracle.heads.policy_logits(hidden, head).astype(np.float32)
            probs = oppo.masked_probabilities(logits, legal[None])
            np.testing.assert_allclose(record.probs, probs[0], rtol=1e-5, atol=1e-7)
            np.testing.assert_allclose(record.value, oracle.heads.player_values(hidden)[0], rtol=1e-5, atol=2e-6)
            u = replay.random()
            drawn = oppo.sample_rows(probs, legal[None], np.array([u]))[0]
            cdf = np.cumsum(probs[0]).astype(np.float64)
            near = np.abs(cdf - u).min() < 1e-5
            boundary += int(near)
            assert record.action == drawn or near
            checked += 1
    assert checked > 30
    print(f"{checked} decisions against the oracle, {boundary} within 1e-5 of a CDF step")
