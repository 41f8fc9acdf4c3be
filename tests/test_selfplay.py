"""The batch self-play collector (cardgym/rl/selfplay.py:208-484). CPU: its host bookkeeping
against a model whose KV rows hold the tokens written to them. GPU: scripted games over
the plump, piquet and rummy actors, in chunks of at most ``max_rows`` rows and two cohorts, so
that games end mid-chunk and the survivors' KV rows are compacted. Every recorded decision is
checked against an eager prefill of its context (fp32): probabilities, values, and the action
the game's own ``rng`` draws."""

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
    assert collector.stats.compactions > 0 and collector.stats.decisions == sum(len(g.actions) for g in games)
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
    """A KV pool whose rows hold the tokens written at each position (a list per row)."""

    def __init__(self, capacity: int, length: int):
        self.capacity, self.max_len = capacity, length
        self.rows = [[] for _ in range(capacity)]
        self.copies = 0

    def write(self, row: int, position: int, tokens) -> None:
        assert position <= len(self.rows[row]) or position == 0, (row, position, len(self.rows[row]))
        self.rows[row] = self.rows[row][:position] + [tuple(t) for t in tokens]
        assert len(self.rows[row]) < self.max_len

    def copy_rows(self, sources, targets, length: int) -> None:
        self.copies += 1
        staged = [list(self.rows[int(s)][:length]) for s in sources.tolist()]
        for target, tokens in zip(targets.tolist(), staged):
            self.rows[target] = tokens


class _TokenModel:
    """Records what each forward writes; its hidden state is the readout row's index."""

    def __init__(self):
        self.caches = []

    def new_cache(self, capacity, length, dtype):
        self.caches.append(_TokenCache(capacity, length))
        return self.caches[-1]

    def forward_prefill(self, tokens, cache, rows):
        for tok, row in zip(tokens.cpu().numpy(), rows.cpu().numpy()):
            cache.write(int(row), 0, tok)
        return torch.zeros(tokens.shape[0], 1)

    def forward_ragged(self, tokens, positions, cache, offsets, span=None, rows=None):
        assert rows is None
        for row, (tok, position, offset) in enumerate(zip(tokens.cpu().numpy(), positions.cpu().numpy(),
                                                          offsets.cpu().numpy())):
            cache.write(row, int(position), tok[: int(offset) + 1])
        return torch.zeros(tokens.shape[0], 1)


@pytest.mark.parametrize("cohorts", (1, 2))
def test_batch_collector_keeps_every_stream_in_its_rows(cohorts, monkeypatch):
    """Host logic without a GPU: after every wave, each live game's rows hold exactly its
    observers' current contexts (prefill, appends, compaction, context restarts), padding rows
    lie past the live prefix, and decisions replay each game's own rng."""

    from card_playing_gym_b200 import continuous as cont
    from card_playing_gym_b200 import selfplay

    checks = []

    def fake_launch(model, hidden, context, states, uniforms, *, values):
        wave = cont._Wave()
        for state, u in zip(states, uniforms):
            legal = state.pending.legal
            probs = oppo.masked_probabilities(np.zeros((1, legal.shape[0]), np.float32), legal[None])
            action = oppo.sample_rows(probs, legal[None], np.array([u]))
            wave.readouts.append(cont._Readout([state], torch.from_numpy(probs), torch.from_numpy(action), None))
        checks.append(list(states))
        return wave

    monkeypatch.setattr(selfplay, "launch_decisions", fake_launch)
    monkeypatch.setattr(selfplay, "_pinned", lambda array, device: torch.from_numpy(np.ascontiguousarray(array)))
    model = _TokenModel()
    pool = _pool()
    rng = random.Random(23)
    games = [ScriptedGame(rng.randrange(1 << 30), pool, restart=2 if i % 3 == 0 else None) for i in range(25)]
    collector = selfplay.SelfPlayCollector(model, device="cpu", max_rows=40, max_length=64, cohorts=cohorts)

    def verify(cohort):
        for _, state in cohort.live:
            for seat in range(state.game.num_players):
                stream = np.asarray(state.game.streams[seat])
                context = stream[state.offsets[seat]: state.offsets[seat] + state.lengths[seat]]
                stored = np.asarray(cohort.cache.rows[state.base + seat][: state.lengths[seat]])
                assert np.array_equal(stored, context), (state.base, seat)

    original = selfplay.SelfPlayCollector._append

    def checked_append(self, cohort, appends):
        original(self, cohort, appends)
        verify(cohort)
        checks.append(None)

    monkeypatch.setattr(selfplay.SelfPlayCollector, "_append", checked_append)
    results = collector.collect(games)
    assert [t.game for t in results] == games and collector.stats.compactions > 0
    assert 10 < checks.count(None) <= collector.stats.waves  # a cohort's last wave appends nothing
    assert sum(cache.copies for cache in model.caches) == collector.stats.compactions
    for trajectory in results:
        game = trajectory.game
        replay = random.Random(game.seed ^ 0x5EED)
        for record, (seat, head, legal, base, length) in zip(trajectory.decisions, game.log):
            assert record.position == length - 1
            probs = oppo.masked_probabilities(np.zeros((1, legal.shape[0]), np.float32), legal[None])
            assert record.action == oppo.sample_rows(probs, legal[None], np.array([replay.random()]))[0]
        assert [r.action for r in trajectory.decisions] == game.actions
