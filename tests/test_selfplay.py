"""The batch self-play collector (cardgym/rl/selfplay.py:208-484) on a B200: scripted games over
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

pytestmark = pytest.mark.gpu


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
