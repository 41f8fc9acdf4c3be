"""DecodeGraphs (cardgym/rl/graphs.py:66-151): a captured decode wave replays bit-for-bit what
the eager calls compute, across replays of one shape and a second captured shape, and leaves
the same KV cache behind."""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from tests.conftest import load_golden

pytestmark = pytest.mark.gpu


def test_decode_graphs_replay_matches_the_eager_wave():
    from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
    from card_playing_gym_b200.graphs import DecodeGraphs
    from card_playing_gym_b200.plump import PlumpActor

    config = dataclasses.replace(RL_V6, n_layers=3)
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=21), precision="bf16")
    streams = load_golden("plump_streams")["tokens"].astype(np.int64)[:32]
    batch = streams.shape[0]
    graph_cache = actor.new_cache(batch + 1, 16, torch.float16)
    eager_cache = actor.new_cache(batch + 1, 16, torch.float16)
    graphs = DecodeGraphs(actor, graph_cache, values=True)
    cache_rows = np.arange(1, batch + 1, dtype=np.int64)  # row 0 stays the scratch row
    position = 0
    for run in (1, 1, 1, 2, 2, 1):
        tokens = streams[:, position:position + run]
        positions = np.full(batch, position, np.int64)
        offsets = np.full(batch, run - 1, np.int64)
        got = graphs.run(tokens, positions, offsets, cache_rows, span=16).clone()
        cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        hidden = actor.forward_ragged(cuda(tokens), cuda(positions), eager_cache, cuda(offsets), span=16,
                                      rows=cuda(cache_rows))
        want = torch.cat([actor.policy_logits(hidden, head) for head in actor.policy_heads]
                         + [actor.player_values(hidden)], dim=-1)
        assert torch.equal(got, want), (run, position)
        position += run
    assert len(graphs) == 2
    assert set(graphs.columns) == {*actor.policy_heads, "values"}
    assert torch.equal(graph_cache.k_pool, eager_cache.k_pool)
    assert torch.equal(graph_cache.v_pool, eager_cache.v_pool)
