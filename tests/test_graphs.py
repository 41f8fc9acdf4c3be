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


def test_graphed_ppo_step_matches_the_eager_step():
    """The PPO advantage + loss step replayed as one CUDA graph (ppo.GraphedStep) gives the
    eager step's gradients bit for bit, replay after replay, as its inputs are refilled."""

    import bench
    from card_playing_gym_b200 import ppo
    from card_playing_gym_b200.data_parallel import normalize_global_

    batch = bench.synthetic_ppo_batch(20000, seed=3)
    cuda = lambda a, dtype=None: torch.as_tensor(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)  # noqa: E731
    values = cuda(batch["values"], torch.float64)
    seats = cuda(batch["seats"], torch.int32)
    starts = cuda(batch["starts"], torch.int64)
    returns = cuda(batch["returns"], torch.float64)
    logits = cuda(batch["logits"])
    old_probs = cuda(batch["old_probs"])
    actions = cuda(batch["actions"])
    weights = cuda(batch["weights"], torch.float32)
    weights64 = cuda(batch["weights"], torch.float64)
    prediction = cuda(batch["prediction"])
    targets = cuda(batch["targets"])
    players = torch.full((values.shape[0],), 4, dtype=torch.int32, device="cuda")

    def step():
        advantages = ppo.segmented_gae(values, seats, starts, returns, 0.95)
        normalize_global_(advantages, weights64)
        leaf = logits.detach().requires_grad_()
        objective, _ = ppo.policy_objective(leaf, old_probs, actions, advantages, weights, clip_ratio=0.2, alpha=0.01)
        pred = prediction.detach().requires_grad_()
        loss, _ = ppo.value_loss(pred, players, targets, weights, 1.0)
        (objective + loss).backward()
        return leaf.grad, pred.grad

    graphed = ppo.GraphedStep(step)
    for trial in range(3):
        if trial:
            logits.add_(0.01)  # new inputs, refilled in place
            values.mul_(0.9)
        want = [g.clone() for g in step()]
        got = graphed()
        assert all(torch.equal(a, b) for a, b in zip(got, want)), trial
