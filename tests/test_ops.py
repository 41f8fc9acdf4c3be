"""The torch custom ops (card_playing_gym_b200.ops): fake kernels on the CPU (shapes and dtypes a
trace sees, no kernel runs), and on the GPU each op against the direct C-ABI wrapper it stands for,
plus torch.library.opcheck on the ops that only read their inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from card_playing_gym_b200 import ops  # noqa: F401  (registers the ops)

OPS = torch.ops.cardgym_b200


def test_fake_kernels_give_the_output_shapes():
    with FakeTensorMode():
        logits = torch.empty((5, 52))
        probs, actions = OPS.masked_sample(logits, torch.empty((5, 52), dtype=torch.uint8), torch.empty(5, dtype=torch.float64))
        assert probs.shape == (5, 52) and actions.dtype == torch.int64 and actions.shape == (5,)
        adv = OPS.segmented_gae(torch.empty((30, 4), dtype=torch.float64), torch.empty(30, dtype=torch.int32),
                                torch.empty(3, dtype=torch.int64), torch.empty((2, 4), dtype=torch.float64), 0.95)
        assert adv.shape == (30,) and adv.dtype == torch.float64
        dlogits, terms, totals = OPS.ppo_objective(logits, logits, torch.empty(5, dtype=torch.int64), torch.empty(5),
                                                   torch.empty(5), 0.2, 0.01)
        assert dlogits.shape == (5, 52) and terms.shape == (5, 8) and totals.shape == (8,)
        grad, sums = OPS.value_loss(torch.empty((7, 4)), torch.empty(7, dtype=torch.int32), torch.empty((7, 4)),
                                    torch.empty(7), 5.0)
        assert grad.shape == (7, 4) and sums.dtype == torch.float64
        state, prediction = OPS.seat_values(torch.empty((9, 5)), torch.empty(6, dtype=torch.int64),
                                            torch.empty(6, dtype=torch.int64), torch.empty(6, dtype=torch.int64),
                                            None, True)
        assert state.shape == (6, 5) and prediction.shape == (6,)
        desc = [240, 2, 5, 52] + [11, 52] + [0] * 6 + [0] * 8 + [0] * 8 + [0, 0, 0, 0]
        out = OPS.plump_decide(desc, torch.empty(10), torch.empty((4, 240)), None, torch.empty(4, dtype=torch.int32),
                               torch.empty((4, 52), dtype=torch.uint8), torch.empty(4, dtype=torch.float64))
        assert [t.shape for t in out] == [(4, 52), (4, 52), (4,), (4, 5)]
        pool = torch.empty((16, 33, 2, 17, 24), dtype=torch.float16)
        hidden = OPS.trunk_forward_ragged([240, 16, 10, 2, 720, 64, 1, 0, 0], torch.empty(10), torch.empty((8, 1, 240)),
                                          None, None, pool, pool, torch.empty(8, dtype=torch.int64),
                                          torch.empty(8, dtype=torch.int64), None, 17, 1, torch.empty(64, dtype=torch.uint8))
        assert hidden.shape == (8, 240) and hidden.dtype == torch.float32
        q = torch.empty((3, 10, 1, 24), dtype=torch.float16)
        assert OPS.decode_attention(q, pool[0], pool[0], torch.empty(3, dtype=torch.int64),
                                    torch.empty(3, dtype=torch.int64), 17, 0.2).shape == q.shape


@pytest.mark.gpu
def test_ops_match_the_direct_wrappers():
    from card_playing_gym_b200 import ppo, sampling
    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    rng = np.random.default_rng(3)
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    logits = cuda(rng.standard_normal((300, 52)).astype(np.float32))
    mask = cuda(rng.random((300, 52)) < 0.4)
    mask[:, 0] = True
    uniforms = cuda(rng.random(300))
    probs, actions = OPS.masked_sample(logits, mask, uniforms)
    want_probs, want_actions = sampling.masked_sample(logits, mask, uniforms)
    assert torch.equal(probs, want_probs) and torch.equal(actions, want_actions)
    torch.library.opcheck(OPS.masked_sample, (logits, mask.to(torch.uint8), uniforms))

    values = cuda(rng.standard_normal((40, 4)))
    seats = cuda(rng.integers(0, 4, 40).astype(np.int32))
    starts = cuda(np.array([0, 17, 40]))
    returns = cuda(rng.standard_normal((2, 4)))
    assert torch.equal(OPS.segmented_gae(values, seats, starts, returns, 0.9),
                       ppo.segmented_gae(values, seats, starts, returns, 0.9))
    torch.library.opcheck(OPS.segmented_gae, (values, seats, starts, returns, 0.9))

    old = probs
    advantages = cuda(rng.standard_normal(300).astype(np.float32))
    weights = torch.full((300,), 1 / 300, device="cuda")
    dlogits, _, totals = OPS.ppo_objective(logits + 0.05, old, actions, advantages, weights, 0.2, 0.01)
    leaf = (logits + 0.05).requires_grad_()
    objective, want_totals = ppo.policy_objective(leaf, old, actions, advantages, weights, clip_ratio=0.2, alpha=0.01)
    objective.backward()
    assert torch.equal(dlogits, leaf.grad) and torch.equal(totals, want_totals)

    config = PlumpModelConfig()
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=2), precision="bf16")
    hidden = cuda(rng.standard_normal((64, config.d_model)).astype(np.float32))
    heads = cuda(rng.integers(0, 2, 64).astype(np.int32))
    legal = cuda(rng.random((64, 52)) < 0.5)
    legal[:, 0] = True
    draws = cuda(rng.random(64))
    out = OPS.plump_decide(ops.heads_desc_list(actor.heads_desc), actor.heads, hidden, None, heads, legal, draws)
    want = actor.decide(hidden, heads, legal, draws)
    assert all(torch.equal(a, b) for a, b in zip(out, want))

    # The trunk op on its own inputs (Trunk.condition's outputs): the fp32 trunk conditions separately; the bf16
    # trunk folds the conditioning into its first fused layer and takes raw lookups only inside forward_ragged.
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=2), precision="fp32")
    tokens = torch.from_numpy(np.load("tests/golden/plump_streams.npz")["tokens"][:8, :3].astype(np.int64)).cuda()
    x, ple, values_in = actor.prepare(tokens)
    caches = [actor.new_cache(8, 8, torch.float16) for _ in range(2)]
    positions = torch.zeros(8, dtype=torch.int64, device="cuda")
    offsets = torch.full((8,), 2, dtype=torch.int64, device="cuda")
    workspace = torch.empty(actor.trunk.step_workspace_bytes(8, 3), dtype=torch.uint8, device="cuda")
    got = OPS.trunk_forward_ragged(ops.trunk_dims_list(actor.trunk.dims), actor.trunk.blob, x, ple, values_in,
                                   caches[0].k_pool, caches[0].v_pool, positions, offsets, None, 3, 0, workspace)
    want = actor.trunk.forward_ragged(x, ple, values_in, caches[1], positions, offsets, span=3)
    assert torch.equal(got, want)
    assert torch.equal(caches[0].k_pool, caches[1].k_pool) and torch.equal(caches[0].v_pool, caches[1].v_pool)
