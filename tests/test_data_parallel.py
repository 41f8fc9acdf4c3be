"""Data-parallel PPO update helpers on CPU: gloo ranks (world size 2) against one process.

The exchanges of the sharded update (trajectory shards, the batch-global two-pass weighted
mean/std, per-head entropy sums, bucketed gradient SUM-allreduce overlapped with backward)
must reproduce the single-process update on the whole batch.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from card_playing_gym_b200.data_parallel import (
    GradientAllreduce,
    allreduce_head_entropy,
    global_grad_norm,
    global_weighted_mean_std,
    shard_games,
)

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _host_sums(values: torch.Tensor, weights: torch.Tensor, shift: float) -> torch.Tensor:
    """(sum w, sum w (x - shift), sum w (x - shift)^2) on the host, float64 (test stand-in for the kernel)."""

    x = values.to(torch.float64) - shift
    w = weights.to(torch.float64)
    return torch.stack([w.sum(), (w * x).sum(), (w * x * x).sum()])


def _reference_mean_std(values: np.ndarray, weights: np.ndarray) -> tuple[float, float]:
    """ppo.py:147-153 of the reference on one process: two-pass weighted mean and std."""

    total = weights.sum()
    mean = float((weights * values).sum() / total)
    var = float((weights * (values - mean) ** 2).sum() / total)
    return mean, float(np.sqrt(max(var, 1e-12)))


def _batch(seed: int = 3):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(13, 53, 61)
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    n = int(starts[-1])
    advantages = rng.standard_normal(n) * 3.0 + 0.7
    weights = np.full(n, 1.0 / (len(lengths) * 4))
    features = rng.standard_normal((n, 6)).astype(np.float32)
    targets = rng.standard_normal(n).astype(np.float32)
    return starts, advantages, weights, features, targets


class _Actor(torch.nn.Module):
    """A trunk, two heads and a parameter no loss reaches: head_b is used only by the first decisions of
    the batch, which all fall in rank 0's shard, so rank 1 never produces a gradient for it."""

    def __init__(self) -> None:
        super().__init__()
        self.trunk = torch.nn.Sequential(torch.nn.Linear(6, 16), torch.nn.GELU(), torch.nn.Linear(16, 16),
                                         torch.nn.GELU())
        self.head_a = torch.nn.Linear(16, 1)
        self.head_b = torch.nn.Linear(16, 1)
        self.unused = torch.nn.Parameter(torch.zeros(3))


HEAD_B_ROWS = 40  # decisions [0, 40) use head_b as well


def _model(seed: int = 0) -> _Actor:
    torch.manual_seed(seed)
    return _Actor()


def _losses(model, features, targets, weights, first: int):
    """(policy, auxiliary) for decisions [first, first + len) of the batch, like the trainer's two halves:
    weighted sums whose weights already divide by the global count."""

    hidden = model.trunk(torch.from_numpy(features))
    out = model.head_a(hidden).squeeze(-1)
    index = torch.arange(first, first + len(features))
    uses_b = index < HEAD_B_ROWS
    if bool(uses_b.any()):  # head_b only enters the graph of microbatches that use it
        out = out + uses_b.float() * model.head_b(hidden).squeeze(-1)
    w = torch.from_numpy(weights).float()
    policy = (w * (out - torch.from_numpy(targets)) ** 2).sum()
    auxiliary = (w * hidden.square().mean(-1)).sum()
    return policy, auxiliary


def _objective(model, features, targets, weights, first: int = 0) -> torch.Tensor:
    policy, auxiliary = _losses(model, features, targets, weights, first)
    return policy + 0.5 * auxiliary


def _stash(stash, gradients):
    """The reference's _accumulate (trainer.py:206-223): sum autograd.grad results, keeping None."""

    if stash is None:
        return [None if g is None else g.detach().clone() for g in gradients]
    for i, g in enumerate(gradients):
        if g is not None:
            stash[i] = g.detach().clone() if stash[i] is None else stash[i] + g
    return stash


def _step_gradients(model, features, targets, weights, first: int, micro: int = 3):
    """One optimizer step's accumulation over `micro` microbatches: .grad from backward (the budget off), and
    the (policy, auxiliary) stashes from autograd.grad (the budget on)."""

    model.zero_grad(set_to_none=True)
    params = list(model.parameters())
    policy_stash = auxiliary_stash = None
    bounds = np.linspace(0, len(features), micro + 1).astype(int)
    for a, b in zip(bounds[:-1], bounds[1:]):
        _objective(model, features[a:b], targets[a:b], weights[a:b], first + a).backward()
    for a, b in zip(bounds[:-1], bounds[1:]):
        policy, auxiliary = _losses(model, features[a:b], targets[a:b], weights[a:b], first + a)
        auxiliary_stash = _stash(auxiliary_stash, torch.autograd.grad(auxiliary, params, retain_graph=True,
                                                                      allow_unused=True))
        policy_stash = _stash(policy_stash, torch.autograd.grad(policy, params, allow_unused=True))
    return policy_stash, auxiliary_stash


def _as_numpy(grads):
    return [None if g is None else g.detach().numpy().copy() for g in grads]


def _worker(rank: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        starts, advantages, weights, features, targets = _batch()
        g0, g1 = shard_games(starts, WORLD, rank)
        d0, d1 = int(starts[g0]), int(starts[g1])
        local_adv = torch.from_numpy(advantages[d0:d1])
        local_w = torch.from_numpy(weights[d0:d1])
        mean, std = global_weighted_mean_std(local_adv, local_w, sums=_host_sums)

        observed = torch.tensor([[float(local_w.sum()) * (rank + 1), float(local_w.sum())], [0.0, 0.0]],
                                dtype=torch.float64)
        entropy = allreduce_head_entropy(observed)

        model = _model()
        reducer = GradientAllreduce(model.parameters(), bucket_bytes=256)  # several buckets
        head_b_local = model.head_b.weight.grad
        steps = []
        for _ in range(2):  # two optimizer steps through the same reducer
            policy, auxiliary = _step_gradients(model, features[d0:d1], targets[d0:d1], weights[d0:d1], d0)
            head_b_local = model.head_b.weight.grad
            reducer.reduce_grads()
            grads = _as_numpy(p.grad for p in model.parameters())
            norm = float(global_grad_norm(model.parameters()))
            steps.append((grads, norm, _as_numpy(reducer.reduce_(policy)), _as_numpy(reducer.reduce_(auxiliary))))
        results.put((rank, (g0, g1), mean, std, entropy.tolist(), steps, head_b_local is None))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def ranks():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, results)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(WORLD):
            rank, *rest = results.get(timeout=120)
            out[rank] = rest
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    return out


@pytest.mark.parametrize("world", (1, 2, 3, 8))
def test_shards_cover_every_game_once_and_balance_decisions(world):
    starts = _batch()[0]
    edges = [shard_games(starts, world, r) for r in range(world)]
    assert edges[0][0] == 0 and edges[-1][1] == len(starts) - 1
    assert all(a[1] == b[0] for a, b in zip(edges, edges[1:]))
    sizes = [int(starts[g1] - starts[g0]) for g0, g1 in edges]
    assert sum(sizes) == int(starts[-1])
    assert max(sizes) - min(sizes) <= 2 * 52


def test_shard_games_rejects_bad_input():
    with pytest.raises(ValueError):
        shard_games([0, 5, 3], 2, 0)
    with pytest.raises(ValueError):
        shard_games([0, 5], 2, 2)


def test_global_mean_std_matches_one_process(ranks):
    _, advantages, weights, _, _ = _batch()
    mean, std = _reference_mean_std(advantages, weights)
    for rank in range(WORLD):
        got_mean, got_std = ranks[rank][1], ranks[rank][2]
        assert got_mean == pytest.approx(mean, rel=1e-12, abs=1e-15)
        assert got_std == pytest.approx(std, rel=1e-12)


def test_head_entropy_is_the_global_weighted_mean(ranks):
    # rank r reports H = r + 1 on head 0 with its shard's weight; head 1 saw nothing.
    starts, _, weights, _, _ = _batch()
    w = [float(weights[int(starts[g0]):int(starts[g1])].sum()) for g0, g1 in (ranks[r][0] for r in range(WORLD))]
    expected = (w[0] * 1 + w[1] * 2) / (w[0] + w[1])
    for rank in range(WORLD):
        head0, head1 = ranks[rank][3]
        assert head0 == pytest.approx(expected, rel=1e-12)
        assert head1 == 0.0


def _whole_batch_step():
    _, _, weights, features, targets = _batch()
    model = _model()
    policy, auxiliary = _step_gradients(model, features, targets, weights, 0, micro=5)
    grads = _as_numpy(p.grad for p in model.parameters())
    return grads, float(global_grad_norm(model.parameters())), _as_numpy(policy), _as_numpy(auxiliary)


def _assert_same(got, want):
    assert len(got) == len(want)
    for g, w in zip(got, want):
        assert (g is None) == (w is None)
        if w is not None:
            np.testing.assert_allclose(g, w, rtol=1e-5, atol=1e-7)


def test_accumulated_gradients_sum_to_the_whole_batch(ranks):
    """Several backward passes per optimizer step (3 microbatches on each rank, 5 on one process), reduced once
    after the last: .grad, the policy and auxiliary autograd.grad stashes, and the clip norm all equal one
    process's accumulation over the whole batch, on both optimizer steps."""

    grads, norm, policy, auxiliary = _whole_batch_step()
    for rank in range(WORLD):
        for step_grads, step_norm, step_policy, step_aux in ranks[rank][4]:
            _assert_same(step_grads, grads)
            _assert_same(step_policy, policy)
            _assert_same(step_aux, auxiliary)
            assert step_norm == pytest.approx(norm, rel=1e-5)
    for a, b in zip(ranks[0][4][0][0], ranks[1][4][0][0]):
        assert (a is None and b is None) or np.array_equal(a, b)


def test_gradients_present_on_one_rank_only_are_summed_and_absent_ones_stay_none(ranks):
    names = [name for name, _ in _model().named_parameters()]
    unused = names.index("unused")
    head_b = names.index("head_b.weight")
    assert ranks[1][5], "rank 1's shard must never reach head_b"
    assert not ranks[0][5]
    for rank in range(WORLD):
        grads, _, policy, auxiliary = ranks[rank][4][0]
        assert grads[unused] is None and policy[unused] is None and auxiliary[unused] is None
        assert grads[head_b] is not None and policy[head_b] is not None
        assert auxiliary[head_b] is None  # the auxiliary loss never reaches head_b on any rank
