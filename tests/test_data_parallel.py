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


def _model(seed: int = 0) -> torch.nn.Module:
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(6, 16), torch.nn.GELU(), torch.nn.Linear(16, 16), torch.nn.GELU(),
                               torch.nn.Linear(16, 1))


def _objective(model, features, targets, weights) -> torch.Tensor:
    """A weighted-sum objective like the trainer's: weights already divide by the global count."""

    out = model(torch.from_numpy(features)).squeeze(-1)
    return (torch.from_numpy(weights).float() * (out - torch.from_numpy(targets)) ** 2).sum()


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
        _objective(model, features[d0:d1], targets[d0:d1], weights[d0:d1]).backward()
        reducer.finish()
        grads = [p.grad.clone() for p in model.parameters()]
        norm = float(global_grad_norm(model.parameters()))
        # A second backward through the same reducer (re-armed by finish) gives the same sums.
        model.zero_grad(set_to_none=True)
        _objective(model, features[d0:d1], targets[d0:d1], weights[d0:d1]).backward()
        reducer.finish()
        again = all(torch.equal(a, p.grad) for a, p in zip(grads, model.parameters()))
        reducer.close()
        results.put((rank, (g0, g1), mean, std, entropy.tolist(), [g.numpy() for g in grads], norm, again))
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


def test_bucketed_gradient_sum_matches_the_whole_batch(ranks):
    _, _, weights, features, targets = _batch()
    model = _model()
    _objective(model, features, targets, weights).backward()
    expected = [p.grad.numpy() for p in model.parameters()]
    expected_norm = float(global_grad_norm(model.parameters()))
    for rank in range(WORLD):
        for got, want in zip(ranks[rank][4], expected):
            np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)
        assert ranks[rank][5] == pytest.approx(expected_norm, rel=1e-5)
        assert ranks[rank][6]  # re-armed reducer reproduces the sums
    # every rank holds identical reduced gradients
    for a, b in zip(ranks[0][4], ranks[1][4]):
        assert np.array_equal(a, b)
