"""The PPO update drop-in (card_playing_gym_b200.trainer.device_trainer) against the reference's own trainer.

The reference's smoke configuration (configs/plump/smoke.toml: 2-layer d 32 plump actor and critic,
fp32, critic epochs 2, actor value probe, auxiliary-gradient budget 0.25, adaptive entropy targets)
runs three iterations: each iteration's games are collected by the reference's own CPU collector with
the CPU trainer's actor, and the same batch is updated by three trainers that started from the same
weights: the reference on the CPU (the oracle), the reference on the GPU, and the device trainer on the
GPU. Every statistic the update reports must match the CPU oracle within fp32 tolerance, no worse than
the reference's own GPU run does.

The unmodified reference is imported from baseline/_ref (``__graft_entry__.build()`` places it there);
the test is skipped where it is absent.
"""

from __future__ import annotations

import copy
import os
import random
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REFERENCE = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not (REFERENCE / "cardgym").is_dir(),
                                                  reason="the reference is not installed in baseline/_ref")]

# Statistics that are timings, device memory or the learning-rate schedule, not arithmetic.
NOT_COMPARED = ("update_sec", "peak_device_bytes")


def _reference():
    if str(REFERENCE) not in sys.path:
        sys.path.insert(0, str(REFERENCE))
    os.environ["CARDGYM_COMPILE"] = "0"  # eager torch on every device: the comparison is about arithmetic
    from cardgym.rl import loop, setup, trainer

    return loop, setup, trainer


def _trainer(cls, actor, critic, components, device, **extra):
    config = components.config
    game = config.game
    return cls(copy.deepcopy(actor), copy.deepcopy(critic), config.ppo, game.hooks(device, config.run.precision),
               device=device, precision=config.run.precision, policy_heads=game.policy_heads,
               max_players=game.max_players, **extra)


def _relative(a: float, b: float) -> float:
    return abs(a - b) / max(abs(b), 1e-6)


def test_smoke_config_updates_match_the_reference():
    from card_playing_gym_b200.trainer import device_trainer

    loop, setup, reference_trainer = _reference()
    config = setup.load_config(REFERENCE / "configs" / "plump" / "smoke.toml")
    seed = config.run.seed
    torch.manual_seed(seed)
    np.random.seed(seed)
    random.seed(seed)
    components = setup.build_components(config, device="cpu")
    game = config.game
    cpu = components.trainer
    actor, critic = copy.deepcopy(cpu.actor), copy.deepcopy(cpu.critic)
    cuda = torch.device("cuda")
    gpu_reference = _trainer(reference_trainer.PPOTrainer, actor, critic, components, cuda)
    device = _trainer(device_trainer(reference_trainer.PPOTrainer), actor, critic, components, cuda)
    rng = random.Random(seed)
    worst: dict[str, tuple[float, float]] = {}
    for iteration in range(1, config.run.iterations + 1):
        cpu.actor.eval()
        trajectories = components.collector.collect(game.new_games(rng, iteration))
        components.collector.release()
        sequences = [game.sequences(trajectory) for trajectory in trajectories]
        batch = loop.build_batch(
            trajectories, sequences, max_players=game.max_players, actor_labels=game.actor_labels,
            critic_labels=game.critic_labels, bucket_width=config.ppo.sequence_bucket_width,
            critic_bucket_width=config.ppo.critic_sequence_bucket_width, max_length=game.max_length,
            critic_max_length=game.critic_max_length, min_group_sequences=config.ppo.min_group_sequences)
        gpu_batch, device_batch = copy.deepcopy(batch), copy.deepcopy(batch)
        want = cpu.update(batch, iteration)
        baseline = gpu_reference.update(gpu_batch, iteration)
        got = device.update(device_batch, iteration)
        assert set(got) == set(want), set(got) ^ set(want)
        for key, value in want.items():
            if key in NOT_COMPARED or not np.isfinite(value):
                continue
            ours, theirs = _relative(got[key], value), _relative(baseline[key], value)
            old = worst.get(key, (0.0, 0.0))
            worst[key] = (max(old[0], ours), max(old[1], theirs))
        for head in batch.decisions:
            np.testing.assert_allclose(device_batch.decisions[head].advantages, batch.decisions[head].advantages,
                                       rtol=1e-5, atol=1e-6)
    report = sorted(worst.items(), key=lambda item: -item[1][0])
    print("largest relative deviations from the CPU reference (device trainer, reference on the GPU):")
    for key, (ours, theirs) in report[:12]:
        print(f"  {key}: {ours:.2e}  {theirs:.2e}")
    for key, (ours, theirs) in worst.items():
        assert ours <= max(1e-4, 2.0 * theirs), (key, ours, theirs)
    # Weights after three Adam steps: Adam divides by the root of the second moment, so an entry whose
    # gradient is near zero moves by up to the learning rate on any rounding difference. The bar is the
    # reference's own GPU run.
    for model in ("actor", "critic"):
        states = [getattr(t, model).state_dict() for t in (device, gpu_reference, cpu)]
        for name, ref in states[2].items():
            ours = float((states[0][name].cpu() - ref).abs().max())
            theirs = float((states[1][name].cpu() - ref).abs().max())
            assert ours <= 2.0 * theirs + 1e-6, (model, name, ours, theirs)


def _dp_worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from card_playing_gym_b200.data_parallel import rescale_batch_weights, shard_games
    from card_playing_gym_b200.trainer import device_trainer

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        loop, setup, reference_trainer = _reference()
        config = setup.load_config(REFERENCE / "configs" / "plump" / "smoke.toml")
        torch.manual_seed(0)
        np.random.seed(0)
        random.seed(0)
        components = setup.build_components(config, device="cpu")
        game = config.game
        actor, critic = copy.deepcopy(components.trainer.actor), copy.deepcopy(components.trainer.critic)
        trajectories = components.collector.collect(game.new_games(random.Random(0), 1))
        sequences = [game.sequences(t) for t in trajectories]

        def batch_of(items):
            return loop.build_batch(
                [t for t, _ in items], [s for _, s in items], max_players=game.max_players,
                actor_labels=game.actor_labels, critic_labels=game.critic_labels,
                bucket_width=config.ppo.sequence_bucket_width,
                critic_bucket_width=config.ppo.critic_sequence_bucket_width, max_length=game.max_length,
                critic_max_length=game.critic_max_length, min_group_sequences=config.ppo.min_group_sequences)

        pairs = list(zip(trajectories, sequences))
        starts = np.concatenate([[0], np.cumsum([len(t.decisions) for t in trajectories])])
        g0, g1 = shard_games(starts, world, rank)
        shard = batch_of(pairs[g0:g1])
        rescale_batch_weights(shard, g1 - g0, len(pairs))
        device = torch.device("cuda", rank)
        cls = device_trainer(reference_trainer.PPOTrainer)
        alone = [dist.new_group([r]) for r in range(world)]  # every rank creates every group
        out = {}
        if rank == 0:
            single = _trainer(cls, actor, critic, components, device, process_group=alone[0])
            out["single"] = single.update(batch_of(pairs), 1)
            out["single_weights"] = {k: v.cpu() for k, v in single.actor.state_dict().items()}
        dist.barrier()
        sharded = _trainer(cls, actor, critic, components, device, process_group=dist.group.WORLD)
        out["sharded"] = sharded.update(shard, 1)
        out["sharded_weights"] = {k: v.cpu() for k, v in sharded.actor.state_dict().items()}
        results.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_update_matches_one_process():
    """The same smoke-config batch: one process updating it whole against two NCCL ranks updating halves of its
    trajectories (global decision weights, per-step gradient SUM-allreduce, global normalisation and totals)."""

    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, value = results.get(timeout=600)
            out[rank] = value
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    single, sharded = out[0]["single"], out[0]["sharded"]
    same = {k: v for k, v in sharded.items() if k not in NOT_COMPARED}
    assert {k: v for k, v in out[1]["sharded"].items() if k not in NOT_COMPARED} == same  # the ranks agree
    for key, value in single.items():
        if key in NOT_COMPARED or not np.isfinite(value):
            continue
        assert _relative(sharded[key], value) < 1e-3 or abs(sharded[key] - value) < 1e-6, (key, sharded[key], value)
    for name, want in out[0]["single_weights"].items():
        torch.testing.assert_close(out[0]["sharded_weights"][name], want, rtol=1e-4, atol=2e-6)
        assert torch.equal(out[0]["sharded_weights"][name], out[1]["sharded_weights"][name])
