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


def _trainer(cls, actor, critic, components, device):
    config = components.config
    game = config.game
    return cls(copy.deepcopy(actor), copy.deepcopy(critic), config.ppo, game.hooks(device, config.run.precision),
               device=device, precision=config.run.precision, policy_heads=game.policy_heads,
               max_players=game.max_players)


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
