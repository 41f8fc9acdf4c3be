"""Parity at the benchmarked configurations themselves (B200 only).

bench.py times the rl-v6 rollout wave at 4,096 concurrent 4-player games (16,384 KV rows,
lengths U[16, 256], fp16 KV, bf16 GEMM operands) and the PPO advantage + loss step on a
262,144-decision batch with 52-way masks. These tests run exactly those workloads (the
bench's own input builders) and hold the outputs to the oracle:

* the wave: 512 readout rows (the 256 longest streams and 256 others, both heads) through
  the oracle's ragged decode from the same KV pool contents, at the kernels' rounding points
  (bf16 mode) or in fp32 (fp32 mode, fp32 KV); hidden states, both heads' logits and the
  values; the draws bit-exact with numpy's sampler on the kernel's logits;
* the PPO step: GAE bit-exact (float64, the reference's operation order), the global
  normalisation, the fused objective with its gradient and every reporting total, and the
  value loss with its gradient, against the float64 oracle.

Errors are max |got - expected| / max |expected| per tensor.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle import plump as oplump
from oracle import ppo as oppo
from oracle.trunk import Precision

pytestmark = pytest.mark.gpu

GAMES, MIN_LEN, MAX_LEN = 4096, 16, 256
CHECKED_ROWS = 512
ORACLE_BATCH = 128
# bf16 mode, at the oracle's own rounding points (bf16 GEMM operands, fp16 K/V/q/probabilities):
# the kernels differ from it only in the order of fp32 sums (tensor-core accumulation, the online
# softmax), and a last-bit fp32 difference can flip one bf16 rounding of an operand. Measured on
# a B200: hidden 7.6e-4, bid / play logits and values 7.2e-4 to 7.4e-4 (fp32 mode: 4.4e-7 to 6.5e-7).
BF16_HIDDEN_TOL = 1e-3
BF16_LOGIT_TOL = 1e-3
FP32_TOL = 1e-5


def scaled_error(got: np.ndarray, expected: np.ndarray) -> float:
    return float(np.abs(got - expected).max() / max(np.abs(expected).max(), 1e-30))


def _oracle_config(config) -> dict:
    return {k: getattr(config, k) for k in ("d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff", "per_layer_dim",
                                            "value_embeddings", "max_players", "max_hand_size")}


def _checked_readouts(wave: dict) -> np.ndarray:
    """Indices of the readouts (games) to check: the longest 256 streams and 256 others, both heads."""

    lengths = wave["lengths"]
    longest = np.argsort(-lengths, kind="stable")[: CHECKED_ROWS // 2]
    rest = np.setdiff1d(np.arange(GAMES), longest)
    others = np.random.default_rng(99).choice(rest, CHECKED_ROWS - len(longest), replace=False)
    chosen = np.sort(np.concatenate([longest, others]))
    assert set(wave["heads"][chosen]) == {0, 1}
    return chosen


@pytest.mark.parametrize("precision,kv", [("bf16", "fp16"), ("fp32", "fp32")])
def test_rlv6_bench_wave_matches_the_oracle(precision, kv):
    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    device = torch.device("cuda")
    config = PlumpModelConfig()
    state = synthetic_plump_actor_state(config, seed=1)
    actor = PlumpActor(config, state, device=device, precision=precision)
    wave = bench.synthetic_wave(GAMES, MIN_LEN, MAX_LEN, seed=1000)
    rows = 4 * GAMES
    dtype = {"fp16": torch.float16, "fp32": torch.float32}[kv]
    cache = actor.new_cache(rows + 1, MAX_LEN + 1, dtype)
    generator = torch.Generator(device=device).manual_seed(17)
    for pool in (cache.k_pool, cache.v_pool):
        for layer in range(pool.shape[0]):
            pool[layer].normal_(generator=generator)
    chosen = _checked_readouts(wave)
    cache_rows = wave["readout_rows"][chosen]
    index = torch.from_numpy(cache_rows).to(device)
    # The pool contents the checked rows decode against, before the wave appends to them.
    k_before = cache.k_pool.index_select(1, index).float().cpu().numpy()
    v_before = cache.v_pool.index_select(1, index).float().cpu().numpy()

    dev = {k: torch.from_numpy(v).to(device) for k, v in wave.items()}
    hidden = actor.forward_ragged(dev["tokens"], dev["positions"], cache, dev["offsets"], span=MAX_LEN + 1)
    logits, probs, actions, values = actor.decide(hidden, dev["heads"], dev["legal"], dev["uniforms"],
                                                  dev["readout_rows"])
    got_hidden = hidden.index_select(0, index).cpu().numpy()
    logits, probs, actions, values = (t.cpu().numpy()[chosen] for t in (logits, probs, actions, values))

    oracle = oplump.PlumpActor(state, _oracle_config(config), Precision(gemm=precision, kv=kv))
    expected_hidden = np.zeros_like(got_hidden, dtype=np.float64)
    for at in range(0, len(chosen), ORACLE_BATCH):
        part = slice(at, at + ORACLE_BATCH)
        count = len(cache_rows[part])
        ocache = oracle.new_cache(count, MAX_LEN + 1)
        ocache.k[:] = k_before[:, part]
        ocache.v[:] = v_before[:, part]
        expected_hidden[part] = oracle.forward_ragged(wave["tokens"][cache_rows[part]].astype(np.int64),
                                                      wave["positions"][cache_rows[part]], ocache,
                                                      wave["offsets"][cache_rows[part]], span=MAX_LEN + 1)
    heads = wave["heads"][chosen]
    errors = {"hidden": scaled_error(got_hidden, expected_hidden)}
    for head, (name, width) in enumerate((("bid", 11), ("play", 52))):
        sel = heads == head
        expected = oracle.heads.policy_logits(expected_hidden[sel], name)
        errors[name] = scaled_error(logits[sel, :width], expected)
    errors["values"] = scaled_error(values, oracle.heads.player_values(expected_hidden))
    print(f"rl-v6 bench wave, {precision} / {kv} KV, {len(chosen)} readouts: "
          + ", ".join(f"{k} {v:.3e}" for k, v in errors.items()))
    if precision == "fp32":
        assert max(errors.values()) < FP32_TOL, errors
    else:
        assert errors["hidden"] < BF16_HIDDEN_TOL, errors
        assert max(errors["bid"], errors["play"], errors["values"]) < BF16_LOGIT_TOL, errors

    # The draws: numpy's sampler over each head's own width, on the kernel's logits, bit for bit.
    legal = wave["legal"][chosen].astype(bool)
    uniforms = wave["uniforms"][chosen]
    for head, width in ((0, 11), (1, 52)):
        sel = heads == head
        expected_probs = oppo.masked_probabilities(logits[sel, :width], legal[sel, :width])
        assert np.array_equal(probs[sel, :width].view(np.uint32), expected_probs.view(np.uint32))
        assert np.array_equal(actions[sel], oppo.sample_rows(expected_probs, legal[sel, :width], uniforms[sel]))


def test_ppo_step_at_the_bench_batch_matches_the_oracle():
    from card_playing_gym_b200 import ppo
    from card_playing_gym_b200.data_parallel import normalize_global_

    device = torch.device("cuda")
    batch = bench.synthetic_ppo_batch(262_144, seed=5)
    to = lambda a, dtype=None: torch.as_tensor(np.ascontiguousarray(a)).to(device=device, dtype=dtype)  # noqa: E731
    advantages = ppo.segmented_gae(to(batch["values"], torch.float64), to(batch["seats"], torch.int32),
                                   to(batch["starts"]), to(batch["returns"], torch.float64), 0.95)
    expected_adv = oppo.segmented_gae(batch["values"], batch["seats"], batch["starts"], batch["returns"], 0.95)
    assert np.array_equal(advantages.cpu().numpy(), expected_adv)

    weights = batch["weights"]
    normalize_global_(advantages, to(weights, torch.float64))
    mean, std = oppo.weighted_mean_std(expected_adv, weights)
    normalized = (expected_adv - mean) / std
    assert scaled_error(advantages.cpu().numpy(), normalized) < 1e-12

    leaf = to(batch["logits"]).requires_grad_()
    objective, totals = ppo.policy_objective(leaf, to(batch["old_probs"]), to(batch["actions"]),
                                             advantages.float(), to(weights, torch.float32), clip_ratio=0.2,
                                             alpha=0.01)
    objective.backward()
    adv32 = normalized.astype(np.float32)
    terms, expected_objective, expected_grad = oppo.policy_objective(
        batch["logits"], batch["old_probs"], batch["actions"], adv32, weights.astype(np.float32), 0.2, 0.01)
    w = weights.astype(np.float32).astype(np.float64)
    expected_totals = {
        "policy_loss": float((w * terms["losses"]).sum()),
        "row_weight": float(w.sum()),
        "entropy_raw": float((w * terms["entropy"]).sum()),
        "entropy": float((w * terms["entropy_eligible"] * terms["normalized_entropy"]).sum()),
        "entropy_weight": float((w * terms["entropy_eligible"]).sum()),
        "clip": float((w * terms["clipped"]).sum()),
        "behavior_kl": float((w * terms["divergences"]).sum()),
        "objective": expected_objective,
    }
    got_totals = dict(zip(ppo.TOTAL_KEYS, totals.tolist()))
    relative = {k: abs(got_totals[k] - v) / max(abs(v), 1e-30) for k, v in expected_totals.items()}
    grad_error = scaled_error(leaf.grad.cpu().numpy(), expected_grad)
    print("PPO objective at 262,144 x 52: gradient", f"{grad_error:.3e};",
          ", ".join(f"{k} {v:.3e}" for k, v in relative.items()))
    assert abs(objective.item() - expected_objective) <= 1e-5 * abs(expected_objective)
    assert grad_error < 1e-5
    for key, value in relative.items():
        if key == "clip":  # a sum of weights over rows whose ratio crosses 1 +- clip: counts must agree
            assert value < 1e-5 or abs(got_totals[key] - expected_totals[key]) <= 2 * float(w.max())
        else:
            assert value < 1e-5, (key, value)

    players = np.full(len(weights), bench.PPO_PLAYERS, dtype=np.int32)
    prediction = to(batch["prediction"]).requires_grad_()
    loss, value_totals = ppo.value_loss(prediction, to(players), to(batch["targets"]), to(weights, torch.float32),
                                        1.0)
    loss.backward()
    expected_loss, expected_squared, expected_value_grad = oppo.value_loss(
        batch["prediction"], players, batch["targets"], weights.astype(np.float32), 1.0)
    assert abs(loss.item() - expected_loss) <= 1e-5 * abs(expected_loss)
    assert abs(value_totals[1].item() - expected_squared) <= 1e-5 * abs(expected_squared)
    assert scaled_error(prediction.grad.cpu().numpy(), expected_value_grad) < 1e-5
