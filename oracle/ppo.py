"""Numpy restatement of the PPO math on the hot path (oracle only).

Restates cardgym/rl/ppo.py (``ppo_terms`` 28-72, ``masked_probabilities`` 75-82,
``sample_rows`` 85-94, ``center_zero_sum`` 97-108, ``gae_advantages`` 121-144,
``weighted_mean_std`` 147-153) and the trainer steps around them in
cardgym/rl/trainer.py (``_gae`` 634-649, the per-head policy objective of
``_policy_loss`` 733-802, ``_value_loss`` 822-850). Gradients are written out
analytically; tests hold them against the reference's autograd.
"""

from __future__ import annotations

import math

import numpy as np


def masked_probabilities(logits: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """float32 softmax over legal entries; illegal entries exactly zero (ppo.py:75-82).

    Uses numpy's float32 exp and last-axis sum, the operations the reference's
    host sampler runs, so the result is bit-identical to it.
    """

    logits = np.asarray(logits, dtype=np.float32)
    constrained = np.where(mask, logits, np.float32(-np.inf))
    shifted = constrained - constrained.max(axis=-1, keepdims=True)
    weights = np.exp(shifted)
    weights[~mask] = 0.0
    return weights / weights.sum(axis=-1, keepdims=True)


def sample_rows(probabilities: np.ndarray, mask: np.ndarray, uniforms: np.ndarray) -> np.ndarray:
    """Inverse-CDF draw per row, clamped to the last legal index (ppo.py:85-94)."""

    width = probabilities.shape[1]
    below = np.cumsum(probabilities, axis=1) < np.asarray(uniforms, dtype=np.float64)[:, None]
    sampled = below.sum(axis=1)
    last_legal = width - 1 - np.argmax(mask[:, ::-1], axis=1)
    sampled = np.minimum(sampled, last_legal)
    illegal = ~mask[np.arange(len(sampled)), sampled]
    sampled[illegal] = last_legal[illegal]
    return sampled


def boundary_distance(probabilities: np.ndarray, uniforms: np.ndarray) -> np.ndarray:
    """Per row, |cdf_k - u| at the nearest CDF step: how close a draw sits to flipping."""

    cdf = np.cumsum(probabilities, axis=1).astype(np.float64)
    return np.abs(cdf - np.asarray(uniforms, np.float64)[:, None]).min(axis=1)


def center_zero_sum(values: np.ndarray, num_players: np.ndarray) -> np.ndarray:
    """Projection onto the active seats' zero-sum subspace (ppo.py:97-108)."""

    active = np.arange(values.shape[1])[None, :] < np.asarray(num_players)[:, None]
    mean = (values * active).sum(axis=-1, keepdims=True) / np.asarray(num_players, values.dtype)[:, None]
    return (values - mean) * active


def gae_advantages(state_values: np.ndarray, terminal_returns: np.ndarray, gae_lambda: float) -> np.ndarray:
    """Undiscounted GAE over one game's decision states, every seat (ppo.py:121-144).

    running = (next - V[s]) + lambda * running, scanned from the last state back;
    the terminal successor is the realised return.
    """

    advantages = np.zeros_like(state_values)
    next_value = np.asarray(terminal_returns, dtype=state_values.dtype)
    running = np.zeros_like(next_value)
    for index in range(state_values.shape[0] - 1, -1, -1):
        running = (next_value - state_values[index]) + gae_lambda * running
        advantages[index] = running
        next_value = state_values[index]
    return advantages


def segmented_gae(
    values: np.ndarray, seats: np.ndarray, starts: np.ndarray, returns: np.ndarray, gae_lambda: float
) -> np.ndarray:
    """Acting-seat GAE for consecutive game segments (trainer.py:634-649).

    ``values`` [N, P] are each decision state's seat values with every game's
    states contiguous and in decision order; game g owns rows starts[g]:starts[g+1];
    ``returns`` [G, P]. Returns advantages [N] at each row's acting seat.
    """

    out = np.zeros(values.shape[0], dtype=np.float64)
    for game in range(len(starts) - 1):
        lo, hi = int(starts[game]), int(starts[game + 1])
        if hi <= lo:
            continue
        adv = gae_advantages(values[lo:hi].astype(np.float64), returns[game].astype(np.float64), gae_lambda)
        out[lo:hi] = adv[np.arange(hi - lo), seats[lo:hi]]
    return out


def weighted_mean_std(values: np.ndarray, weights: np.ndarray) -> tuple[float, float]:
    """ppo.py:147-153: weighted mean and std with a sqrt(1e-12) floor; (0, 1) without weight."""

    total = float(weights.sum())
    if total <= 0:
        return 0.0, 1.0
    mean = float(np.dot(weights, values) / total)
    variance = float(np.dot(weights, (values - mean) ** 2) / total)
    return mean, math.sqrt(max(variance, 1e-12))


def ppo_terms(logits, old_probs, actions, advantages, clip_ratio: float) -> dict[str, np.ndarray]:
    """Masked PPO terms (ppo.py:28-72), float64; legal actions are those with old_probs > 0."""

    logits = np.asarray(logits, np.float64)
    old = np.asarray(old_probs, np.float64)
    adv = np.asarray(advantages, np.float64)
    rows = np.arange(logits.shape[0])
    legal = old > 0
    masked = np.where(legal, logits, -np.inf)
    peak = masked.max(axis=-1, keepdims=True)
    log_z = np.log(np.exp(masked - peak).sum(axis=-1, keepdims=True)) + peak
    log_probs = np.where(legal, masked - log_z, 0.0)
    old_log = np.log(np.maximum(old, 1e-12))
    ratios = np.exp(log_probs[rows, actions] - old_log[rows, actions])
    clipped_ratios = np.clip(ratios, 1.0 - clip_ratio, 1.0 + clip_ratio)
    losses = -np.minimum(ratios * adv, clipped_ratios * adv)
    divergences = (old * (old_log - log_probs) * legal).sum(axis=-1)
    probabilities = np.exp(log_probs) * legal
    entropy = -(probabilities * log_probs).sum(axis=-1)
    count = legal.sum(axis=-1)
    eligible = count > 1
    normalized = np.where(eligible, entropy / np.log(np.maximum(count, 2)), 0.0)
    return {
        "losses": losses,
        "divergences": divergences,
        "entropy": entropy,
        "normalized_entropy": normalized,
        "entropy_eligible": eligible,
        "log_probs": log_probs,
        "ratios": ratios,
        "clipped": np.abs(ratios - 1.0) > clip_ratio,
        "probabilities": probabilities,
        "legal_count": count,
    }


def policy_objective(logits, old_probs, actions, advantages, weights, clip_ratio: float, alpha: float):
    """The head objective of _policy_loss (trainer.py:774-797) and its gradient w.r.t. logits.

    L = sum_i w_i * loss_i - alpha * sum_i (w_i * eligible_i) * normalized_entropy_i.
    Returns (terms, L, dL/dlogits). The surrogate's gradient follows torch's
    minimum/clamp conventions: inside the clip range both branches tie and the
    gradient is the unclipped one's; outside it, only the selected branch counts.
    """

    t = ppo_terms(logits, old_probs, actions, advantages, clip_ratio)
    adv = np.asarray(advantages, np.float64)
    w = np.asarray(weights, np.float64)
    rows = np.arange(len(adv))
    r = t["ratios"]
    lo, hi = 1.0 - clip_ratio, 1.0 + clip_ratio
    unclipped = r * adv
    clipped = np.clip(r, lo, hi) * adv
    inside = (r >= lo) & (r <= hi)
    # d(-min(rA, clip(r)A))/dr
    d_ratio = np.where(unclipped < clipped, -adv, np.where(unclipped > clipped, -adv * inside, -adv))
    legal = np.asarray(old_probs) > 0
    p = t["probabilities"]
    grad = np.zeros_like(p)
    d_logp_action = w * d_ratio * r
    onehot = np.zeros_like(p)
    onehot[rows, actions] = 1.0
    grad += d_logp_action[:, None] * (onehot - p) * legal
    count = t["legal_count"]
    scale = np.where(t["entropy_eligible"], 1.0 / np.log(np.maximum(count, 2)), 0.0)
    # d H / d z_k = -p_k (log p_k + H)
    d_entropy = -p * (t["log_probs"] + t["entropy"][:, None]) * legal
    grad += (-alpha * w * scale)[:, None] * d_entropy
    objective = float((w * t["losses"]).sum() - alpha * (w * t["entropy_eligible"] * t["normalized_entropy"]).sum())
    return t, objective, grad


def value_loss(prediction, players, targets, weights, reward_scale: float):
    """Dense zero-sum value regression (trainer.py:822-850) and d loss / d prediction.

    loss = sum_i 0.5 * w_i * sum_active ((centered - target) / scale)^2 / players_i.
    Returns (loss, squared_error_total, grad [N, P]).
    """

    pred = np.asarray(prediction, np.float64)
    n = np.asarray(players, np.int64)
    tgt = np.asarray(targets, np.float64)
    w = np.asarray(weights, np.float64)
    active = (np.arange(pred.shape[1])[None, :] < n[:, None]).astype(np.float64)
    centered = center_zero_sum(pred, n)
    raw = centered - tgt
    error = raw / reward_scale
    loss = float((0.5 * w * (error * error * active).sum(-1) / n).sum())
    squared = float(((w / n) * (raw * raw * active).sum(-1)).sum())
    g = (w / n)[:, None] * error / reward_scale * active  # d loss / d centered
    grad = active * (g - (g * active).sum(-1, keepdims=True) / n[:, None])
    return loss, squared, grad


def seat_values(values: np.ndarray, shift: np.ndarray, players: np.ndarray, seat: np.ndarray,
                center: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """Per-decision seat values and the prediction, as PPOTrainer._baseline / _recorded_values compute them.

    center=False (trainer.py:556-571): the stream's values [N, P] (already zero-sum centred float32), absolute
    seat i read from column (i - shift) mod players, inactive seats zero; prediction = the acting seat's entry.
    center=True (trainer.py:610-632): recorded raw values centred over the active seats in float64, state
    columns (i - shift) mod players of the centred row, prediction = centred column 0.
    Returns float64 (state [N, P], prediction [N]).
    """

    values = np.asarray(values)
    players = np.asarray(players, np.int64)
    count = values.shape[1]
    seats = np.arange(count)[None, :]
    active = seats < players[:, None]
    columns = (seats - np.asarray(shift, np.int64)[:, None]) % players[:, None]
    if center:
        raw = values.astype(np.float64) * active
        centred = (raw - raw.sum(-1, keepdims=True) / players[:, None]) * active
        state = np.take_along_axis(centred, columns, axis=1) * active
        return state, centred[:, 0]
    state = (np.take_along_axis(values, columns, axis=1) * active).astype(np.float64)
    return state, state[np.arange(len(state)), np.asarray(seat, np.int64)]
