"""PPO advantage and loss step on the B200.

Reference interfaces (cardgym/rl/ppo.py, cardgym/rl/trainer.py):

* ``gae_advantages(state_values, terminal_returns, gae_lambda)`` (ppo.py:121-144) and the
  trainer's per-game loop ``PPOTrainer._gae`` (trainer.py:634-649) become one segmented
  kernel, ``segmented_gae``, over every game of the batch.
* ``weighted_mean_std`` (ppo.py:147-153) keeps its two-pass definition.
* ``ppo_terms`` (ppo.py:28-72) returns the same ``PPOTerms`` fields.
* ``policy_objective`` is the per-head objective of ``_policy_loss`` (trainer.py:774-797),
  ``sum w * loss - alpha * sum w * eligible * normalized_entropy``, as one fused kernel
  that also writes dL/dlogits; wrapped in ``torch.autograd.Function`` so the trainer's
  separate policy/auxiliary backward passes (trainer.py:866-895) keep working.
* ``value_loss`` is ``_value_loss`` (trainer.py:822-850) with its gradient.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _native as nat


# -- GAE ------------------------------------------------------------------------------------
def segmented_gae(values: torch.Tensor, seats: torch.Tensor, starts: torch.Tensor, returns: torch.Tensor,
                  gae_lambda: float) -> torch.Tensor:
    """Acting-seat GAE for every game: values f64 [N, P] (game g = rows starts[g]:starts[g+1], decision
    order), seats [N], returns f64 [G, P] -> advantages f64 [N]."""

    values = values.to(torch.float64).contiguous()
    returns = returns.to(torch.float64).contiguous()
    players = values.shape[1]
    games = starts.shape[0] - 1
    out = torch.zeros(values.shape[0], dtype=torch.float64, device=values.device)
    nat.call("cg_gae_segments", nat.ptr(values), players, nat.ptr(seats.to(torch.int32).contiguous()),
             nat.ptr(starts.to(torch.int64).contiguous()), games, nat.ptr(returns), float(gae_lambda), nat.ptr(out),
             nat.stream_handle(values.device))
    return out


def gae_advantages(state_values: torch.Tensor, terminal_returns: torch.Tensor, gae_lambda: float) -> torch.Tensor:
    """One game's GAE for every seat, [S, P] (the reference signature, ppo.py:121-144)."""

    states, players = state_values.shape
    device = state_values.device
    starts = torch.tensor([0, states], dtype=torch.int64, device=device)
    columns = []
    for seat in range(players):
        seats = torch.full((states,), seat, dtype=torch.int32, device=device)
        columns.append(segmented_gae(state_values, seats, starts, terminal_returns.reshape(1, players), gae_lambda))
    return torch.stack(columns, dim=1)


# -- normalisation ---------------------------------------------------------------------------
def weighted_sums(values: torch.Tensor, weights: torch.Tensor, shift: float = 0.0) -> torch.Tensor:
    """(sum w, sum w (x - shift), sum w (x - shift)^2) in float64, deterministic."""

    values = values.to(torch.float64).contiguous()
    weights = weights.to(torch.float64).contiguous()
    n = values.numel()
    out = torch.empty(3, dtype=torch.float64, device=values.device)
    need = nat.query("cg_weighted_sums_workspace_bytes", n)
    workspace = nat.Workspace.get(values.device, need, "reduce")
    nat.call("cg_weighted_sums", nat.ptr(values), nat.ptr(weights), n, float(shift), nat.ptr(out), nat.ptr(workspace),
             workspace.numel(), nat.stream_handle(values.device))
    return out


def weighted_sums_shifted(values: torch.Tensor, weights: torch.Tensor, shift_sums: torch.Tensor) -> torch.Tensor:
    """The second pass with its shift (the mean of a first pass's sums) read on the device."""

    values = values.to(torch.float64).contiguous()
    weights = weights.to(torch.float64).contiguous()
    n = values.numel()
    out = torch.empty(3, dtype=torch.float64, device=values.device)
    need = nat.query("cg_weighted_sums_workspace_bytes", n)
    workspace = nat.Workspace.get(values.device, need, "reduce")
    nat.call("cg_weighted_sums_shifted", nat.ptr(values), nat.ptr(weights), n, nat.ptr(shift_sums.contiguous()),
             nat.ptr(out), nat.ptr(workspace), workspace.numel(), nat.stream_handle(values.device))
    return out


def normalize_from_sums_(values: torch.Tensor, first: torch.Tensor, second: torch.Tensor) -> torch.Tensor:
    """normalize_ with mean and std computed on the device from both passes' sums (no host read)."""

    if values.dtype != torch.float64 or not values.is_contiguous():
        raise ValueError("normalize_from_sums_ works in place on a contiguous float64 tensor")
    nat.call("cg_normalize_from_sums", nat.ptr(values), values.numel(), nat.ptr(first.contiguous()),
             nat.ptr(second.contiguous()), nat.stream_handle(values.device))
    return values


def mean_std_from_sums(total: float, weighted: float, second: float | None = None) -> tuple[float, float]:
    """weighted_mean_std's arithmetic on reduced sums (ppo.py:147-153)."""

    if total <= 0:
        return 0.0, 1.0
    mean = weighted / total
    if second is None:
        return mean, float("nan")
    return mean, math.sqrt(max(second / total, 1e-12))


def weighted_mean_std(values: torch.Tensor, weights: torch.Tensor) -> tuple[float, float]:
    first = weighted_sums(values, weights).tolist()
    mean, _ = mean_std_from_sums(first[0], first[1])
    if first[0] <= 0:
        return 0.0, 1.0
    second = weighted_sums(values, weights, shift=mean).tolist()
    return mean_std_from_sums(first[0], first[1], second[2])


def normalize_(values: torch.Tensor, mean: float, std: float) -> torch.Tensor:
    """values <- (values - mean) / std in place (float64)."""

    if values.dtype != torch.float64 or not values.is_contiguous():
        raise ValueError("normalize_ works in place on a contiguous float64 tensor")
    nat.call("cg_normalize", nat.ptr(values), values.numel(), float(mean), float(std), nat.stream_handle(values.device))
    return values


# -- PPO objective ------------------------------------------------------------------------------
@dataclass
class PPOTerms:
    losses: torch.Tensor
    divergences: torch.Tensor
    entropy: torch.Tensor
    normalized_entropy: torch.Tensor
    entropy_eligible: torch.Tensor
    log_probs: torch.Tensor | None
    ratios: torch.Tensor
    clipped: torch.Tensor
    action_log_probs: torch.Tensor


TOTAL_KEYS = ("policy_loss", "row_weight", "entropy_raw", "entropy", "entropy_weight", "clip", "behavior_kl", "objective")


def _run_objective(logits, old_probs, actions, advantages, weights, clip, alpha, want_grad: bool, want_terms: bool):
    rows, width = logits.shape
    logits = logits.float().contiguous()
    old_probs = old_probs.float().contiguous()
    device = logits.device
    dlogits = torch.empty_like(logits) if want_grad else None
    terms = torch.empty((rows, 8), device=device) if want_terms else None
    totals = torch.empty(8, dtype=torch.float64, device=device)
    need = nat.query("cg_ppo_objective_workspace_bytes", rows)
    workspace = nat.Workspace.get(device, need, "reduce")
    nat.call("cg_ppo_objective", nat.ptr(logits), nat.ptr(old_probs), rows, width, width,
             nat.ptr(actions.to(torch.int64).contiguous()), nat.ptr(advantages.float().contiguous()),
             nat.ptr(weights.float().contiguous()), float(clip), float(alpha), nat.ptr(dlogits), nat.ptr(terms),
             nat.ptr(totals), nat.ptr(workspace), workspace.numel(), nat.stream_handle(device))
    return dlogits, terms, totals


class _PolicyObjective(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, old_probs, actions, advantages, weights, clip, alpha):
        dlogits, _, totals = _run_objective(logits, old_probs, actions, advantages, weights, clip, alpha,
                                            want_grad=logits.requires_grad, want_terms=False)
        ctx.save_for_backward(dlogits if dlogits is not None else torch.empty(0, device=logits.device))
        ctx.mark_non_differentiable(totals)
        return totals[7].to(torch.float32), totals

    @staticmethod
    def backward(ctx, grad_objective, _grad_totals):
        (dlogits,) = ctx.saved_tensors
        return dlogits * grad_objective, None, None, None, None, None, None


def policy_objective(logits: torch.Tensor, old_probs: torch.Tensor, actions: torch.Tensor, advantages: torch.Tensor,
                     weights: torch.Tensor, *, clip_ratio: float, alpha: float):
    """The fused per-head PPO objective and its reporting totals.

    Returns (objective, totals): objective is a differentiable fp32 scalar
    ``sum w loss - alpha sum w eligible normalized_entropy``; totals is float64 [8] in
    ``TOTAL_KEYS`` order (the trainer's totals of trainer.py:786-795).
    """

    return _PolicyObjective.apply(logits, old_probs, actions, advantages, weights, float(clip_ratio), float(alpha))


def ppo_terms(logits: torch.Tensor, old_probs: torch.Tensor, actions: torch.Tensor, advantages: torch.Tensor, *,
              clip_ratio: float) -> PPOTerms:
    """Masked PPO terms per row (ppo.py:28-72); computed, not differentiable (use policy_objective).

    The per-row terms come from the fused kernel. ``log_probs`` [N, A] (log pi over the legal actions,
    0 elsewhere), which only the reference's gated-head entropies read, is torch's masked log_softmax,
    as the reference computes it.
    """

    rows = logits.shape[0]
    weights = torch.zeros(rows, device=logits.device)
    _, terms, _ = _run_objective(logits.detach(), old_probs, actions, advantages, weights, clip_ratio, 0.0,
                                 want_grad=False, want_terms=True)
    legal = old_probs > 0
    masked = logits.detach().float().masked_fill(~legal, float("-inf"))
    log_probs = torch.where(legal, torch.log_softmax(masked, dim=-1), torch.zeros((), device=logits.device))
    return PPOTerms(
        losses=terms[:, 0], divergences=terms[:, 1], entropy=terms[:, 2], normalized_entropy=terms[:, 3],
        entropy_eligible=terms[:, 4] > 0, log_probs=log_probs, ratios=terms[:, 5], clipped=terms[:, 6] > 0,
        action_log_probs=terms[:, 7],
    )


# -- value loss ----------------------------------------------------------------------------------
class _ValueLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, prediction, targets, players, weights, scale):
        rows, width = prediction.shape
        prediction = prediction.float().contiguous()
        device = prediction.device
        grad = torch.empty_like(prediction) if ctx.needs_input_grad[0] else None
        totals = torch.empty(4, dtype=torch.float64, device=device)
        need = nat.query("cg_value_loss_workspace_bytes", rows)
        workspace = nat.Workspace.get(device, need, "reduce")
        nat.call("cg_value_loss", nat.ptr(prediction), nat.ptr(targets.float().contiguous()),
                 nat.ptr(players.to(torch.int32).contiguous()), nat.ptr(weights.float().contiguous()), rows, width,
                 float(scale), nat.ptr(grad), nat.ptr(totals), nat.ptr(workspace), workspace.numel(),
                 nat.stream_handle(device))
        ctx.save_for_backward(grad if grad is not None else torch.empty(0, device=device))
        ctx.mark_non_differentiable(totals)
        return totals[0].to(torch.float32), totals

    @staticmethod
    def backward(ctx, grad_loss, _grad_totals):
        (grad,) = ctx.saved_tensors
        return grad * grad_loss, None, None, None, None


def value_loss(prediction: torch.Tensor, players: torch.Tensor, targets: torch.Tensor, weights: torch.Tensor,
               reward_scale: float):
    """Dense zero-sum value regression (trainer.py:822-850). Returns (loss, totals f64 [4]:
    loss, sum w/n sum raw^2, sum w/n sum target^2, sum w)."""

    return _ValueLoss.apply(prediction, targets, players, weights, float(reward_scale))


# -- baseline seat values -------------------------------------------------------------------------
def seat_values(values: torch.Tensor, shift: torch.Tensor, players: torch.Tensor, seat: torch.Tensor,
                flat: torch.Tensor | None = None, *, center: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Each decision's per-seat state values and its prediction (trainer.py:556-571, 610-632).

    values fp32 [M, P]; decision i reads row ``flat[i]`` (or i). Absolute seat s is column
    ``(s - shift[i]) mod players[i]``; seats past ``players[i]`` are zero. ``center=False``: the values
    are already zero-sum centred and the prediction is the acting seat's entry; ``center=True``: raw
    recorded values, centred over the active seats in float64, prediction = centred column 0.
    Returns (state f64 [N, P], prediction f64 [N]).
    """

    values = values.float().contiguous()
    count = shift.shape[0]
    seats = values.shape[1]
    state = torch.empty((count, seats), dtype=torch.float64, device=values.device)
    prediction = torch.empty(count, dtype=torch.float64, device=values.device)
    as64 = lambda t: t.to(device=values.device, dtype=torch.int64).contiguous()  # noqa: E731
    nat.call("cg_seat_values", nat.ptr(values), values.shape[0], seats, nat.ptr(None if flat is None else as64(flat)),
             nat.ptr(as64(shift)), nat.ptr(as64(players)), nat.ptr(as64(seat)), count, 1 if center else 0,
             nat.ptr(state), nat.ptr(prediction), nat.stream_handle(values.device))
    return state, prediction


def center_zero_sum(values: torch.Tensor, num_players: torch.Tensor) -> torch.Tensor:
    """Projection onto the active seats' zero-sum subspace, padded seats zero (ppo.py:97-108); fp32."""

    values = values.float().contiguous()
    out = torch.empty_like(values)
    nat.call("cg_center_zero_sum", nat.ptr(values), nat.ptr(num_players.to(torch.int64).contiguous()),
             values.shape[0], values.shape[1], nat.ptr(out), nat.stream_handle(values.device))
    return out


# -- one captured step ------------------------------------------------------------------------
class GraphedStep:
    """A fixed-shape step captured once as a CUDA graph and replayed (the update's advantage +
    loss step is a few dozen short kernels; replayed, it costs its device time, not its launches).

    ``fn`` takes no arguments; the tensors it reads and writes must keep their storage between
    calls (refill inputs in place). Every call returns what ``fn`` returned on the capture: the
    same tensors, rewritten by the replay. The first call runs ``fn`` ``warmup`` times on a side
    stream, so that every kernel and library workspace is configured at its final size before
    the capture, then captures and replays it. Collectives belong outside the captured step.
    """

    def __init__(self, fn, warmup: int = 2) -> None:
        self.fn = fn
        self.warmup = warmup
        self.graph: torch.cuda.CUDAGraph | None = None
        self.outputs = None

    def __call__(self):
        if self.graph is None:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(self.warmup):
                    self.fn()
            torch.cuda.current_stream().wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.outputs = self.fn()
        self.graph.replay()
        return self.outputs
