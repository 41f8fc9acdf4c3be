"""Data-parallel PPO update: trajectory shards, batch-global statistics, gradient allreduce.

Self-play needs no collective: every rank runs its own games, KV pool and seed. The PPO
update of cardgym/rl/trainer.py:430-520 runs on one process in the reference; sharded over
ranks it needs these exchanges per optimizer step, and nothing else:

* the advantage normalisation's batch-global weighted mean and std (trainer.py:601-607 with
  ppo.py:147-153): two allreduces of three float64 sums, keeping the reference's two-pass
  definition (mean first, then the centred second moment);
* the entropy controller's observed per-head entropy (rl/entropy.py:51-69): per head,
  (sum w * H_norm, sum w) summed over ranks;
* the gradients, SUM-reduced once per optimizer step after its last backward (the decision
  weights already divide by the global game and seat counts, so per-rank gradients are
  partial sums of the global objective's gradient). Under the auxiliary budget
  (trainer.py:897-937) the policy and auxiliary stashes, which both span every actor
  parameter, are reduced separately, because one is scaled against the other's global norm.

Shards are whole trajectories (GAE segments never cross ranks), contiguous in decision
order and balanced by decision count. The collectives run on the process group given
(NCCL on the GPUs; gloo works the same for host tensors).
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Sequence

import numpy as np
import torch
import torch.distributed as dist

from .ppo import mean_std_from_sums, normalize_from_sums_, weighted_sums, weighted_sums_shifted


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


# -- shards ------------------------------------------------------------------------------------
def shard_games(starts: Sequence[int] | torch.Tensor, world_size: int, rank: int) -> tuple[int, int]:
    """Game range [g0, g1) of `rank`: whole games, contiguous, balanced by decision count.

    `starts` holds G + 1 decision offsets (game g owns decisions starts[g]:starts[g+1]).
    Rank r takes the games whose first decision lies in [N r / W, N (r + 1) / W), so every
    game lands on exactly one rank and shards differ by at most one game's length.
    """

    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside a world of {world_size}")
    bounds = torch.as_tensor(starts, dtype=torch.int64).cpu()
    if bounds.ndim != 1 or bounds.numel() < 1 or bool((bounds[1:] < bounds[:-1]).any()):
        raise ValueError("starts must be a non-decreasing vector of G + 1 offsets")
    games = bounds.numel() - 1
    total = int(bounds[-1] - bounds[0])

    def edge(r: int) -> int:
        if r <= 0:
            return 0
        if r >= world_size:
            return games
        target = int(bounds[0]) + (total * r) // world_size
        return int(torch.searchsorted(bounds[:-1], torch.tensor(target), right=False))

    return edge(rank), edge(rank + 1)


def rescale_batch_weights(batch, local_games: int, global_games: int) -> None:
    """Give a rank's batch the global decision weights, in place.

    The reference's batch builder weighs every decision row and dense position by 1 / G of the
    games it was given (cardgym/rl/batch.py:147-178). A rank built from its shard of G_r of the G
    games scales them by G_r / G, so that the ranks' weights (and their SUM-reduced gradients) are
    the whole batch's.
    """

    if local_games == global_games:
        return
    scale = np.float32(local_games / global_games)
    for rows in batch.decisions.values():
        rows.weight *= scale
    for group in [*batch.actor_groups, *batch.critic_groups]:
        group.position_weight *= scale


# -- batch-global statistics ---------------------------------------------------------------------
def allreduce_sums(sums: torch.Tensor, group=None) -> torch.Tensor:
    """SUM-allreduce of a small float64 vector of partial sums (in place; returned)."""

    if _world(group)[1] > 1:
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    return sums


def global_weighted_mean_std(values: torch.Tensor, weights: torch.Tensor, group=None,
                             sums: Callable[..., torch.Tensor] = weighted_sums) -> tuple[float, float]:
    """weighted_mean_std (ppo.py:147-153) over the union of every rank's shard.

    Pass 1 reduces (sum w, sum w x), pass 2 the centred (sum w (x - mean)^2): the same
    two-pass arithmetic as the reference on one process. `sums(values, weights, shift)`
    returns a float64 tensor (sum w, sum w (x - shift), sum w (x - shift)^2) for the local
    shard; by default the device reduction kernel.
    """

    first = allreduce_sums(sums(values, weights, 0.0).to(torch.float64), group).tolist()
    if first[0] <= 0:
        return 0.0, 1.0
    mean, _ = mean_std_from_sums(first[0], first[1])
    second = allreduce_sums(sums(values, weights, mean).to(torch.float64), group).tolist()
    return mean_std_from_sums(first[0], first[1], second[2])


def normalize_global_(values: torch.Tensor, weights: torch.Tensor, group=None) -> torch.Tensor:
    """global_weighted_mean_std + normalize_ with no host read: both passes' sums stay on the
    device and are allreduced there (NCCL), so the step can run ahead of the host or inside a
    CUDA graph. Bit-identical to the host-read path (the same float64 arithmetic)."""

    first = allreduce_sums(weighted_sums(values, weights, 0.0), group)
    second = allreduce_sums(weighted_sums_shifted(values, weights, first), group)
    return normalize_from_sums_(values, first, second)


def allreduce_head_entropy(observed: torch.Tensor, group=None) -> torch.Tensor:
    """Per-head (sum w * normalized entropy, sum w) [heads, 2] summed over ranks, then the
    observed entropy per head (sum / weight; 0 where a head saw no weight)."""

    totals = allreduce_sums(observed.to(torch.float64).clone(), group)
    weight = totals[:, 1]
    return torch.where(weight > 0, totals[:, 0] / weight.clamp_min(1e-300), torch.zeros_like(weight))


# -- gradients ------------------------------------------------------------------------------------
class GradientAllreduce:
    """SUM-allreduce of one parameter list's gradients, once per optimizer step, in flat buckets.

    The reference trainer accumulates many backward passes into one optimizer step: one per
    microbatch of every sequence group (trainer.py:700-731), either into ``.grad`` or, under the
    auxiliary budget, into two stashes of ``torch.autograd.grad`` results (trainer.py:866-895).
    The gradients are therefore reduced as they stand after the last of those passes, by an
    explicit call: ``reduce_grads()`` for ``.grad``, ``reduce_(stash)`` for a stash (a list
    aligned with ``params``).

    A parameter that no pass reached has no gradient (``None``); what one rank's shard reached
    another's may not have. One small MAX-allreduce of per-parameter presence flags goes first,
    so every rank flattens the same parameters into the same buckets: a gradient present on any
    rank is summed (ranks without one contribute zeros), one present on none stays ``None``
    (so Adam still skips it, as on one process). Buckets (reverse parameter order, at most
    ``bucket_bytes``) are all launched asynchronously before the first is waited on, so their
    transfers overlap each other's flattening and unflattening. Reduced values are written back
    into the existing gradient tensors, so other references to them see the sums.
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], group=None, bucket_bytes: int = 32 << 20):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.bucket_bytes = int(bucket_bytes)

    @property
    def world_size(self) -> int:
        return _world(self.group)[1]

    def _present(self, grads: Sequence[torch.Tensor | None]) -> list[bool]:
        flags = torch.tensor([g is not None for g in grads], dtype=torch.int32,
                             device=self.params[0].device if self.params else "cpu")
        if self.world_size > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.group)
        return [bool(v) for v in flags.tolist()]

    def _buckets(self, present: list[bool]) -> list[list[int]]:
        buckets: list[list[int]] = []
        current: list[int] = []
        size = 0
        for index in reversed(range(len(self.params))):
            if not present[index]:
                continue
            p = self.params[index]
            nbytes = p.numel() * p.element_size()
            if current and size + nbytes > self.bucket_bytes:
                buckets.append(current)
                current, size = [], 0
            current.append(index)
            size += nbytes
        if current:
            buckets.append(current)
        return buckets

    def reduce_(self, grads: Sequence[torch.Tensor | None] | None) -> list[torch.Tensor | None] | None:
        """Sum ``grads`` (aligned with ``params``; None entries allowed) over the ranks.

        Returns the list of summed gradients: the same tensor objects where this rank had one,
        new tensors where only other ranks did, None where no rank did. ``None`` in place of the
        whole list (a stash that received nothing on this rank) is treated as all-None; it comes
        back as None only if every rank's was empty.
        """

        empty = grads is None
        grads = [None] * len(self.params) if grads is None else list(grads)
        if len(grads) != len(self.params):
            raise ValueError(f"{len(grads)} gradients for {len(self.params)} parameters")
        present = self._present(grads)
        if not any(present):
            return None if empty else grads
        if self.world_size == 1:
            return grads
        launched = []
        for bucket in self._buckets(present):
            parts = [grads[i] if grads[i] is not None else torch.zeros_like(self.params[i]) for i in bucket]
            flat = torch.cat([part.reshape(-1) for part in parts])
            work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            launched.append((bucket, flat, work))
        for bucket, flat, work in launched:
            work.wait()
            at = 0
            for index in bucket:
                p = self.params[index]
                value = flat[at:at + p.numel()].view_as(p)
                at += p.numel()
                if grads[index] is None:
                    grads[index] = value.clone()
                else:
                    grads[index].copy_(value)
        return grads

    def reduce_grads(self) -> None:
        """Sum every parameter's ``.grad`` over the ranks, after the step's last backward."""

        reduced = self.reduce_([p.grad for p in self.params])
        if reduced is None:
            return
        for p, g in zip(self.params, reduced):
            if p.grad is None and g is not None:
                p.grad = g


def global_grad_norm(params: Iterable[torch.nn.Parameter]) -> torch.Tensor:
    """L2 norm of the (already reduced) gradients, as clip_grad_norm computes it (trainer.py:175-183)."""

    grads = [p.grad.detach().reshape(-1) for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    return torch.linalg.vector_norm(torch.cat(grads).to(torch.float32))
