"""Data-parallel PPO update: trajectory shards, batch-global statistics, gradient allreduce.

Self-play needs no collective: every rank runs its own games, KV pool and seed. The PPO
update of cardgym/rl/trainer.py:430-520 runs on one process in the reference; sharded over
ranks it needs these exchanges per optimizer step, and nothing else:

* the advantage normalisation's batch-global weighted mean and std (trainer.py:601-607 with
  ppo.py:147-153): two allreduces of three float64 sums, keeping the reference's two-pass
  definition (mean first, then the centred second moment);
* the entropy controller's observed per-head entropy (rl/entropy.py:51-69): per head,
  (sum w * H_norm, sum w) summed over ranks;
* the gradients, SUM-reduced (the decision weights already divide by the global game and
  seat counts, so per-rank gradients are partial sums of the global objective's gradient).
  The policy and auxiliary gradient sets are reduced separately because the auxiliary
  budget (trainer.py:897-937) scales one against the other's global norm.

Shards are whole trajectories (GAE segments never cross ranks), contiguous in decision
order and balanced by decision count. The collectives run on the process group given
(NCCL on the GPUs; gloo works the same for host tensors).
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Sequence

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
    """SUM-allreduce of one gradient set in flat buckets, overlapped with backward.

    Buckets are filled in reverse registration order (the order backward produces the
    gradients of a feed-forward stack). A post-accumulate hook marks each parameter ready;
    when every parameter of a bucket is ready the bucket is flattened and its allreduce is
    launched asynchronously, so communication runs while backward computes earlier layers.
    `finish()` waits for every bucket, writes the reduced values back into `.grad` and
    re-arms for the next backward. Parameters without a gradient after backward are reduced
    as zeros, so every rank launches the same collectives in the same order.
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], group=None, bucket_bytes: int = 32 << 20):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.buckets: list[list[torch.nn.Parameter]] = []
        current: list[torch.nn.Parameter] = []
        size = 0
        for p in reversed(self.params):
            nbytes = p.numel() * p.element_size()
            if current and size + nbytes > bucket_bytes:
                self.buckets.append(current)
                current, size = [], 0
            current.append(p)
            size += nbytes
        if current:
            self.buckets.append(current)
        self._bucket_of = {id(p): i for i, bucket in enumerate(self.buckets) for p in bucket}
        self._pending = [len(bucket) for bucket in self.buckets]
        self._flat: list[torch.Tensor | None] = [None] * len(self.buckets)
        self._work: list = [None] * len(self.buckets)
        self._next = 0  # buckets launch in index order, so every rank issues the same sequence
        self._hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in self.params]

    @property
    def world_size(self) -> int:
        return _world(self.group)[1]

    def _ready(self, param: torch.nn.Parameter) -> None:
        index = self._bucket_of[id(param)]
        self._pending[index] -= 1
        while self._next < len(self.buckets) and self._pending[self._next] == 0:
            self._launch(self._next)
            self._next += 1

    def _launch(self, index: int) -> None:
        bucket = self.buckets[index]
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in bucket]
        flat = torch.cat([g.reshape(-1) for g in grads])
        self._flat[index] = flat
        if self.world_size > 1:
            self._work[index] = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    def finish(self) -> None:
        """Wait for every bucket (launching any not yet launched) and write the sums back."""

        while self._next < len(self.buckets):
            self._launch(self._next)
            self._next += 1
        for index, bucket in enumerate(self.buckets):
            if self._work[index] is not None:
                self._work[index].wait()
            flat = self._flat[index]
            at = 0
            for p in bucket:
                n = p.numel()
                value = flat[at:at + n].view_as(p)
                if p.grad is None:
                    p.grad = value.clone()
                else:
                    p.grad.copy_(value)
                at += n
        self._pending = [len(bucket) for bucket in self.buckets]
        self._flat = [None] * len(self.buckets)
        self._work = [None] * len(self.buckets)
        self._next = 0

    def close(self) -> None:
        for hook in self._hooks:
            hook.remove()
        self._hooks = []


def global_grad_norm(params: Iterable[torch.nn.Parameter]) -> torch.Tensor:
    """L2 norm of the (already reduced) gradients, as clip_grad_norm computes it (trainer.py:175-183)."""

    grads = [p.grad.detach().reshape(-1) for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    return torch.linalg.vector_norm(torch.cat(grads).to(torch.float32))
