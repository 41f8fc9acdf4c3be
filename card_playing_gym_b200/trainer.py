"""The PPO update on this library's kernels, as a drop-in subclass of the reference's trainer.

``device_trainer(PPOTrainer)`` takes the reference's ``cardgym.rl.trainer.PPOTrainer`` class
(the caller's; nothing here imports the reference) and returns a subclass with the same
constructor and ``update(batch, iteration) -> dict`` (trainer.py:430-520). The actor and critic
forward and backward stay PyTorch autograd on the GPU (cuBLAS), and the optimizer, the entropy
controller, the auxiliary-gradient budget and the single global clip stay the reference's code;
the PPO arithmetic between them runs here:

* ``_baseline`` (trainer.py:531-608): the critic's pending values stay on the device; each
  decision's seat values are gathered by ``cg_seat_values`` (column (seat - shift) mod players,
  the zero-sum centring of recorded values in float64), Monte Carlo advantages or segmented GAE
  (``cg_gae_segments``) and the batch-weighted mean/std normalisation run on the device; one
  read brings the advantages and the reporting values to the host.
* ``_policy_loss`` (trainer.py:733-802) for heads without an entropy gate: the fused objective
  kernel (clipped surrogate, KL, entropy, normalised entropy and dL/dlogits in one pass) behind
  an autograd function; gated heads keep the reference's torch code.
* ``_value_loss`` (trainer.py:822-850): the fused value-loss kernel with its gradient.

With a process group (one process per GPU, ``torch.distributed``), every rank holds a shard of
whole trajectories (``data_parallel.shard_games``) with decision weights over the global game
count (``data_parallel.rescale_batch_weights``), and the update exchanges: the advantage
normalisation's global weighted sums; the actor's gradients (``.grad``, or both auxiliary-budget
stashes) and the critic's, SUM-allreduced once per optimizer step after the last microbatch;
and every reported total (so the entropy controller sees the global entropy).
"""

from __future__ import annotations

import sys
import numpy as np
import torch
import torch.distributed as dist

from . import ppo
from .data_parallel import GradientAllreduce, _world, allreduce_sums, global_weighted_mean_std


def _gather_arrays(arrays: list[np.ndarray], group) -> list[np.ndarray]:
    """Each array concatenated over the ranks, rank order (reporting only)."""

    if _world(group)[1] == 1:
        return arrays
    gathered: list = [None] * _world(group)[1]
    dist.all_gather_object(gathered, arrays, group=group)
    return [np.concatenate([rank[i] for rank in gathered]) for i in range(len(arrays))]


def device_trainer(base: type) -> type:
    """A subclass of the reference's ``PPOTrainer`` whose PPO arithmetic runs on the B200 kernels."""

    reference = sys.modules[base.__module__]  # the reference's own helpers (autocast, statistics, _reduce)

    class DevicePPOTrainer(base):
        def __init__(self, *args, process_group=None, **kwargs) -> None:
            super().__init__(*args, **kwargs)
            if self.device.type != "cuda":
                raise ValueError("the device trainer runs on a CUDA device (there is no CPU path)")
            self.process_group = process_group
            self._actor_sync = GradientAllreduce(self.actor_parameters, group=process_group)
            self._critic_sync = GradientAllreduce(self.critic_parameters, group=process_group)

        @property
        def world_size(self) -> int:
            return _world(self.process_group)[1]

        # -- the update: every reported total summed over the ranks -------------------------------
        def update(self, batch, iteration: int) -> dict[str, float]:
            if self.world_size == 1:
                return super().update(batch, iteration)
            local_reduce = reference._reduce
            group = self.process_group

            def reduce_over_ranks(totals):
                local = local_reduce(totals)
                keys: list = [None] * self.world_size
                dist.all_gather_object(keys, sorted(local), group=group)
                union = sorted(set().union(*keys))
                sums = torch.tensor([local.get(key, 0.0) for key in union], dtype=torch.float64,
                                    device=self.device)
                allreduce_sums(sums, group)
                return dict(zip(union, sums.tolist()))

            reference._reduce = reduce_over_ranks
            try:
                stats = super().update(batch, iteration)
            finally:
                reference._reduce = local_reduce
            # The batch sizes the update reports are counted from each rank's shard.
            counts = [key for key in ("policy_rows", "positions") if key in stats]
            summed = allreduce_sums(torch.tensor([stats[key] for key in counts], dtype=torch.float64,
                                                 device=self.device), group)
            stats.update(zip(counts, summed.tolist()))
            return stats

        # -- gradients: summed over the ranks once the step's last backward is done ----------------
        def _unscale(self, parameters, *stashes):
            super()._unscale(parameters, *stashes)
            if self.world_size == 1:
                return
            if parameters is self.actor_parameters:
                self._actor_sync.reduce_grads()
                self._policy_grads = self._actor_sync.reduce_(self._policy_grads)
                self._auxiliary_grads = self._actor_sync.reduce_(self._auxiliary_grads)
            elif parameters is self.critic_parameters:
                self._critic_sync.reduce_grads()

        # -- advantages (trainer.py:531-649) ---------------------------------------------------------
        def _baseline(self, batch, pending: list) -> dict[str, float]:
            device = self.device
            heads = list(batch.decisions)
            gae = self.config.advantage_estimator == "gae"
            players_max = self.max_players
            state: dict[str, torch.Tensor] = {}
            prediction: dict[str, torch.Tensor] = {}
            dense_parts: list[tuple[np.ndarray, np.ndarray, np.ndarray]] = []
            hosted = None
            if pending:
                values = torch.cat([entry[3] for entry in pending]).float()  # centred critic values, on the device
                index = {head: reference.RowIndex(rows.critic_group, rows.critic_seq)
                         for head, rows in batch.decisions.items()}
                columns = {head: ([], [], [], [], []) for head in heads}  # selected, flat, shift, players, seat
                offset = 0
                dense_flat = []
                for group_index, group, micro, entry in pending:
                    start, stop = micro.start, micro.stop
                    for head, rows in batch.decisions.items():
                        selected = index[head].select(group_index, start, stop)
                        if not selected.size:
                            continue
                        seq = rows.critic_seq[selected] - start
                        out = columns[head]
                        out[0].append(selected)
                        out[1].append(offset + micro.flat(seq, rows.critic_position[selected]))
                        out[2].append(rows.critic_shift[selected])
                        out[3].append(group.player_counts[start:stop][seq])
                        out[4].append(rows.seat[selected])
                    seq_dense, pos_dense = np.nonzero(group.position_weight[start:stop] > 0)
                    players = group.player_counts[start:stop][seq_dense]
                    weight = group.position_weight[start:stop][seq_dense, pos_dense].astype(np.float64)
                    dense_flat.append(offset + micro.flat(seq_dense, pos_dense))
                    dense_parts.append((players, group.returns[start:stop][seq_dense], weight))
                    offset += entry.shape[0]
                for head, rows in batch.decisions.items():
                    parts = columns[head]
                    if not parts[0]:
                        state[head] = torch.zeros((len(rows), players_max), dtype=torch.float64, device=device)
                        prediction[head] = torch.zeros(len(rows), dtype=torch.float64, device=device)
                        continue
                    cat = [torch.from_numpy(np.concatenate(p).astype(np.int64)).to(device) for p in parts]
                    head_state, head_pred = ppo.seat_values(values, cat[2], cat[3], cat[4], cat[1], center=False)
                    state[head] = torch.zeros((len(rows), players_max), dtype=torch.float64, device=device)
                    prediction[head] = torch.zeros(len(rows), dtype=torch.float64, device=device)
                    state[head][cat[0]] = head_state
                    prediction[head][cat[0]] = head_pred
                hosted = (values, dense_flat)
            else:
                for head, rows in batch.decisions.items():
                    if rows.values is None:
                        raise AssertionError("Every decision needs a recorded value or a baseline pass.")
                    players = np.array([batch.actor_groups[g].player_counts[s] for g, s in zip(rows.group, rows.seq)],
                                       dtype=np.int64)
                    upload = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64)).to(device)  # noqa: E731
                    state[head], prediction[head] = ppo.seat_values(
                        torch.from_numpy(np.ascontiguousarray(rows.values, dtype=np.float32)).to(device),
                        upload(rows.seat), upload(players), upload(np.zeros(len(rows))), None, center=True)

            advantages = self._device_advantages(batch, state, prediction, gae)
            weights = torch.from_numpy(np.concatenate([rows.weight for rows in batch.decisions.values()])
                                       .astype(np.float64)).to(device)
            # The reference stores advantages as float32 (DecisionRows.advantages) before its statistics.
            all_advantages = torch.cat([advantages[head] for head in heads]).float().double()
            mean, std = global_weighted_mean_std(all_advantages, weights, self.process_group)
            if self.config.advantage_normalize:
                ppo.normalize_(all_advantages, mean, std)
            host_advantages = all_advantages.cpu().numpy()
            host_prediction = torch.cat([prediction[head] for head in heads]).cpu().numpy()
            at = 0
            for rows in batch.decisions.values():
                rows.advantages[:] = host_advantages[at:at + len(rows)]
                at += len(rows)

            stats: dict[str, float] = {}
            all_target = np.concatenate([rows.returns for rows in batch.decisions.values()]).astype(np.float64)
            all_weight = weights.cpu().numpy()
            host_prediction, all_target, all_weight = _gather_arrays([host_prediction, all_target, all_weight],
                                                                     self.process_group)
            acting = reference.weighted_regression_stats(host_prediction, all_target, all_weight)
            stats.update({f"value_{key}": value for key, value in acting.items()})
            if hosted is not None and dense_parts:
                values_np = hosted[0].cpu().numpy()
                dense_prediction, dense_target, dense_weight = [], [], []
                for flat, (players, returns, weight) in zip(hosted[1], dense_parts):
                    active = np.arange(players_max)[None, :] < players[:, None]
                    dense_prediction.append(values_np[flat][active])
                    dense_target.append(returns[active])
                    dense_weight.append(np.repeat(weight / players, players))
                parts = _gather_arrays([np.concatenate(dense_prediction).astype(np.float64),
                                        np.concatenate(dense_target).astype(np.float64),
                                        np.concatenate(dense_weight)], self.process_group)
                dense = reference.weighted_regression_stats(*parts)
                stats["critic_dense_rmse"] = dense["rmse"]
                stats["critic_dense_correlation"] = dense["correlation"]
            stats["advantage_mean"] = mean
            stats["advantage_std"] = std
            return stats

        def _device_advantages(self, batch, state, prediction, gae: bool) -> dict[str, torch.Tensor]:
            """Monte Carlo ``R - V(s)`` or undiscounted GAE over each game's decision states (trainer.py:583-649)."""

            device = self.device
            if not gae:
                return {head: torch.from_numpy(rows.returns.astype(np.float64)).to(device) - prediction[head]
                        for head, rows in batch.decisions.items()}
            heads = list(batch.decisions)
            game = np.concatenate([batch.decisions[h].game for h in heads]).astype(np.int64)
            order = np.concatenate([batch.decisions[h].order for h in heads]).astype(np.int64)
            sizes = [len(batch.decisions[h]) for h in heads]
            ranked = np.lexsort((order, game))  # each game's states in decision order
            starts = np.searchsorted(game[ranked], np.unique(game[ranked]), side="left")
            games = np.unique(game[ranked])
            starts = np.append(starts, len(ranked)).astype(np.int64)
            returns = np.zeros((len(games), self.max_players))
            for slot, g in enumerate(games.tolist()):
                realised = batch.game_returns[g]
                returns[slot, : realised.shape[0]] = realised
            all_state = torch.cat([state[h] for h in heads])
            seats = torch.from_numpy(np.concatenate([batch.decisions[h].seat for h in heads]).astype(np.int32))
            permutation = torch.from_numpy(ranked).to(device)
            advantages = ppo.segmented_gae(all_state.index_select(0, permutation), seats.to(device)[permutation],
                                           torch.from_numpy(starts).to(device), torch.from_numpy(returns).to(device),
                                           self.config.gae_lambda)
            unsorted = torch.empty_like(advantages)
            unsorted[permutation] = advantages
            return dict(zip(heads, unsorted.split(sizes)))

        # -- losses (trainer.py:733-850) ---------------------------------------------------------------
        def _policy_loss(self, hidden, micro, context, rows, selected, head, alpha, totals):
            if any(gate_head == head for gate_head in self.gates.values()):
                return super()._policy_loss(hidden, micro, context, rows, selected, head, alpha, totals)
            at = self.upload(micro.flat(rows.seq[selected] - micro.start, rows.position[selected]))
            tokens = micro.tokens.reshape(-1, micro.tokens.shape[-1])
            # Candidate lists are padded to the batch's longest; the microbatch's own longest is enough
            # (rows.probs is zero past each row's actions).
            width = int(np.flatnonzero(rows.probs[selected].any(axis=0)).max()) + 1
            features = None if rows.features is None else {
                key: self.upload(value[selected][:, :width]) for key, value in rows.features.items()}
            with reference.autocast_context(self.device, self.precision):
                logits = self.actor.policy_logits(
                    hidden.reshape(-1, hidden.shape[-1])[at], head, features, tokens[at],
                    None if context is None else context.reshape(-1, *context.shape[-2:])[at])
            weight = self.upload(rows.weight[selected])
            objective, sums = ppo.policy_objective(
                logits.float()[:, :width], self.upload(rows.probs[selected][:, :width]),
                self.upload(rows.action[selected]), self.upload(rows.advantages[selected]), weight,
                clip_ratio=self.config.clip_ratio, alpha=alpha[head])
            named = dict(zip(ppo.TOTAL_KEYS, sums))
            totals["policy_loss"].append(named["policy_loss"])
            totals[f"policy_loss_{head}"].append(named["policy_loss"])
            totals["row_weight"].append(named["row_weight"])
            totals["entropy_raw"].append(named["entropy_raw"])
            totals[f"entropy_{head}"].append(named["entropy"])
            totals[f"entropy_weight_{head}"].append(named["entropy_weight"])
            totals["clip"].append(named["clip"])
            totals["behavior_kl"].append(named["behavior_kl"])
            return objective

        def _value_loss(self, model, hidden, dense, group, totals, prefix, values=None):
            if values is None:
                with reference.autocast_context(self.device, self.precision):
                    values = model.player_values(hidden.reshape(-1, hidden.shape[-1]))
            prediction = values[dense.flat].float()
            players = self.upload(group.player_counts[dense.start:][dense.seq])
            targets = self.upload(group.returns[dense.start:][dense.seq])
            loss, sums = ppo.value_loss(prediction, players, targets, dense.weight, self.config.value_reward_scale)
            totals[f"{prefix}_loss"].append(sums[0])
            totals[f"{prefix}_squared_error"].append(sums[1])
            totals[f"{prefix}_target_squared"].append(sums[2])
            totals[f"{prefix}_weight"].append(sums[3])
            return loss

    DevicePPOTrainer.__name__ = DevicePPOTrainer.__qualname__ = f"Device{base.__name__}"
    return DevicePPOTrainer
