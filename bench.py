#!/usr/bin/env python
"""Self-play decode benchmark: decisions/s of one rl-v6 rollout wave, per GPU and whole box.

One step = one merged rollout wave of the reference's batch collector
(cardgym/rl/selfplay.py:406-454 + 486-567) at the BASELINE.json rl-v6 configuration:
4096 concurrent 4-player games = 16,384 KV-cache rows, each appending one token at
its own length (per-game length U[16, 256], shared by the game's four observers;
fp16 KV pool of 257 positions), the fused plump field lookup, the 16-layer trunk,
the final norm, and for each game's acting observer the heads, the legal mask and
an inverse-CDF draw from a host-supplied uniform. Weights are synthetic N(0, 0.02)
in the rl-v6 architecture (no checkpoint is read); tokens, masks and uniforms are
seeded synthetic data.

``value``: decisions/s with every input resident in HBM (4096 decisions per step per
GPU, summed over GPUs; the KV stream alone is ~6.9 GB per wave, far beyond L2, so no
flush is needed). ``e2e``: the same metric through the public API with the step's
inputs copied from pinned host memory and the actions + probabilities copied back,
every step. ``roofline``: the decode-attention kernel, timed live with CUDA events
around each of its launches inside the timed region, against the measured HBM copy
bandwidth. ``cpu_baseline``: the numpy CPU port of the reference path (oracle/) on a
bounded sample, on this host's cores.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "self-play decisions/sec (whole box, 1/2/4/8 B200); PPO-iteration wall time"
UNIT = "decisions/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0
# DRAM bytes (read + write) per decode-attention launch divided by its algorithmic bytes,
# from an ncu capture of the same kernel on the 2,048-game wave (profiles/
# attn_tc_kernel_rlv6_decode.md: 219.12 MB read + 4.83 MB written against 219.24 MB
# algorithmic). The full 4,096-game launch is too large for a multi-pass capture; its traffic
# grows with the keys streamed, so it is reported as this ratio times its algorithmic bytes.
ATTENTION_DRAM_TRAFFIC_RATIO = (219.116544e6 + 4.828672e6) / 219.2448e6


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=300)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--games", type=int, default=4096, help="concurrent 4-player games per GPU")
    parser.add_argument("--min-len", type=int, default=16)
    parser.add_argument("--max-len", type=int, default=256)
    parser.add_argument("--kv", choices=("fp16", "bf16", "fp32"), default="fp16")
    parser.add_argument("--precision", choices=("bf16", "fp32"), default="bf16")
    parser.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    parser.add_argument("--cpu-games", type=int, default=32, help="games per CPU-baseline wave")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--ppo-decisions", type=int, default=262144,
                        help="PPO update batch (whole job, sharded by trajectory); 0 skips the PPO leg")
    parser.add_argument("--ppo-steps", type=int, default=20)
    parser.add_argument("--piquet-steps", type=int, default=20,
                        help="waves of the piquet-scale decode leg (8,192 two-player deals); 0 skips it")
    parser.add_argument("--t2-steps", type=int, default=20,
                        help="waves of the rl-v6 T = 2 leg (two tokens appended per row); 0 skips it")
    parser.add_argument("--pointer-steps", type=int, default=20,
                        help="waves of the piquet and rummy-style pointer-head legs; 0 skips them")
    parser.add_argument("--pointer-divisor", type=int, default=1,
                        help="divide the pointer legs' slots and decoded rows (a small case for profilers)")
    parser.add_argument("--prefill-steps", type=int, default=10,
                        help="prefills of the rl-v6 new-game leg (every row's prefix from position 0); 0 skips it")
    parser.add_argument("--prefill-tokens", type=int, default=16, help="prefix tokens per row in the prefill leg")
    parser.add_argument("--reference-cuda-steps", type=int, default=20,
                        help="waves of each reference-on-this-GPU leg (eager, compiled + graphed); 0 skips them")
    return parser.parse_args(argv)


def world() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def workload_name(args) -> str:
    return (f"rl-v6 rollout decode wave: {args.games} concurrent 4-player games ({4 * args.games} KV rows), "
            f"1 token/row, per-game length U[{args.min_len},{args.max_len}], {args.kv} KV, {args.precision} GEMMs")


# ---------------------------------------------------------------------------------------------
# synthetic wave inputs (numpy, seeded)
# ---------------------------------------------------------------------------------------------
def synthetic_wave(games: int, min_len: int, max_len: int, seed: int) -> dict[str, np.ndarray]:
    from card_playing_gym_b200.plump_schema import PlumpSchema, TOKEN_WIDTH, TOKEN_TRICK_WIN

    rng = np.random.default_rng(seed)
    schema = PlumpSchema()
    rows = 4 * games
    lengths = rng.integers(min_len, max_len + 1, games)  # keys each row attends after the append
    positions = np.repeat(lengths - 1, 4).astype(np.int64)
    tokens = np.zeros((rows, 1, TOKEN_WIDTH), dtype=np.int16)
    sizes = schema.base_vocab_sizes
    tokens[:, 0, 0] = rng.integers(1, 7, rows)
    for slot in range(1, 16):
        tokens[:, 0, slot] = rng.integers(0, sizes[slot], rows)
    tokens[:, 0, 16:25] = rng.integers(0, 53, (rows, 9))
    tokens[:, 0, 25] = rng.integers(0, 12, rows)
    tokens[rng.random(rows) < 0.2, 0, 0] = TOKEN_TRICK_WIN
    seat = rng.integers(0, 4, games)
    readout_rows = (4 * np.arange(games) + seat).astype(np.int64)
    heads = rng.integers(0, 2, games).astype(np.int32)
    legal = rng.random((games, 52)) < 0.3
    legal[np.arange(games), rng.integers(0, 11, games)] = True
    legal[heads == 0, 11:] = False
    uniforms = rng.random(games)
    return dict(tokens=tokens, positions=positions, offsets=np.zeros(rows, np.int64), readout_rows=readout_rows,
                heads=heads, legal=legal.astype(np.uint8), uniforms=uniforms, lengths=lengths)


# ---------------------------------------------------------------------------------------------
# PPO update leg: segmented GAE -> global normalisation -> fused PPO objective + value loss
# ---------------------------------------------------------------------------------------------
PPO_PLAYERS = 4
PPO_ACTIONS = 52
TRUNK_PARAMS = 8_500_000  # the actor trunk's gradient, allreduced once per optimizer step


def synthetic_ppo_batch(decisions: int, seed: int) -> dict[str, np.ndarray]:
    """The PPO-update config: trajectories of U[13,52] decisions (the last one cut to the total),
    values N(0,1), zero-sum terminal returns N(0,1), 52-way Bernoulli(0.3) legal masks with one
    forced legal action, new logits = old + N(0,0.05), actions drawn from the old policy."""

    rng = np.random.default_rng(seed)
    lengths = []
    while sum(lengths) < decisions:
        lengths.append(int(rng.integers(13, 53)))
    lengths[-1] -= sum(lengths) - decisions
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    games = len(lengths)
    returns = rng.standard_normal((games, PPO_PLAYERS))
    returns -= returns.mean(axis=1, keepdims=True)
    legal = rng.random((decisions, PPO_ACTIONS)) < 0.3
    legal[np.arange(decisions), rng.integers(0, PPO_ACTIONS, decisions)] = True
    old = rng.standard_normal((decisions, PPO_ACTIONS)).astype(np.float32)
    masked = np.where(legal, old, -np.inf)
    probs = np.exp(masked - masked.max(axis=1, keepdims=True))
    probs /= probs.sum(axis=1, keepdims=True)
    cdf = np.cumsum(probs, axis=1)
    actions = np.minimum((cdf < rng.random((decisions, 1))).sum(axis=1), PPO_ACTIONS - 1)
    return dict(
        starts=starts, values=rng.standard_normal((decisions, PPO_PLAYERS)), seats=rng.integers(0, 4, decisions),
        returns=returns, logits=old + rng.normal(0.0, 0.05, old.shape).astype(np.float32),
        old_probs=probs.astype(np.float32), actions=actions.astype(np.int64),
        weights=np.full(decisions, 1.0 / (games * PPO_PLAYERS)),
        prediction=rng.standard_normal((decisions, PPO_PLAYERS)).astype(np.float32),
        targets=np.repeat(returns, lengths, axis=0).astype(np.float32),
    )


def run_ppo(args, device, rank: int, world_size: int) -> dict:
    """Time the PPO advantage + loss step on this rank's trajectory shard (max over ranks)."""

    import torch
    import torch.distributed as dist

    from card_playing_gym_b200 import ppo
    from card_playing_gym_b200.data_parallel import normalize_global_, shard_games

    batch = synthetic_ppo_batch(args.ppo_decisions, seed=5)
    g0, g1 = shard_games(batch["starts"], world_size, rank)
    d0, d1 = int(batch["starts"][g0]), int(batch["starts"][g1])
    to = lambda a, dtype=None: torch.as_tensor(np.ascontiguousarray(a)).to(device=device, dtype=dtype)  # noqa: E731
    values = to(batch["values"][d0:d1], torch.float64)
    seats = to(batch["seats"][d0:d1], torch.int32)
    starts = to(batch["starts"][g0:g1 + 1] - d0, torch.int64)
    returns = to(batch["returns"][g0:g1], torch.float64)
    logits = to(batch["logits"][d0:d1])
    old_probs = to(batch["old_probs"][d0:d1])
    actions = to(batch["actions"][d0:d1])
    weights = to(batch["weights"][d0:d1], torch.float32)
    weights64 = to(batch["weights"][d0:d1], torch.float64)
    prediction = to(batch["prediction"][d0:d1])
    targets = to(batch["targets"][d0:d1])
    players = torch.full((d1 - d0,), PPO_PLAYERS, dtype=torch.int32, device=device)
    gradient = torch.zeros(TRUNK_PARAMS, device=device) if world_size > 1 else None

    def local_step():
        advantages = ppo.segmented_gae(values, seats, starts, returns, 0.95)
        normalize_global_(advantages, weights64)  # batch-global two-pass mean/std, no host read
        leaf = logits.detach().requires_grad_()
        objective, _ = ppo.policy_objective(leaf, old_probs, actions, advantages, weights, clip_ratio=0.2, alpha=0.01)
        pred = prediction.detach().requires_grad_()
        loss, _ = ppo.value_loss(pred, players, targets, weights, 1.0)
        (objective + loss).backward()
        return leaf.grad, pred.grad

    # One GPU: the whole step replays as one CUDA graph. Several: the step's kernels replay as three
    # graphs, and its collectives run between them (no collective is captured): GAE and the first
    # pass's sums | allreduce | the second pass's sums | allreduce | normalise, objective, value
    # loss, backward | the gradient allreduce.
    graphed = ppo.GraphedStep(local_step) if world_size == 1 else None
    if world_size > 1:
        first_graph = ppo.GraphedStep(lambda: (lambda a: (a, ppo.weighted_sums(a, weights64, 0.0)))(
            ppo.segmented_gae(values, seats, starts, returns, 0.95)))
        held: dict = {}

        def second_pass():
            advantages, first = first_graph.outputs
            return ppo.weighted_sums_shifted(advantages, weights64, first)

        def finish():
            advantages, first = first_graph.outputs
            ppo.normalize_from_sums_(advantages, first, held["second"].outputs)
            leaf = logits.detach().requires_grad_()
            objective, _ = ppo.policy_objective(leaf, old_probs, actions, advantages, weights, clip_ratio=0.2,
                                                alpha=0.01)
            pred = prediction.detach().requires_grad_()
            loss, _ = ppo.value_loss(pred, players, targets, weights, 1.0)
            (objective + loss).backward()
            return leaf.grad, pred.grad

        held["second"] = ppo.GraphedStep(second_pass)
        finish_graph = ppo.GraphedStep(finish)

    def step():
        if graphed is not None:
            return graphed()
        _, first = first_graph()
        dist.all_reduce(first)
        second = held["second"]()
        dist.all_reduce(second)
        grads = finish_graph()
        dist.all_reduce(gradient)
        return grads

    for _ in range(3):
        step()
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.ppo_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / args.ppo_steps
    kernels_ms = allreduce_ms = None
    if world_size > 1:
        # The same steps split in their two parts: this rank's kernels alone, then the gradient
        # allreduce alone (the one collective whose cost grows with the ranks).
        dist.barrier()
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(args.ppo_steps):
            first_graph()
            held["second"]()
            finish_graph()
        end.record(stream)
        torch.cuda.synchronize(device)
        kernels_ms = start.elapsed_time(end) / args.ppo_steps
        dist.barrier()
        torch.cuda.synchronize(device)
        start.record(stream)
        for _ in range(args.ppo_steps):
            dist.all_reduce(gradient)
        end.record(stream)
        torch.cuda.synchronize(device)
        allreduce_ms = start.elapsed_time(end) / args.ppo_steps
        t = torch.tensor([ms, kernels_ms, allreduce_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kernels_ms, allreduce_ms = (float(v) for v in t.tolist())
    n, g, a, pl = d1 - d0, g1 - g0, PPO_ACTIONS, PPO_PLAYERS
    # Bytes the kernels must move on this rank: GAE, two normalisation passes + the in-place
    # normalise, the fused objective (logits, old probs, actions, advantages, weights in; dlogits
    # out) and the value loss (prediction, targets, players, weights in; gradient out).
    algorithmic = (n * pl * 8 + n * 4 + g * pl * 8 + (g + 1) * 8 + n * 8) + 2 * (n * 16) + n * 16 \
        + (3 * n * a * 4 + n * 8 + n * 4 + n * 4) + (3 * n * pl * 4 + n * 8)
    peak, peak_kind = measured_peak()
    achieved = algorithmic / (ms / 1000.0) / 1e9
    return {
        "workload": (f"PPO advantage + loss step: {args.ppo_decisions} decisions in U[13,52] trajectories, "
                     f"{PPO_PLAYERS} seats, {PPO_ACTIONS}-way legal-masked logits, lambda 0.95, clip 0.2"),
        "decisions": args.ppo_decisions, "decisions_per_gpu": n, "games_per_gpu": g, "ms_per_step": ms,
        "decisions_per_s": args.ppo_decisions / (ms / 1000.0), "scaling": "strong",
        "steps": args.ppo_steps, "algorithmic_bytes_per_gpu": algorithmic, "achieved_gbs": achieved,
        "hbm_frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
        "collectives": ("none" if world_size == 1 else
                        f"2 x 3-scalar allreduce (global mean/std) + {TRUNK_PARAMS * 4 / 1e6:.0f} MB gradient "
                        "allreduce (NCCL) per step"),
        "includes": "GAE, global two-pass mean/std and normalise on the device (no host read), fused PPO "
                    "objective fwd+grad, value loss fwd+grad, autograd backward",
        "launch": ("one CUDA graph replay per step (ppo.GraphedStep)" if world_size == 1 else
                   "three CUDA graph replays per step with the collectives between them"),
        "kernels_ms_per_step": kernels_ms, "gradient_allreduce_ms_per_step": allreduce_ms,
        "gradient_allreduce_bus_gbs": (None if allreduce_ms is None else
                                   TRUNK_PARAMS * 4 * 2 * (world_size - 1) / world_size / (allreduce_ms / 1000.0) / 1e9),
    }


# ---------------------------------------------------------------------------------------------
# Piquet-scale decode leg: the same wave at the piquet-scale trunk's dimensions
# ---------------------------------------------------------------------------------------------
def run_piquet_scale(args, device, rank: int, world_size: int) -> dict:
    """8,192 two-player deals per GPU (16,384 KV rows), one token per row, lengths U[32, 512],
    fp16 KV, through PlumpActor at PIQUET_SCALE dims (d 256, 16 layers, 8/2 heads of 32,
    d_ff 512; the plump field lookup and heads stand in for piquet's)."""

    import torch
    import torch.distributed as dist

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.config import PIQUET_SCALE, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    deals, max_len = 8192, 512
    actor = PlumpActor(PIQUET_SCALE, synthetic_plump_actor_state(PIQUET_SCALE, seed=1), device=device,
                       precision="bf16")
    wave = synthetic_wave(deals // 2, 32, max_len, seed=2000 + 7919 * rank)  # 4 rows per group of 2 deals
    rows = 4 * (deals // 2)
    cache = actor.new_cache(rows + 1, max_len + 1, torch.float16)
    generator = torch.Generator(device=device).manual_seed(23 + rank)
    for pool in (cache.k_pool, cache.v_pool):
        for layer in range(pool.shape[0]):
            pool[layer].normal_(generator=generator)
    dev = {k: torch.from_numpy(v).to(device) for k, v in wave.items()}
    # one decision per deal: the readout row of each deal's acting player
    readout = torch.arange(0, rows, 2, device=device, dtype=torch.int64)
    heads = torch.randint(0, 2, (deals,), device=device, dtype=torch.int32, generator=generator)
    legal = dev["legal"].repeat_interleave(2, dim=0)
    uniforms = dev["uniforms"].repeat_interleave(2, dim=0)

    def step():
        hidden = actor.forward_ragged(dev["tokens"], dev["positions"], cache, dev["offsets"], span=max_len + 1)
        return actor.decide(hidden, heads, legal, uniforms, readout, logits=False, values=False)

    for _ in range(3):
        step()
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.piquet_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / args.piquet_steps
    nat.attention_profiling(True, capacity=args.piquet_steps * 16 + 16)
    for _ in range(args.piquet_steps):
        step()
    attention_ms = nat.attention_timings()
    nat.attention_profiling(False)
    if world_size > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    trunk = PIQUET_SCALE.trunk()
    keys = float(np.minimum(wave["positions"] + 1, max_len + 1).sum())
    algorithmic = keys * trunk.n_kv_heads * trunk.head_dim * 2 * 2 + rows * trunk.n_heads * trunk.head_dim * 4
    mean_ms = statistics.fmean(attention_ms)
    achieved = algorithmic / (mean_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    return {
        "workload": (f"piquet-scale decode wave: {deals} two-player deals ({rows} KV rows), 1 token/row, lengths "
                     f"U[32,{max_len}], fp16 KV, trunk d256/16L/8-2 heads of 32/d_ff 512 (plump lookup and heads "
                     "stand in for piquet's)"),
        "value": world_size * deals / (ms / 1000.0), "unit": "decisions/s", "rows_per_s": world_size * rows / (ms / 1000.0),
        "ms_per_step": ms, "steps": args.piquet_steps,
        "attention_roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                               "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                               "algorithmic_bytes_per_launch": algorithmic, "mean_launch_ms": mean_ms},
    }


def run_two_token_wave(args, device, rank: int, world_size: int, actor, cache, wave: dict, span: int) -> dict:
    """The rl-v6 wave with T = 2 tokens appended per row (both readouts' rows decide on the
    second), the same games, cache and heads as the headline wave."""

    import torch
    import torch.distributed as dist

    rows = wave["tokens"].shape[0]
    tokens = np.repeat(wave["tokens"], 2, axis=1)
    tokens[:, 1, 1:16] = np.roll(tokens[:, 1, 1:16], 1, axis=0)  # a different second token
    positions = np.maximum(wave["positions"] - 1, 0)
    dev = {k: torch.from_numpy(v).to(device) for k, v in wave.items()}
    dev_tokens = torch.from_numpy(tokens).to(device)
    dev_positions = torch.from_numpy(positions).to(device)
    offsets = torch.ones(rows, dtype=torch.int64, device=device)

    def step():
        hidden = actor.forward_ragged(dev_tokens, dev_positions, cache, offsets, span=span)
        return actor.decide(hidden, dev["heads"], dev["legal"], dev["uniforms"], dev["readout_rows"], logits=False,
                            values=True)

    for _ in range(3):
        step()
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.t2_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / args.t2_steps
    if world_size > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    games = wave["heads"].shape[0]
    return {"workload": f"rl-v6 decode wave with T = 2 tokens per row: {games} games ({rows} rows), same lengths, "
                        "fp16 KV, readout at the second token",
            "value": world_size * games / (ms / 1000.0), "unit": "decisions/s",
            "tokens_per_s": world_size * 2 * rows / (ms / 1000.0), "ms_per_step": ms, "steps": args.t2_steps}


def dense_flops(trunk, row_tokens: int) -> int:
    """FLOPs of every projection of one pass over ``row_tokens`` row-tokens: the first
    launch's PLE context and QKV GEMMs, then per layer out, up, down and the next layer's QKV."""

    d, f, qkv = trunk.d_model, trunk.d_ff, (trunk.n_heads + 2 * trunk.n_kv_heads) * trunk.head_dim
    ple_w = trunk.n_layers * trunk.per_layer_dim
    layer_flops = 2 * (d * d + 2 * d * f + d * qkv)
    return row_tokens * 2 * (ple_w * d + qkv * d) + row_tokens * (trunk.n_layers - 1) * layer_flops \
        + row_tokens * (layer_flops - 2 * d * qkv)


def run_prefill(args, device, rank: int, world_size: int, actor, cache) -> dict:
    """New games: every row of the rl-v6 pool encodes a fresh prefix of ``--prefill-tokens``
    tokens from position 0 (``forward_prefill``, trunk.py:376-389) and each game's first
    decision is read at its actor's prefix end. The dense layers run over rows x T row-tokens."""

    import torch
    import torch.distributed as dist

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.config import RL_V6

    steps_t = args.prefill_tokens
    parts = [synthetic_wave(args.games, args.min_len, args.max_len, seed=5000 + 31 * t + 7919 * rank)
             for t in range(steps_t)]
    first = parts[0]
    tokens = torch.from_numpy(np.concatenate([p["tokens"] for p in parts], axis=1)).to(device)
    dev = {k: torch.from_numpy(first[k]).to(device) for k in ("heads", "legal", "uniforms", "readout_rows")}
    rows = tokens.shape[0]

    def step():
        hidden = actor.forward_prefill(tokens, cache, rows=None)
        return actor.decide(hidden, dev["heads"], dev["legal"], dev["uniforms"], dev["readout_rows"], logits=False,
                            values=True)

    for _ in range(3):
        step()
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.prefill_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / args.prefill_steps
    nat.dense_profiling(True, capacity=args.prefill_steps * (RL_V6.n_layers + 1) + 16)
    for _ in range(args.prefill_steps):
        step()
    torch.cuda.synchronize(device)
    dense_ms = nat.dense_timings()
    nat.dense_profiling(False)
    if world_size > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    trunk = RL_V6.trunk()
    flops = dense_flops(trunk, rows * steps_t)
    dense_pass_ms = statistics.fmean(dense_ms) * (trunk.n_layers + 1) if dense_ms else float("nan")
    tflops = flops / (dense_pass_ms / 1000.0) / 1e12
    tpeak, tpeak_kind = measured_peak("bf16_tflops_sustained")
    return {"workload": (f"rl-v6 prefill: {rows} rows x {steps_t} prefix tokens from position 0, fp16 KV, "
                         "field lookup + trunk + heads at each game's actor"),
            "tokens_per_s": world_size * rows * steps_t / (ms / 1000.0), "ms_per_step": ms, "steps": args.prefill_steps,
            "dense_layers": {"achieved": tflops, "unit": "TFLOP/s", "peak": tpeak, "frac": tflops / tpeak,
                             "peak_source": f"{tpeak_kind} (MEASURED_PEAKS.json bf16_tflops_sustained)",
                             "mean_launch_ms": statistics.fmean(dense_ms) if dense_ms else None,
                             "flops_per_pass": flops}}


def run_pointer_wave(args, device, rank: int, world_size: int, kind: str) -> dict:
    """A decode wave through the piquet or rummy actor (``piquet.PiquetActor``,
    ``rummy.RummyActor``; synthetic weights under the reference's parameter names) and a
    pointer head with masked sampling.

    piquet: the 16-layer actor (d256/8-2/d_ff 512), 8,192 two-player deals (16,384 KV rows, all
      decoded), lengths U[32, 512], one play decision per deal scored by the play CardScorer over
      the readout token's 32 grid cards.
    rummy: the base actor (d256/8L/8-2/d_ff 768), 8,192 slots, half of them decoded per wave
      through gathered rows (the continuous collector's form), lengths U[8, 384], 1 in 32 decoded
      rows a replaced game's first token at position 0, one play decision per three decoded rows
      scored by CandidateScorer over U[1, 64] candidates (padded to the wave's max) with the
      readout token's 52 ledger cards.
    Each wave runs the actor's grid over the decoded tokens (piquet's card grid, rummy's ledger
    grid), fuses its summary into the one-hot field lookup of the first trunk layer, decodes, and
    scores the readouts with the grid cards ``pop_context`` hands back."""

    import torch
    import torch.distributed as dist

    from card_playing_gym_b200 import piquet, rummy
    from card_playing_gym_b200.sampling import masked_sample

    rng = np.random.default_rng(3000 + 7919 * rank + (0 if kind == "piquet" else 1))
    gen = torch.Generator(device=device).manual_seed(31 + rank)
    if kind == "piquet":
        config = piquet.PiquetModelConfig()
        actor = piquet.PiquetActor(config, piquet.synthetic_piquet_actor_state(config, seed=5), device=device)
        vocab, card_codes, card_slots = piquet.FIELD_VOCAB, 12, 32
        slots, decoded, min_len, max_len = 16384, 16384, 32, 512
    else:
        config = rummy.RummyModelConfig()
        actor = rummy.RummyActor(config, rummy.synthetic_rummy_actor_state(config, seed=5), device=device)
        vocab, card_codes, card_slots = rummy.FIELD_VOCAB, rummy.CARD_VOCAB, 52
        slots, decoded, min_len, max_len = 8192, 4096, 8, 384
    divisor = max(1, args.pointer_divisor)
    slots, decoded = max(2, slots // divisor // 2 * 2), max(2, decoded // divisor // 2 * 2)
    cache = actor.new_cache(slots + 1, max_len + 1, torch.float16)
    for pool in (cache.k_pool, cache.v_pool):
        for layer in range(pool.shape[0]):
            pool[layer].normal_(generator=gen)
    lengths = rng.integers(min_len, max_len + 1, slots)
    fields = np.stack([rng.integers(0, v, decoded) for v in vocab], axis=-1)
    codes = rng.integers(0, card_codes, (decoded, card_slots))
    tokens = np.concatenate([fields, codes], axis=-1).astype(np.int16)[:, None, :]
    rows = np.sort(rng.choice(slots, decoded, replace=False)) if decoded < slots else np.arange(slots)
    positions = (lengths[rows] - 1).astype(np.int64)
    if kind == "rummy":
        # Games that finished and were replaced in this wave: the slot's length resets and the
        # new game's first token goes to position 0 (continuous.py:383-408).
        positions[rng.random(decoded) < 1.0 / 32] = 0
    dev_tokens = torch.from_numpy(tokens).to(device)
    dev_rows = torch.from_numpy(rows.astype(np.int64)).to(device)
    dev_positions = torch.from_numpy(positions).to(device)
    offsets = torch.zeros(decoded, dtype=torch.int64, device=device)
    if kind == "piquet":
        decisions, width = decoded // 2, 32
        readout = torch.arange(0, decoded, 2, device=device)
        legal = torch.from_numpy(rng.random((decisions, width)) < 0.4).to(device)
        legal[:, 0] = True
        features = None
    else:
        decisions = decoded // 3
        readout = torch.from_numpy(np.sort(rng.choice(decoded, decisions, replace=False))).to(device)
        counts = rng.integers(1, 65, decisions)
        width = int(counts.max())
        cand_cards = np.full((decisions, width, 13), rummy.NO_CARD, dtype=np.int64)
        cand_cards[..., :3] = rng.integers(0, 52, (decisions, width, 3))
        cand_cards[..., 1:3][rng.random((decisions, width)) < 0.7] = rummy.NO_CARD
        features = {"kind": torch.from_numpy(rng.integers(0, 7, (decisions, width))).to(device),
                    "cards": torch.from_numpy(cand_cards).to(device),
                    "target": torch.full((decisions, width, 13), rummy.NO_CARD, dtype=torch.int64, device=device)}
        legal = torch.from_numpy(np.arange(width)[None, :] < counts[:, None]).to(device)
    uniforms = torch.from_numpy(rng.random(decisions)).to(device)

    def step():
        hidden = actor.forward_ragged(dev_tokens, dev_positions, cache, offsets, span=max_len + 1, rows=dev_rows)
        cards = actor.pop_context()[:, 0].index_select(0, readout)  # T = 1: the readout is the only token
        logits = actor.policy_logits(hidden.index_select(0, readout), "play", features, None, cards)
        return masked_sample(logits, legal, uniforms)

    for _ in range(3):
        step()
    if world_size > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.pointer_steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / args.pointer_steps
    if world_size > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    desc = {
        "piquet": (f"piquet decode wave through PiquetActor: {decisions} deals ({decoded} KV rows, 1 token/row), "
                   f"lengths U[{min_len},{max_len}], fp16 KV, card grid (2 blocks) + summary, one-hot field lookup "
                   "(32 fields, 964 rows) fused into the trunk d256/16L/8-2/d_ff 512 -> play CardScorer over the "
                   "readout's 32 grid cards -> masked sampling"),
        "rummy": (f"rummy-style continuous wave through RummyActor: {slots} slots, {decoded} gathered rows decoded "
                  f"(1 token/row), lengths U[{min_len},{max_len}] (1 in 32 a replaced game at position 0), fp16 KV, "
                  "ledger grid (52 cards, 2 blocks) + summary, one-hot lookup of rummy's 26 fields (931 rows) fused "
                  f"into the trunk d256/8L/8-2/d_ff 768 -> CandidateScorer over U[1,64] candidates (padded to {width}) "
                  "-> masked sampling"),
    }[kind]
    return {"workload": desc, "value": world_size * decisions / (ms / 1000.0), "unit": "decisions/s",
            "rows_per_s": world_size * decoded / (ms / 1000.0), "ms_per_step": ms, "steps": args.pointer_steps}


# ---------------------------------------------------------------------------------------------
# CPU port of the reference path (oracle/): the baseline leg and the reference arm
# ---------------------------------------------------------------------------------------------
class CpuWave:
    """One rollout wave of the numpy port on a bounded sample of games (float32, all host cores)."""

    def __init__(self, games: int, min_len: int, max_len: int, seed: int):
        from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
        from oracle import plump as oplump
        from oracle.trunk import Precision

        config = {k: getattr(RL_V6, k) for k in ("d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff",
                                                  "per_layer_dim", "value_embeddings", "max_players", "max_hand_size")}
        state = synthetic_plump_actor_state(RL_V6, seed=0)
        self.actor = oplump.PlumpActor(state, config, Precision(kv="fp32", dtype=np.float32))
        self.wave = synthetic_wave(games, min_len, max_len, seed)
        self.games = games
        rng = np.random.default_rng(seed + 1)
        self.cache = self.actor.new_cache(4 * games, max_len + 1)
        self.cache.k[...] = rng.standard_normal(self.cache.k.shape, dtype=np.float32)
        self.cache.v[...] = rng.standard_normal(self.cache.v.shape, dtype=np.float32)
        self.span = max_len + 1

    def step(self) -> np.ndarray:
        from oracle import ppo as oppo

        w = self.wave
        hidden = self.actor.forward_ragged(w["tokens"].astype(np.int64), w["positions"], self.cache, w["offsets"],
                                           span=self.span)
        readout = hidden[w["readout_rows"]]
        actions = np.zeros(self.games, dtype=np.int64)
        for head, (name, width) in enumerate((("bid", 11), ("play", 52))):
            rows = w["heads"] == head
            logits = self.actor.heads.policy_logits(readout[rows], name).astype(np.float32)
            mask = w["legal"][rows, :width].astype(bool)
            probs = oppo.masked_probabilities(logits, mask)
            actions[rows] = oppo.sample_rows(probs, mask, w["uniforms"][rows])
        self.actor.heads.player_values(readout)
        return actions


# ---------------------------------------------------------------------------------------------
# the unmodified reference (baseline/_ref): its own CPU path and its own CUDA paths
# ---------------------------------------------------------------------------------------------
REFERENCE_PATH = REPO / "baseline" / "_ref"
REFERENCE_MODEL_FIELDS = ("max_players", "max_hand_size", "d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff",
                          "per_layer_dim", "value_embeddings")


def reference_import() -> str | None:
    """Make the reference package in baseline/_ref importable; the reason it is not, or None."""

    if not (REFERENCE_PATH / "cardgym" / "__init__.py").exists():
        return "the reference package is not installed in baseline/_ref (__graft_entry__.build() places it there)"
    if str(REFERENCE_PATH) not in sys.path:
        sys.path.insert(0, str(REFERENCE_PATH))
    try:
        import cardgym.games.plump.model  # noqa: F401
        import cardgym.rl.ppo  # noqa: F401
    except Exception as exc:  # noqa: BLE001 - reported in the bench line
        return f"importing the reference failed: {type(exc).__name__}: {exc}"
    return None


def reference_actor(config, state: dict, device):
    """The reference's own PlumpActor (cardgym/games/plump/model.py) holding the synthetic weights."""

    import torch
    from cardgym.games.plump.model import PlumpActor as RefActor
    from cardgym.games.plump.model import PlumpModelConfig as RefConfig

    actor = RefActor(RefConfig(**{k: getattr(config, k) for k in REFERENCE_MODEL_FIELDS}))
    missing, unexpected = actor.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()}, strict=False)
    if unexpected:
        raise RuntimeError(f"synthetic weights the reference actor does not have: {unexpected[:4]}")
    return actor.to(device).eval()


class ReferenceCpuWave:
    """One rollout wave of the reference's own CPU path on a bounded sample of games: its PlumpActor's
    forward_ragged (fp32 PyTorch on every host core, fp32 KV pool), the heads, and its numpy
    masked_probabilities / sample_rows (cardgym/nn/model.py:76-89, cardgym/rl/ppo.py:75-94)."""

    def __init__(self, games: int, min_len: int, max_len: int, seed: int):
        import torch

        from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state

        torch.set_num_threads(os.cpu_count() or 1)
        self.actor = reference_actor(RL_V6, synthetic_plump_actor_state(RL_V6, seed=0), "cpu")
        self.wave = synthetic_wave(games, min_len, max_len, seed)
        self.games = games
        self.cache = self.actor.new_cache(4 * games, max_len + 1, torch.float32)
        generator = torch.Generator().manual_seed(seed + 1)
        for layer in range(len(self.cache.k)):
            self.cache.k[layer].normal_(generator=generator)
            self.cache.v[layer].normal_(generator=generator)
        w = self.wave
        self.inputs = [torch.from_numpy(w["tokens"].astype(np.int64)), torch.from_numpy(w["positions"]),
                       torch.from_numpy(w["offsets"])]
        self.span = max_len + 1

    def step(self) -> np.ndarray:
        import torch
        from cardgym.rl.ppo import masked_probabilities, sample_rows

        w = self.wave
        tokens, positions, offsets = self.inputs
        with torch.inference_mode():
            hidden = self.actor.forward_ragged(tokens, positions, self.cache, offsets, span=self.span)
            readout = hidden[torch.from_numpy(w["readout_rows"])]
            actions = np.zeros(self.games, dtype=np.int64)
            for head, (name, width) in enumerate((("bid", 11), ("play", 52))):
                rows = w["heads"] == head
                logits = self.actor.policy_logits(readout[torch.from_numpy(rows)], name).float().numpy()
                mask = w["legal"][rows, :width].astype(bool)
                probs = masked_probabilities(logits, mask)
                actions[rows] = sample_rows(probs, mask, w["uniforms"][rows])
            self.actor.player_values(readout)
        return actions


def cpu_wave(args):
    """The reference's own CPU wave when baseline/_ref holds it, else the numpy port (oracle/)."""

    reason = reference_import()
    if reason is None:
        return ReferenceCpuWave(args.cpu_games, args.min_len, args.max_len, seed=99), "reference", None
    return CpuWave(args.cpu_games, args.min_len, args.max_len, seed=99), "port", reason


def cpu_sample_text(kind: str, games: int) -> str:
    if kind == "reference":
        return (f"{games} games ({4 * games} rows) per wave of the same workload through the reference's own "
                "PlumpActor.forward_ragged + heads (fp32 PyTorch, fp32 KV) and numpy sampler, from baseline/_ref")
    return f"{games} games ({4 * games} rows) per wave of the same workload, numpy float32 port (oracle/)"


def cpu_baseline(args, seconds: float) -> dict:
    wave, kind, reason = cpu_wave(args)
    wave.step()  # warm-up
    count, start = 0, time.perf_counter()
    while True:
        wave.step()
        count += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds or count >= 1000:
            break
    out = {
        "value": count * args.cpu_games / elapsed,
        "unit": UNIT,
        "cores": os.cpu_count(),
        "kind": kind,
        "sample": f"{count} waves: " + cpu_sample_text(kind, args.cpu_games) + f", {elapsed:.1f} s",
    }
    if reason:
        out["reference_unavailable"] = reason
    return out


def run_reference(args) -> int:
    rank, world_size, _ = world()
    if rank != 0:
        return 0
    wave, kind, reason = cpu_wave(args)
    for _ in range(max(args.warmup, 1)):
        wave.step()
    start = time.perf_counter()
    for _ in range(args.steps):
        wave.step()
    elapsed = time.perf_counter() - start
    value = args.steps * args.cpu_games / elapsed
    sample = cpu_sample_text(kind, args.cpu_games)
    if reason:
        sample += f" (the reference itself: {reason})"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world_size,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args), "cpu_sample_games": args.cpu_games},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _cuda_ms(step, steps: int, device) -> float:
    """Mean device milliseconds of `step` over `steps` calls (CUDA events on the current stream)."""

    import torch

    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize(device)
    return start.elapsed_time(end) / steps


class ReferenceCudaWave:
    """The rl-v6 bench wave (same games, lengths, tokens, fp16 KV pool of random contents) through the
    reference's own PlumpActor on this GPU, as its batch collector runs it: bf16 autocast around
    forward_ragged, the readouts gathered, each head's logits and the values in fp32 on their way to
    pinned host memory (cardgym/rl/selfplay.py:406-454, 486-530). Host sampling is not timed."""

    def __init__(self, args, device):
        import torch

        from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state

        self.device = device
        self.actor = reference_actor(RL_V6, synthetic_plump_actor_state(RL_V6, seed=0), device)
        wave = synthetic_wave(args.games, args.min_len, args.max_len, seed=1000)
        self.games = args.games
        self.span = args.max_len + 1
        self.cache = self.actor.new_cache(4 * args.games + 1, self.span, torch.float16)
        generator = torch.Generator(device=device).manual_seed(17)
        for layer in range(len(self.cache.k)):
            self.cache.k[layer].normal_(generator=generator)
            self.cache.v[layer].normal_(generator=generator)
        self.tokens = torch.from_numpy(wave["tokens"].astype(np.int64)).to(device)
        self.positions = torch.from_numpy(wave["positions"]).to(device)
        self.offsets = torch.from_numpy(wave["offsets"]).to(device)
        self.readout = torch.from_numpy(wave["readout_rows"]).to(device)
        self.groups = [(name, torch.from_numpy(np.flatnonzero(wave["heads"] == head)).to(device))
                       for head, name in enumerate(("bid", "play"))]

    def heads(self, hidden):
        readout = hidden.index_select(0, self.readout)
        outputs = [self.actor.policy_logits(readout.index_select(0, rows), name) for name, rows in self.groups]
        outputs.append(self.actor.player_values(readout))
        return [output.float() for output in outputs]

    def eager_step(self):
        import torch

        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            hidden = self.actor.forward_ragged(self.tokens, self.positions, self.cache, self.offsets, span=self.span)
            return [output.to("cpu", non_blocking=True) for output in self.heads(hidden)]

    def graphed_step(self):
        """torch.compile + one CUDA graph, as the reference's DecodeGraphs builds it (cardgym/rl/graphs.py:66-151):
        the body compiled by cardgym.nn.compile.compiled, warmed up on a side stream, captured, replayed. The plump
        embedder's nonzero() cannot be captured (a data-dependent shape with a host sync), so the raw field lookup
        runs once beforehand and the graph holds Trunk.condition, the 16-layer forward_ragged and the heads."""

        import torch
        from cardgym.nn.compile import compiled

        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
            lookups = [t if t is None else t.clone() for t in self.actor.embed(self.tokens)]

        def outputs(x, ple, values):
            # DecodeGraphs._outputs (graphs.py:88-102): every head on every readout, then the values.
            with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
                conditioned = self.actor.trunk.condition(x, ple, values)
                hidden = self.actor.trunk.forward_ragged(*conditioned, self.cache, self.positions, self.offsets,
                                                         self.span, None)
                readout = hidden.index_select(0, self.readout)
                heads = [self.actor.policy_logits(readout, name) for name, _ in self.groups]
                return torch.cat([o.float() for o in (*heads, self.actor.player_values(readout))], dim=-1)

        body = compiled(outputs, self.device)
        stream = torch.cuda.current_stream(self.device)
        with torch.inference_mode():
            side = torch.cuda.Stream(self.device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                body(*lookups)
                body(*lookups)
            stream.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                output = body(*lookups)
        host = torch.empty(output.shape, dtype=output.dtype).pin_memory()

        def step():
            graph.replay()
            host.copy_(output, non_blocking=True)

        return step, graph


def run_reference_k1(device, steps: int = 2000) -> dict:
    """The reference's one CUDA kernel (cardgym/nn/cuda_decode.py:46-151, JIT-built by its own load_inline) against
    this repo's decode attention at the kernel's own envelope: head_dim 32, spans <= 64, fp16, 384 rows x 3 tokens
    (the shape its docstring times, cuda_decode.py:5-9)."""

    import torch
    from cardgym.nn import cuda_decode as k1

    from card_playing_gym_b200.cuda_decode import decode_attention

    generator = torch.Generator(device=device).manual_seed(3)
    batch, heads, kv_heads, dim, tokens, span = 384, 8, 2, 32, 3, 64
    q = torch.randn((batch, heads, tokens, dim), device=device, generator=generator).half()
    k = torch.randn((batch, kv_heads, span, dim), device=device, generator=generator).half()
    v = torch.randn((batch, kv_heads, span, dim), device=device, generator=generator).half()
    rows = torch.arange(batch, device=device)
    lengths = torch.randint(1, span - tokens + 2, (batch,), device=device, generator=generator)
    scale = dim ** -0.5
    theirs = k1.decode_attention(q, k, v, rows, lengths, span, scale)
    ours = decode_attention(q, k, v, rows, lengths, span, scale)
    difference = float((theirs.float() - ours.float()).abs().max())
    # Each op is called `per_graph` times inside one CUDA graph, so the device time is measured and not the
    # host's launch rate (a Python custom-op call costs more host time than either kernel takes).
    per_graph = 100

    def graphed(op):
        stream = torch.cuda.current_stream(device)
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                op(q, k, v, rows, lengths, span, scale)
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(per_graph):
                op(q, k, v, rows, lengths, span, scale)
        graph.replay()
        return graph

    k1_graph, ours_graph = graphed(k1.decode_attention), graphed(decode_attention)
    replays = max(1, steps // per_graph)
    k1_ms = _cuda_ms(k1_graph.replay, replays, device) / per_graph
    ours_ms = _cuda_ms(ours_graph.replay, replays, device) / per_graph
    del k1_graph, ours_graph
    return {"shape": "384 rows x 3 tokens, 8 query / 2 KV heads of 32, spans <= 64, fp16 (L2-resident)",
            "reference_us": 1000 * k1_ms, "b200_us": 1000 * ours_ms, "speedup": k1_ms / ours_ms,
            "max_abs_difference": difference, "calls": replays * per_graph,
            "timing": f"CUDA events around graph replays of {per_graph} back-to-back calls per op"}


def run_reference_cuda(args, device) -> dict:
    """The unmodified reference on this GPU at the rl-v6 bench config: eager, torch.compile + CUDA graph, and K1."""

    reason = reference_import()
    if reason is not None:
        return {"unavailable": reason}
    import torch

    out: dict = {"source": "baseline/_ref (the reference package, unmodified)"}
    steps = args.reference_cuda_steps
    try:
        wave = ReferenceCudaWave(args, device)
        for _ in range(3):
            wave.eager_step()
        ms = _cuda_ms(wave.eager_step, steps, device)
        out["eager"] = {"value": args.games / (ms / 1000.0), "unit": UNIT, "ms_per_step": ms, "steps": steps,
                        "path": "SequenceModel.forward_ragged under bf16 autocast + heads, eager (how plump rolls out)"}
    except Exception as exc:  # noqa: BLE001 - reported in the bench line
        out["eager"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:400]}
        wave = None
    if wave is not None:
        started = time.perf_counter()
        try:
            step, graph = wave.graphed_step()
            compile_s = time.perf_counter() - started
            for _ in range(3):
                step()
            ms = _cuda_ms(step, steps, device)
            out["compiled_graph"] = {"value": args.games / (ms / 1000.0), "unit": UNIT, "ms_per_step": ms,
                                     "steps": steps, "compile_and_capture_s": compile_s,
                                     "path": "cardgym.nn.compile.compiled body (Trunk.condition + forward_ragged "
                                             "+ heads) captured in one CUDA graph; the field lookup precomputed"}
            del graph
        except Exception as exc:  # noqa: BLE001
            out["compiled_graph"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:400]}
        del wave
        torch.cuda.empty_cache()
    try:
        out["k1"] = run_reference_k1(device)
    except Exception as exc:  # noqa: BLE001
        out["k1"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:400]}
    return out


# ---------------------------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------------------------
CLOCK_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.seek(0)
        clocks, maxima, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            try:
                clocks.append(float(parts[1]))
                maxima.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.file.name)
        return {
            "sm_mhz": statistics.median(clocks) if clocks else None,
            "sm_max_mhz": max(maxima) if maxima else None,
            "reasons": sorted(reasons),
            "samples": len(clocks),
        }


def measured_peak(key: str = "hbm_gbs") -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks[key]), "measured"
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops_sustained": FALLBACK_BF16_TFLOPS_SUSTAINED}[key], "fallback"


# ---------------------------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------------------------
def run_b200(args) -> int:
    import torch
    import torch.distributed as dist

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.config import RL_V6, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    rank, world_size, local = world()
    if world_size > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    kv_dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[args.kv]

    state = synthetic_plump_actor_state(RL_V6, seed=0)
    actor = PlumpActor(RL_V6, state, device=device, precision=args.precision)
    wave = synthetic_wave(args.games, args.min_len, args.max_len, seed=1000 + 7919 * rank)
    rows = 4 * args.games
    max_len = args.max_len + 1
    cache = actor.new_cache(rows + 1, max_len, kv_dtype)  # + the collector's spare scratch row
    generator = torch.Generator(device=device).manual_seed(17 + rank)
    for pool in (cache.k_pool, cache.v_pool):
        for layer in range(pool.shape[0]):
            pool[layer].normal_(generator=generator)
    dev = {k: torch.from_numpy(v).to(device) for k, v in wave.items()}
    span = max_len
    games = args.games

    def step():
        hidden = actor.forward_ragged(dev["tokens"], dev["positions"], cache, dev["offsets"], span=span)
        return actor.decide(hidden, dev["heads"], dev["legal"], dev["uniforms"], dev["readout_rows"], logits=False,
                            values=True)

    def barrier():
        if world_size > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(value: float) -> float:
        if world_size == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    stream = torch.cuda.current_stream(device)
    clocks = ClockSampler(list(range(world_size)) if rank == 0 else []) if rank == 0 else None
    launches0 = nat.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    barrier()
    launches = nat.launch_count() - launches0
    device_ms = start.elapsed_time(end)
    # Attention launch durations for the roofline: the same steps again with CUDA events
    # around every attention launch. Events between kernels stop a kernel from starting
    # while the one before drains, so the headline pass above runs without them.
    profiled_steps = min(args.steps, 100)
    nat.attention_profiling(True, capacity=profiled_steps * RL_V6.n_layers + 16)
    nat.dense_profiling(True, capacity=profiled_steps * (RL_V6.n_layers + 1) + 16)
    for _ in range(profiled_steps):
        step()
    torch.cuda.synchronize(device)
    attention_ms = nat.attention_timings()
    dense_ms = nat.dense_timings()
    nat.attention_profiling(False)
    nat.dense_profiling(False)
    # nvidia-smi needs a few hundred ms to start and samples every 100 ms: when the timed steps
    # are shorter than that, every rank keeps running the same wave (untimed) until ~0.6 s of
    # load have passed since sampling began, so the clocks and throttle reasons are read under load.
    extra = max(0, int(600.0 / max(device_ms / args.steps, 1e-3)) - args.steps - profiled_steps)
    for _ in range(extra):
        step()
    torch.cuda.synchronize(device)
    barrier()
    clock_info = clocks.stop() if clocks else None
    if clock_info is not None and extra:
        clock_info["sampled_over"] = f"the timed steps and {extra} more untimed waves of the same workload"
    device_ms = max_over_ranks(device_ms)
    ms_per_step = device_ms / args.steps
    value = world_size * games * args.steps / (device_ms / 1000.0)

    # e2e: public API, pinned host inputs in, actions + probabilities out, every step.
    host = {k: torch.from_numpy(v).pin_memory() for k, v in wave.items() if k != "lengths"}
    out_actions = torch.empty(games, dtype=torch.int64).pin_memory()
    out_probs = torch.empty((games, 52), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_actions.numel() * 8 + out_probs.numel() * 4

    def e2e_step():
        inputs = {k: v.to(device, non_blocking=True) for k, v in host.items()}
        hidden = actor.forward_ragged(inputs["tokens"], inputs["positions"], cache, inputs["offsets"], span=span)
        _, probs, actions, _ = actor.decide(hidden, inputs["heads"], inputs["legal"], inputs["uniforms"],
                                            inputs["readout_rows"], logits=False, values=False)
        out_actions.copy_(actions, non_blocking=True)
        out_probs.copy_(probs, non_blocking=True)
        stream.synchronize()  # the host needs the actions before it can step its games

    for _ in range(max(2, args.warmup // 2)):
        e2e_step()
    barrier()
    start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    end.record(stream)
    barrier()
    e2e_eager_ms = max_over_ranks(start.elapsed_time(end))

    # The same step captured once as a CUDA graph, copies included: the host writes the next
    # wave's inputs into the pinned buffers and replays (as DecodeGraphs does for the
    # collector), so no launch waits on the host after each wave's synchronize.
    static_in = {k: torch.empty(v.shape, dtype=v.dtype, device=device) for k, v in host.items()}
    graph_workspace = torch.empty(actor.step_workspace_bytes(rows, 1), dtype=torch.uint8, device=device)

    def e2e_body():
        for k, v in host.items():
            static_in[k].copy_(v, non_blocking=True)
        hidden = actor.forward_ragged(static_in["tokens"], static_in["positions"], cache, static_in["offsets"],
                                      span=span, workspace=graph_workspace)
        _, probs, actions, _ = actor.decide(hidden, static_in["heads"], static_in["legal"], static_in["uniforms"],
                                            static_in["readout_rows"], logits=False, values=False)
        out_actions.copy_(actions, non_blocking=True)
        out_probs.copy_(probs, non_blocking=True)

    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        e2e_body()
    stream.wait_stream(side)
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_body()

    def e2e_graph_step():
        e2e_graph.replay()
        stream.synchronize()

    for _ in range(max(2, args.warmup // 2)):
        e2e_graph_step()
    barrier()
    start.record(stream)
    for _ in range(args.steps):
        e2e_graph_step()
    end.record(stream)
    barrier()
    e2e_ms = max_over_ranks(start.elapsed_time(end))
    del e2e_graph
    e2e_value = world_size * games * args.steps / (e2e_ms / 1000.0)
    e2e_eager_value = world_size * games * args.steps / (e2e_eager_ms / 1000.0)
    ppo_line = None
    if args.ppo_decisions > 0:
        with torch.cuda.nvtx.range("ppo"):  # lets a profiler select this leg's launches
            ppo_line = run_ppo(args, device, rank, world_size)
    piquet_line = run_piquet_scale(args, device, rank, world_size) if args.piquet_steps > 0 else None
    pointer_lines = {}
    if args.t2_steps > 0:
        pointer_lines["rlv6_t2"] = run_two_token_wave(args, device, rank, world_size, actor, cache, wave, span)
    if args.pointer_steps > 0:
        with torch.cuda.nvtx.range("piquet_pointer"):  # lets a profiler select each leg's launches
            pointer_lines["piquet_pointer"] = run_pointer_wave(args, device, rank, world_size, "piquet")
        with torch.cuda.nvtx.range("rummy_style"):
            pointer_lines["rummy_style"] = run_pointer_wave(args, device, rank, world_size, "rummy")
    reference_cuda = None
    if args.reference_cuda_steps > 0 and world_size == 1:
        with torch.cuda.nvtx.range("reference_cuda"):
            reference_cuda = run_reference_cuda(args, device)
    if args.prefill_steps > 0:  # last: it overwrites the first positions of every cache row
        with torch.cuda.nvtx.range("rlv6_prefill"):  # lets a profiler select this leg's launches
            pointer_lines["rlv6_prefill"] = run_prefill(args, device, rank, world_size, actor, cache)

    if rank == 0:
        head_dim = RL_V6.trunk().head_dim
        esize = torch.tensor([], dtype=kv_dtype).element_size()
        keys = np.minimum(wave["positions"] + 1, span).sum()  # T = 1: key_length = position + 1
        kv_bytes = float(keys) * RL_V6.n_kv_heads * head_dim * esize * 2
        qo_bytes = rows * RL_V6.n_heads * head_dim * (esize + 2)  # q in the cache dtype, bf16 output
        algorithmic = kv_bytes + qo_bytes
        mean_ms = statistics.fmean(attention_ms) if attention_ms else float("nan")
        achieved = algorithmic / (mean_ms / 1000.0) / 1e9
        peak, peak_kind = measured_peak()
        traffic = ATTENTION_DRAM_TRAFFIC_RATIO * algorithmic
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world_size, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.precision, "data": "synthetic (seeded tokens, masks, uniforms; N(0,0.02) weights)",
            "config": {
                "workload": workload_name(args), "games_per_gpu": games, "rows_per_gpu": rows, "tokens_per_row": 1,
                "max_context": args.max_len, "kv_dtype": args.kv, "precision": args.precision,
                "decisions_per_step_per_gpu": games, "l2": "inputs larger than L2 (KV read ~6.9 GB per wave per GPU)",
                "parallelism": f"independent self-play games on each of {world_size} GPU(s), no collective",
            },
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "launch": "one CUDA graph replay per step (pinned inputs in, wave, actions + probabilities out)",
                    "eager_value": e2e_eager_value},
            "roofline": {
                "kernel": "decode attention (attn_tc_kernel)", "bound": "hbm", "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "traffic": traffic, "traffic_source": "ncu dram bytes of the 2,048-game wave, scaled by algorithmic bytes",
                "algorithmic_bytes_per_launch": algorithmic, "mean_launch_ms": mean_ms,
                "launches_timed": len(attention_ms),
                "timing": (f"CUDA events around each attention launch over {profiled_steps} steps run right after "
                           "the timed region, same workload"),
            },
            "gpu_launches": int(launches),
            "clocks": clock_info,
        }
        # Dense layers (tcgen05): the projections' FLOPs per wave over the summed dense-launch
        # time per wave, against the measured sustained bf16 GEMM rate (timed inside a long step).
        trunk = RL_V6.trunk()
        wave_flops = dense_flops(trunk, rows)
        launches_per_wave = trunk.n_layers + 1
        dense_wave_ms = statistics.fmean(dense_ms) * launches_per_wave if dense_ms else float("nan")
        tflops = wave_flops / (dense_wave_ms / 1000.0) / 1e12
        tpeak, tpeak_kind = measured_peak("bf16_tflops_sustained")
        line["dense_layers"] = {
            "kernel": "tc_dense_kernel (tcgen05, 2-SM pairs)", "bound": "tensor", "achieved": tflops, "peak": tpeak,
            "unit": "TFLOP/s", "frac": tflops / tpeak,
            "peak_source": f"{tpeak_kind} (MEASURED_PEAKS.json bf16_tflops_sustained)",
            "flops_per_wave": wave_flops, "mean_launch_ms": statistics.fmean(dense_ms) if dense_ms else None,
            "launches_timed": len(dense_ms),
            "timing": "CUDA events around each dense launch in the same profiled pass as the attention roofline",
        }
        if ppo_line is not None:
            line["ppo"] = ppo_line
        if piquet_line is not None:
            line["piquet_scale"] = piquet_line
        line.update(pointer_lines)
        if reference_cuda is not None:
            line["reference_cuda"] = reference_cuda
            for key in ("eager", "compiled_graph"):
                base = reference_cuda.get(key, {}).get("value")
                if base:
                    reference_cuda[key]["b200_speedup"] = value / base
                    reference_cuda[key]["b200_e2e_speedup"] = e2e_value / base
        if world_size == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world_size > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
