"""Regenerate the golden fixtures in tests/golden/ by running the reference itself.

Run in a container where the reference checkout is mounted (default
``/root/reference``; override with ``CARDGYM_REFERENCE``)::

    python tests/golden/make_golden.py

Every fixture stores the inputs, the seed of the synthetic weights
(``card_playing_gym_b200.config.synthetic_plump_actor_state``, regenerated
bit-for-bit on any machine from the seed) and the outputs the reference's own
code computed from them. Nothing here is needed at run time on the GPU box: the
.npz files are committed.

Fixtures:
  plump_streams.npz   real plump observer streams from the reference game engine
  trunk_<name>.npz    full forward, prefill + ragged cached steps, heads (fp32),
                      and the reference's own bf16-autocast/fp16-KV ragged outputs
  sampling.npz        masked_probabilities / sample_rows
  ppo.npz             ppo_terms terms and the autograd gradient of the head objective
  gae.npz             gae_advantages per game, acting-seat advantages
  value_loss.npz      PPOTrainer._value_loss and its autograd gradient
  piquet_bags.npz     the piquet field lookup (``_onehot_bags``) in fp32, bf16 and fp16
  card_scorer.npz     the piquet card pointer head (``CardScorer``) in fp32 and bf16 autocast
  candidate_scorer.npz the rummy candidate pointer head (``CandidateScorer``), draw and play calls
  card_grid.npz       the piquet card grid (``CardGrid``) in fp32 and bf16 autocast
  ledger_grid.npz     rummy's ledger grid (52 cards, circular 5-tap convolution), same forms
  piquet_actor.npz    the piquet actor (lookup + card grid + trunk + heads) at a small trunk, fp32
  rummy_actor.npz     the rummy actor (lookup + ledger grid + trunk + candidate heads), same form

``python tests/golden/make_golden.py piquet_bags`` regenerates one fixture.
"""

from __future__ import annotations

import os
import random
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REFERENCE = Path(os.environ.get("CARDGYM_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REFERENCE))

from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state  # noqa: E402

TRUNK_CONFIGS = {
    # tests/conftest.py:16-19 of the reference with all-layer value embeddings (d % ple == 0 branch)
    "tiny_div": dict(d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, per_layer_dim=8, value_embeddings="all"),
    # d % ple != 0: the truncated-repeat PLE branch rl-v6 takes, GQA group 5, one KV head
    "tiny_cat": dict(d_model=40, n_layers=3, n_heads=5, n_kv_heads=1, d_ff=48, per_layer_dim=16, value_embeddings="alternating"),
    # the rl-v6 architecture with synthetic weights
    "rlv6": dict(d_model=240, n_layers=16, n_heads=10, n_kv_heads=2, d_ff=720, per_layer_dim=64, value_embeddings="alternating"),
}


def plump_streams(count: int, seed: int) -> list[np.ndarray]:
    """Observer streams of random complete plump rounds (the reference's tests/nn/test_trunk.py:18-35 recipe)."""

    from cardgym.games.plump.env import PlumpEnv
    from cardgym.games.plump.rounds import RoundSpec, round_game_config
    from cardgym.games.plump.tokens import Schema, seat_tokens

    rng = random.Random(seed)
    result = []
    for index in range(count):
        players, hand = rng.choice([3, 4, 5]), rng.choice(range(3, 11))
        start = rng.randrange(players)
        env = PlumpEnv(round_game_config(RoundSpec(players, hand), bidding_start_player=start), seed=seed * 1000 + index)
        env.reset(seed=seed * 1000 + index)
        while not env.is_done():
            env.step(rng.choice(env.legal_actions()))
        observer = rng.randrange(players)
        result.append(
            seat_tokens(Schema(), env.state.event_log, observer, players, hand,
                        env.state.current_round.initial_hands[observer], start)
        )
    return result


def pad(streams: list[np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    lengths = np.array([s.shape[0] for s in streams], dtype=np.int64)
    out = np.zeros((len(streams), lengths.max(), streams[0].shape[1]), dtype=np.int64)
    for row, s in enumerate(streams):
        out[row, : s.shape[0]] = s
    return out, lengths


def reference_actor(config: dict, seed: int):
    from cardgym.games.plump.model import PlumpActor
    from cardgym.games.plump.model import PlumpModelConfig as RefConfig

    actor = PlumpActor(RefConfig(**config))
    state = synthetic_plump_actor_state(PlumpModelConfig(**config), seed=seed)
    missing, unexpected = actor.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()}, strict=False)
    # Auxiliary heads stay at their init: they are off the rollout path.
    assert not unexpected and all(
        name.startswith(("suit_head", "rank_boundary_head", "trick_head", "next_winner_head", "bid_hit_head"))
        for name in missing
    ), (missing, unexpected)
    return actor.eval()


def ragged_schedule(lengths: np.ndarray, prefix: int, seed: int) -> list[np.ndarray]:
    """Per wave, the tokens each row appends (0..3), as the reference's test_trunk.py:51-56 draws them."""

    rng = random.Random(seed)
    cursor = [prefix] * len(lengths)
    waves = []
    while any(c < n for c, n in zip(cursor, lengths)):
        counts = [min(rng.randint(0, 3), int(n) - c) for c, n in zip(cursor, lengths)]
        if not any(counts):
            continue
        waves.append(np.array(counts, dtype=np.int64))
        cursor = [c + n for c, n in zip(cursor, counts)]
    return waves


def run_ragged(actor, padded, lengths, prefix, waves, kv_dtype, autocast: bool):
    """Prefill then the ragged waves; returns per-wave (tokens, positions, offsets, hidden, bid, card, values)."""

    from contextlib import nullcontext

    ctx = torch.autocast("cpu", dtype=torch.bfloat16) if autocast else nullcontext()
    records = []
    with torch.no_grad():
        cache = actor.new_cache(len(lengths), int(lengths.max()) + 1, kv_dtype)
        with ctx:
            hidden = actor.forward_prefill(torch.from_numpy(padded[:, :prefix]), cache, None)
        prefill_hidden = hidden.float().numpy()
        cursor = np.full(len(lengths), prefix, dtype=np.int64)
        for counts in waves:
            run = int(counts.max())
            tokens = np.zeros((len(lengths), run, padded.shape[2]), dtype=np.int64)
            offsets = np.zeros(len(lengths), dtype=np.int64)
            for row, (start, count) in enumerate(zip(cursor, counts)):
                if not count:
                    continue
                block = padded[row, start : start + count]
                tokens[row, :count] = block
                tokens[row, count:] = block[-1]
                offsets[row] = count - 1
            with ctx:
                h = actor.forward_ragged(torch.from_numpy(tokens), torch.from_numpy(cursor.copy()), cache, torch.from_numpy(offsets))
                bid = actor.policy_logits(h, "bid").float()
                card = actor.policy_logits(h, "play").float()
                values = actor.player_values(h).float()
            records.append((tokens, cursor.copy(), offsets, h.float().numpy(), bid.numpy(), card.numpy(), values.numpy()))
            cursor = cursor + counts
    return prefill_hidden, records


def make_trunk(name: str, config: dict, streams: list[np.ndarray], seed: int) -> None:
    actor = reference_actor(config, seed)
    padded, lengths = pad(streams)
    prefix = 4
    waves = ragged_schedule(lengths, prefix, seed + 1)
    out: dict[str, np.ndarray] = {
        "seed": np.int64(seed),
        "config_keys": np.array(list(config.keys())),
        "config_values": np.array([str(v) for v in config.values()]),
        "tokens": padded.astype(np.int16),
        "lengths": lengths,
        "prefix": np.int64(prefix),
        "n_waves": np.int64(len(waves)),
    }
    with torch.no_grad():
        full = actor.forward_hidden(torch.from_numpy(padded))
        out["full_hidden"] = full.numpy()
        out["full_bid"] = actor.policy_logits(full, "bid").numpy()
        out["full_card"] = actor.policy_logits(full, "play").numpy()
        out["full_values"] = actor.player_values(full).numpy()
    prefill, records = run_ragged(actor, padded, lengths, prefix, waves, torch.float32, autocast=False)
    out["prefill_hidden"] = prefill
    for i, (tokens, positions, offsets, hidden, bid, card, values) in enumerate(records):
        out[f"wave{i}_counts"] = waves[i]
        out[f"wave{i}_tokens"] = tokens.astype(np.int16)
        out[f"wave{i}_positions"] = positions
        out[f"wave{i}_offsets"] = offsets
        out[f"wave{i}_hidden"] = hidden
        out[f"wave{i}_bid"] = bid
        out[f"wave{i}_card"] = card
        out[f"wave{i}_values"] = values
    # The reference's own reduced-precision rollout (bf16 autocast, fp16 KV): its deviation
    # from fp32 is the accuracy bar a bf16 kernel has to stay within.
    _, low = run_ragged(actor, padded, lengths, prefix, waves, torch.float16, autocast=True)
    for i, (_, _, _, hidden, bid, card, values) in enumerate(low):
        out[f"wave{i}_bf16_hidden"] = hidden
        out[f"wave{i}_bf16_card"] = card
        out[f"wave{i}_bf16_bid"] = bid
        out[f"wave{i}_bf16_values"] = values
    np.savez_compressed(HERE / f"trunk_{name}.npz", **out)


def make_sampling() -> None:
    from cardgym.rl.ppo import masked_probabilities, sample_rows

    rng = np.random.default_rng(11)
    cases = {}
    for width in (11, 52, 64):
        rows = 1024
        mask = rng.random((rows, width)) < 0.3
        mask[np.arange(rows), rng.integers(0, width, rows)] = True
        logits = (rng.standard_normal((rows, width)) * 2.0).astype(np.float32)
        uniforms = rng.random(rows)
        uniforms[:8] = [0.0, 1.0, 1.0 - 1e-12, 1e-12, 0.5, 0.25, 0.75, 0.999]
        probs = masked_probabilities(logits, mask)
        cases[f"w{width}_logits"] = logits
        cases[f"w{width}_mask"] = mask
        cases[f"w{width}_uniforms"] = uniforms
        cases[f"w{width}_probs"] = probs.astype(np.float32)
        cases[f"w{width}_actions"] = sample_rows(probs, mask, uniforms).astype(np.int64)
    np.savez_compressed(HERE / "sampling.npz", **cases)


def make_ppo() -> None:
    from cardgym.rl.ppo import ppo_terms

    rng = np.random.default_rng(12)
    rows, width = 1024, 52
    legal = rng.random((rows, width)) < 0.3
    legal[np.arange(rows), rng.integers(0, width, rows)] = True
    legal[:16] = False
    legal[:16, 3] = True  # forced moves: one legal action, entropy ineligible
    old_logits = rng.standard_normal((rows, width)).astype(np.float32)
    old = torch.softmax(torch.from_numpy(old_logits).masked_fill(~torch.from_numpy(legal), float("-inf")), -1).numpy()
    old = np.where(legal, old, 0.0).astype(np.float32)
    actions = np.array([rng.choice(np.flatnonzero(old[r] > 0), p=old[r][old[r] > 0] / old[r][old[r] > 0].sum()) for r in range(rows)])
    new_logits = (old_logits + rng.normal(0.0, 0.05, (rows, width))).astype(np.float32)
    new_logits[16:64] += rng.normal(0.0, 2.0, (48, width)).astype(np.float32)  # far outside the clip range
    new_logits[64:72] = old_logits[64:72]  # ratio exactly 1
    advantages = rng.standard_normal(rows).astype(np.float32)
    advantages[72:80] = 0.0
    weights = (rng.random(rows) / rows).astype(np.float32)
    clip, alpha = 0.2, 0.05
    logits_t = torch.from_numpy(new_logits).requires_grad_()
    terms = ppo_terms(logits_t, torch.from_numpy(old), torch.from_numpy(actions), torch.from_numpy(advantages), clip_ratio=clip)
    w = torch.from_numpy(weights)
    loss = (w * terms.losses).sum()
    eligible = w * terms.entropy_eligible.float()
    objective = loss - alpha * (eligible * terms.normalized_entropy).sum()
    objective.backward()
    np.savez_compressed(
        HERE / "ppo.npz",
        logits=new_logits, old_probs=old, actions=actions.astype(np.int64), advantages=advantages, weights=weights,
        clip=np.float32(clip), alpha=np.float32(alpha),
        losses=terms.losses.detach().numpy(), divergences=terms.divergences.detach().numpy(),
        entropy=terms.entropy.detach().numpy(), normalized_entropy=terms.normalized_entropy.detach().numpy(),
        entropy_eligible=terms.entropy_eligible.numpy(), ratios=terms.ratios.detach().numpy(),
        clipped=terms.clipped.numpy(), log_probs=terms.log_probs.detach().numpy(),
        objective=np.float64(objective.item()), grad=logits_t.grad.numpy(),
    )


def make_gae() -> None:
    from cardgym.rl.ppo import gae_advantages

    rng = np.random.default_rng(13)
    games, players = 160, 4
    lengths = rng.integers(13, 53, games)
    lengths[:3] = [1, 2, 3]
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    values = rng.standard_normal((starts[-1], players))
    seats = rng.integers(0, players, starts[-1])
    returns = rng.standard_normal((games, players))
    returns -= returns.mean(axis=1, keepdims=True)
    out = {}
    for lam in (0.0, 0.95, 1.0):
        adv = np.zeros(starts[-1])
        for g in range(games):
            lo, hi = starts[g], starts[g + 1]
            a = gae_advantages(values[lo:hi], returns[g], lam)
            adv[lo:hi] = a[np.arange(hi - lo), seats[lo:hi]]
        out[f"adv_{lam}"] = adv
    np.savez_compressed(HERE / "gae.npz", values=values, seats=seats, starts=starts, returns=returns, **out)


def make_value_loss() -> None:
    from cardgym.rl.trainer import PPOTrainer

    rng = np.random.default_rng(14)
    rows, players_max = 1024, 5
    players = rng.integers(3, 6, rows)
    returns = rng.standard_normal((rows, players_max)) * (np.arange(players_max)[None, :] < players[:, None])
    prediction = torch.from_numpy(rng.standard_normal((rows, players_max)).astype(np.float32)).requires_grad_()
    weight = (rng.random(rows) / rows).astype(np.float32)
    scale = 5.0
    fake = SimpleNamespace(
        config=SimpleNamespace(value_reward_scale=scale), device=torch.device("cpu"),
        upload=lambda array: torch.from_numpy(np.asarray(array)),
    )
    dense = SimpleNamespace(
        flat=torch.arange(rows), seq=np.arange(rows), start=0, weight=torch.from_numpy(weight)
    )
    group = SimpleNamespace(player_counts=players, returns=returns.astype(np.float32))
    totals: dict = {"actor_value_loss": [], "actor_value_squared_error": [], "actor_value_target_squared": [], "actor_value_weight": []}
    from collections import defaultdict

    totals = defaultdict(list)
    loss = PPOTrainer._value_loss(fake, None, None, dense, group, totals, "actor_value", values=prediction)
    loss.backward()
    np.savez_compressed(
        HERE / "value_loss.npz", prediction=prediction.detach().numpy(), players=players, returns=returns.astype(np.float32),
        weight=weight, scale=np.float32(scale), loss=np.float64(loss.item()),
        squared_error=np.float64(totals["actor_value_squared_error"][0].item()), grad=prediction.grad.numpy(),
    )


PIQUET_BAG_WIDTHS = {"wide": (64, 128, 64), "odd": (20, 12, 6)}


def piquet_bag_tables(widths: tuple[int, ...], seed: int) -> list[np.ndarray]:
    """The synthetic field tables of the piquet lookup fixture (regenerated from the seed by the tests)."""

    from oracle.piquet import ROWS

    rng = np.random.default_rng(seed)
    return [(rng.standard_normal((ROWS, w)) * 0.02).astype(np.float32) for w in widths]


def make_piquet_bags() -> None:
    """``_onehot_bags`` and the field part of ``PiquetEmbedding.forward`` on synthetic piquet tokens."""

    from cardgym.games.piquet.model import _onehot_bags
    from cardgym.games.piquet.tokens import FIELD_VOCAB, NUM_FIELDS, WIDTH

    rng = np.random.default_rng(41)
    count = 200
    tokens = np.zeros((count, WIDTH), dtype=np.int64)
    for field, vocab in enumerate(FIELD_VOCAB):
        tokens[:, field] = rng.integers(0, vocab, count)
    tokens[:, NUM_FIELDS:] = rng.integers(0, 12, (count, WIDTH - NUM_FIELDS))
    offsets = np.array([sum(FIELD_VOCAB[:i]) for i in range(NUM_FIELDS)], dtype=np.int64)
    # Ids past their own field's rows land in the next field's: tokens 0..7 repeat a row there.
    for t in range(8):
        field = t
        tokens[t, field + 1] = t % FIELD_VOCAB[field + 1]
        tokens[t, field] = FIELD_VOCAB[field] + tokens[t, field + 1]
    ids = tokens[:, :NUM_FIELDS] + offsets
    cases = {"tokens": tokens.astype(np.int16), "seed": np.int64(43)}
    for name, widths in PIQUET_BAG_WIDTHS.items():
        tables = piquet_bag_tables(widths, 43)
        for storage, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16), ("fp16", torch.float16)):
            sums = _onehot_bags(torch.from_numpy(ids), [torch.from_numpy(t).to(dtype) for t in tables])
            for part, values in zip(("fields", "ple", "values"), sums):
                cases[f"{name}_{storage}_{part}"] = values.float().numpy()
    np.savez_compressed(HERE / "piquet_bags.npz", **cases)


def make_card_scorer() -> None:
    """``CardScorer.forward`` (piquet pointer head) in fp32 and under bf16 autocast."""

    from cardgym.games.piquet.model import CardScorer

    torch.manual_seed(51)
    scorer = CardScorer(256, 32, 64)
    with torch.no_grad():  # the init leaves the norm at 1/0 and the biases at 0: exercise them
        scorer.norm.weight.uniform_(0.5, 1.5)
        for bias in (scorer.norm.bias, scorer.query.bias, scorer.hidden.bias, scorer.out.bias):
            bias.normal_(0.0, 0.1)
    scorer.eval()
    hidden = torch.randn(48, 256)
    grid = torch.randn(48, 32, 32) * 0.5
    with torch.no_grad():
        logits = scorer(hidden, grid)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            logits_bf16 = scorer(hidden, grid.bfloat16())
    state = {f"w_{k}": v.numpy() for k, v in scorer.state_dict().items()}
    np.savez_compressed(HERE / "card_scorer.npz", hidden=hidden.numpy(), grid=grid.numpy(), logits=logits.numpy(),
                        logits_bf16=logits_bf16.float().numpy(), **state)


def make_candidate_scorer() -> None:
    """``CandidateScorer.forward`` (rummy pointer head): a draw call (with taken counts) and a play call."""

    from cardgym.games.rummy.cards import NO_CARD
    from cardgym.games.rummy.model import CandidateScorer

    torch.manual_seed(61)
    scorer = CandidateScorer(256, 32, 64)
    with torch.no_grad():
        scorer.norm.weight.uniform_(0.5, 1.5)
        for bias in (scorer.norm.bias, scorer.query.bias, scorer.hidden.bias, scorer.out.bias):
            bias.normal_(0.0, 0.1)
    scorer.eval()
    rng = np.random.default_rng(62)
    rows, width, listed = 12, 40, 13  # 40 candidates: more than one warp's worth of lanes
    hidden = torch.randn(rows, 256)
    grid = torch.randn(rows, 52, 32) * 0.5
    kind = rng.integers(0, 7, (rows, width))
    cards = np.full((rows, width, listed), NO_CARD, dtype=np.int64)
    target = np.full((rows, width, listed), NO_CARD, dtype=np.int64)
    for r in range(rows):
        for c in range(width):
            n_cards = rng.integers(0, listed + 1)
            cards[r, c, :n_cards] = rng.integers(0, 52, n_cards)  # repeats allowed: they count twice
            if rng.random() < 0.3:
                n_target = rng.integers(1, 6)
                target[r, c, :n_target] = rng.integers(0, 52, n_target)
    taken = (rng.random((rows, width, 52)) < 0.1) * rng.integers(1, 3, (rows, width, 52))
    out = {}
    with torch.no_grad():
        for name, extra in (("draw", torch.from_numpy(taken).to(torch.int8)), ("play", None)):
            logits = scorer(hidden, grid, torch.from_numpy(kind), torch.from_numpy(cards).to(torch.int8),
                            torch.from_numpy(target).to(torch.int8), extra)
            out[f"{name}_logits"] = logits.numpy()
    state = {f"w_{k}": v.numpy() for k, v in scorer.state_dict().items()}
    np.savez_compressed(HERE / "candidate_scorer.npz", hidden=hidden.numpy(), grid=grid.numpy(), kind=kind,
                        cards=cards.astype(np.int8), target=target.astype(np.int8), taken=taken.astype(np.int8),
                        **out, **state)


def make_card_grid() -> None:
    """``CardGrid.forward`` (piquet card grid: two grid blocks, final norm, summary) in fp32
    and under bf16 autocast, on random card codes."""

    from cardgym.games.piquet.model import CardGrid, PiquetModelConfig

    torch.manual_seed(71)
    grid = CardGrid(PiquetModelConfig())
    with torch.no_grad():  # exercise the gains and biases the init leaves at 1 / 0
        for block in grid.blocks:
            block.norm.weight.uniform_(0.5, 1.5)
            block.along_rank.bias.normal_(0.0, 0.05)
            block.out.bias.normal_(0.0, 0.05)
        grid.norm.weight.uniform_(0.5, 1.5)
    grid.eval()
    codes = torch.from_numpy(np.random.default_rng(72).integers(0, 12, (40, 32)))
    with torch.no_grad():
        cards, summary = grid(codes)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            cards16, summary16 = grid(codes)
    # The summary is one plain projection of the flattened cards (a library GEMM here): the
    # fixture keeps the cards, not the 1 MB summary weight.
    del summary, summary16
    state = {f"w_{k}": v.numpy() for k, v in grid.state_dict().items() if not k.startswith("summary")}
    np.savez_compressed(HERE / "card_grid.npz", codes=codes.numpy().astype(np.int8), cards=cards.numpy(),
                        cards_bf16=cards16.float().numpy(), **state)


def make_ledger_grid() -> None:
    """Rummy's ledger grid (``CardGrid`` of cardgym/games/rummy/model.py: 52 cards, 13 ranks,
    a 5-tap circular convolution) in fp32 and under bf16 autocast."""

    from cardgym.games.rummy.model import CardGrid, RummyModelConfig
    from cardgym.games.rummy.tokens import CARD_VOCAB

    torch.manual_seed(81)
    grid = CardGrid(RummyModelConfig())
    with torch.no_grad():
        for block in grid.blocks:
            block.norm.weight.uniform_(0.5, 1.5)
            block.along_rank.bias.normal_(0.0, 0.05)
            block.out.bias.normal_(0.0, 0.05)
        grid.norm.weight.uniform_(0.5, 1.5)
    grid.eval()
    codes = torch.from_numpy(np.random.default_rng(82).integers(0, CARD_VOCAB, (24, 52)))
    with torch.no_grad():
        cards = grid.cards(codes)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            cards16 = grid.cards(codes)
    state = {f"w_{k}": v.numpy() for k, v in grid.state_dict().items() if not k.startswith("summary")}
    np.savez_compressed(HERE / "ledger_grid.npz", codes=codes.numpy().astype(np.int16), cards=cards.numpy(),
                        cards_bf16=cards16.float().numpy(), **state)


PIQUET_ACTOR_CONFIG = dict(d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, per_layer_dim=8)


def make_piquet_actor() -> None:
    """The reference ``PiquetActor`` (cardgym/games/piquet/model.py:365-411) at a small trunk:
    the full causal forward of random piquet token rows (32 field ids + 32 card codes), the
    hidden state at one readout per row, every head's logits there with the readout's grid
    cards as context, and the player values; fp32. The parameters the reference initialises
    to zero (conditioning tables, biases) are drawn small so that every term carries signal."""

    from cardgym.games.piquet.model import FIELD_VOCAB, PiquetActor, PiquetModelConfig

    torch.manual_seed(91)
    model = PiquetActor(PiquetModelConfig(**PIQUET_ACTOR_CONFIG))
    with torch.no_grad():
        for param in model.parameters():
            if not param.any():
                param.normal_(0.0, 0.02)
    model.eval()
    rng = np.random.default_rng(92)
    batch, steps = 6, 12
    fields = np.stack([rng.integers(0, vocab, (batch, steps)) for vocab in FIELD_VOCAB], axis=-1)
    cards = rng.integers(0, 12, (batch, steps, 32))
    tokens = torch.from_numpy(np.concatenate([fields, cards], axis=-1).astype(np.int64))
    readouts = rng.integers(0, steps, batch)
    rows = torch.arange(batch)
    with torch.no_grad():
        hidden = model.forward_hidden(tokens)[rows, readouts]
        context = model.pop_context()[rows, readouts]
        logits = {f"logits_{head}": model.policy_logits(hidden, head, None, None, context).numpy()
                  for head in model.policy_heads}
        values = model.player_values(hidden).numpy()
    state = {f"w_{k}": v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(HERE / "piquet_actor.npz", tokens=tokens.numpy().astype(np.int16), readouts=readouts,
                        hidden=hidden.numpy(), values=values, heads=np.array(model.policy_heads),
                        config_keys=np.array(list(PIQUET_ACTOR_CONFIG)),
                        config_values=np.array([PIQUET_ACTOR_CONFIG[k] for k in PIQUET_ACTOR_CONFIG]),
                        **logits, **state)


RUMMY_ACTOR_CONFIG = dict(d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, per_layer_dim=8)


def make_rummy_actor() -> None:
    """The reference ``RummyActor`` (cardgym/games/rummy/model.py:359-402) at a small trunk: the
    full causal forward of random rummy token rows (26 field ids + a 52-card ledger), the hidden
    state at one readout per row, both heads' candidate logits there (draw with taken counts,
    play without; 9 candidates, the readout's ledger cards as context) and the player values;
    fp32. Zero-initialised parameters are drawn small so that every term carries signal."""

    from cardgym.games.rummy.cards import NO_CARD
    from cardgym.games.rummy.model import RummyActor, RummyModelConfig
    from cardgym.games.rummy.tokens import CARD_VOCAB, FIELD_VOCAB

    torch.manual_seed(101)
    model = RummyActor(RummyModelConfig(**RUMMY_ACTOR_CONFIG))
    with torch.no_grad():
        for param in model.parameters():
            if not param.any():
                param.normal_(0.0, 0.02)
    model.eval()
    rng = np.random.default_rng(102)
    batch, steps, width, listed = 5, 10, 9, 13
    fields = np.stack([rng.integers(0, vocab, (batch, steps)) for vocab in FIELD_VOCAB], axis=-1)
    ledger = rng.integers(0, CARD_VOCAB, (batch, steps, 52))
    tokens = torch.from_numpy(np.concatenate([fields, ledger], axis=-1).astype(np.int64))
    readouts = rng.integers(0, steps, batch)
    kind = rng.integers(0, 7, (batch, width))
    cards = np.full((batch, width, listed), NO_CARD, dtype=np.int64)
    target = np.full((batch, width, listed), NO_CARD, dtype=np.int64)
    for r in range(batch):
        for c in range(width):
            n_cards = rng.integers(0, listed + 1)
            cards[r, c, :n_cards] = rng.integers(0, 52, n_cards)
            if rng.random() < 0.3:
                n_target = rng.integers(1, 6)
                target[r, c, :n_target] = rng.integers(0, 52, n_target)
    taken = (rng.random((batch, width, 52)) < 0.1) * rng.integers(1, 3, (batch, width, 52))
    rows = torch.arange(batch)
    features = {"kind": torch.from_numpy(kind), "cards": torch.from_numpy(cards), "target": torch.from_numpy(target)}
    with torch.no_grad():
        hidden = model.forward_hidden(tokens)[rows, readouts]
        context = model.pop_context()[rows, readouts]
        logits_draw = model.policy_logits(hidden, "draw", {**features, "taken": torch.from_numpy(taken)}, None, context)
        logits_play = model.policy_logits(hidden, "play", features, None, context)
        values = model.player_values(hidden)
    state = {f"w_{k}": v.numpy() for k, v in model.state_dict().items()}
    np.savez_compressed(HERE / "rummy_actor.npz", tokens=tokens.numpy().astype(np.int16), readouts=readouts,
                        hidden=hidden.numpy(), values=values.numpy(), logits_draw=logits_draw.numpy(),
                        logits_play=logits_play.numpy(), kind=kind.astype(np.int8), cards=cards.astype(np.int8),
                        target=target.astype(np.int8), taken=taken.astype(np.int8),
                        field_vocab=np.array(FIELD_VOCAB), config_keys=np.array(list(RUMMY_ACTOR_CONFIG)),
                        config_values=np.array([RUMMY_ACTOR_CONFIG[k] for k in RUMMY_ACTOR_CONFIG]), **state)


def main() -> None:
    only = set(sys.argv[1:])
    if only:
        for name in sorted(only):
            globals()[f"make_{name}"]()
        return
    torch.manual_seed(0)
    streams = plump_streams(48, seed=0)
    padded, lengths = pad(streams)
    np.savez_compressed(HERE / "plump_streams.npz", tokens=padded.astype(np.int16), lengths=lengths)
    make_trunk("tiny_div", TRUNK_CONFIGS["tiny_div"], streams[:6], seed=3)
    make_trunk("tiny_cat", TRUNK_CONFIGS["tiny_cat"], streams[6:12], seed=4)
    make_trunk("rlv6", TRUNK_CONFIGS["rlv6"], streams[12:16], seed=5)
    make_sampling()
    make_ppo()
    make_gae()
    make_value_loss()
    make_piquet_bags()
    make_card_scorer()
    make_candidate_scorer()
    make_card_grid()
    make_ledger_grid()
    make_piquet_actor()
    make_rummy_actor()
    for path in sorted(HERE.glob("*.npz")):
        print(f"{path.name}: {path.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
