"""The rummy candidate pointer head (cardgym/games/rummy/model.py:292-357).

CPU: the oracle against the reference's own ``CandidateScorer`` outputs (tests/golden/candidate_scorer.npz,
a draw call with taken counts and a play call without). GPU: ``cg_candidate_scorer`` against the
same outputs (40 candidates per decision: more than one warp of lanes), bad ids flagged.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import rummy as orummy
from tests.conftest import load_golden


def _weights(data: dict) -> dict:
    return {k[2:]: v for k, v in data.items() if k.startswith("w_")}


def _inputs(data: dict, head: str):
    taken = data["taken"].astype(np.float64) if head == "draw" else None
    return (data["hidden"], data["grid"], data["kind"].astype(np.int64), data["cards"].astype(np.int64),
            data["target"].astype(np.int64), taken)


@pytest.mark.parametrize("head", ("draw", "play"))
def test_oracle_matches_the_reference_scorer(head):
    data = load_golden("candidate_scorer")
    got = orummy.candidate_scorer(*_inputs(data, head), _weights(data))
    np.testing.assert_allclose(got, data[f"{head}_logits"], atol=1e-6, rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("head", ("draw", "play"))
def test_candidate_scorer_matches_the_reference(head):
    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.rummy import CandidateScorer

    data = load_golden("candidate_scorer")
    scorer = CandidateScorer(_weights(data))
    hidden, grid, kind, cards, target, taken = _inputs(data, head)
    cuda = lambda a: None if a is None else torch.from_numpy(a).cuda()  # noqa: E731
    assert nat.fault_status() == 0
    logits = scorer(cuda(hidden), cuda(grid), cuda(kind), cuda(data["cards"]), cuda(data["target"]),
                    None if taken is None else cuda(data["taken"]))
    np.testing.assert_allclose(logits.cpu().numpy(), data[f"{head}_logits"], atol=3e-6, rtol=0)
    # bf16 grid: against the oracle on the same rounded grid
    half = scorer(cuda(hidden), cuda(grid).bfloat16(), cuda(kind), cuda(cards), cuda(target),
                  None if taken is None else cuda(taken))
    want = orummy.candidate_scorer(hidden, cuda(grid).bfloat16().float().cpu().numpy(), kind, cards, target, taken,
                                   _weights(data))
    np.testing.assert_allclose(half.cpu().numpy(), want, atol=3e-6, rtol=0)
    assert nat.fault_status() == 0


@pytest.mark.gpu
def test_candidate_scorer_flags_bad_ids():
    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.rummy import CandidateScorer

    data = load_golden("candidate_scorer")
    scorer = CandidateScorer(_weights(data))
    hidden, grid, kind, cards, target, _ = _inputs(data, "play")
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    for field, value, code in (("cards", 53, 0x220), ("cards", -1, 0x220), ("kind", 7, 0x221)):
        bad_cards, bad_kind = cards.copy(), kind.copy()
        if field == "cards":
            bad_cards[1, 2, 0] = value
        else:
            bad_kind[1, 2] = value
        scorer(cuda(hidden), cuda(grid), cuda(bad_kind), cuda(bad_cards), cuda(target))
        assert nat.fault_status() == code


def _ledger_weights(data: dict) -> dict:
    return {k[2:]: v for k, v in data.items() if k.startswith("w_")}


def test_ledger_grid_oracle_matches_the_reference():
    from oracle import piquet as opiquet

    data = load_golden("ledger_grid")
    cards, _ = opiquet.card_grid(data["codes"], _ledger_weights(data), kernel=5, ranks=13, circular=True)
    np.testing.assert_allclose(cards, data["cards"], atol=1e-5, rtol=0)


@pytest.mark.gpu
def test_ledger_grid_matches_the_reference_autocast_form():
    """Rummy's ledger grid (52 cards, circular 5-tap convolution) through cg_card_grid: as close to
    the reference's bf16-autocast result as one bf16 step of a rare tie-rounded intermediate."""

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.piquet import CardGrid
    from oracle import piquet as opiquet

    data = load_golden("ledger_grid")
    weights = _ledger_weights(data)
    grid = CardGrid(weights)
    assert nat.fault_status() == 0
    tokens = np.zeros((data["codes"].shape[0], 78), dtype=np.int16)
    tokens[:, 26:] = data["codes"]  # the ledger codes sit after rummy's 26 token fields
    cards = grid.cards(torch.from_numpy(tokens).cuda()[:, 26:]).cpu().numpy()
    want16, fp32 = data["cards_bf16"], data["cards"]
    assert cards.shape == fp32.shape
    assert np.abs(cards - want16).max() <= np.abs(want16 - fp32).max()
    assert np.abs(cards - want16).mean() < 0.1 * np.abs(want16 - fp32).mean()
    oracle16, _ = opiquet.card_grid(data["codes"], weights, kernel=5, ranks=13, circular=True, storage="bf16")
    diff = np.abs(cards - oracle16)
    assert (diff > 1e-5).mean() < 0.02 and diff.mean() < 1e-4
    assert nat.fault_status() == 0


def test_rummy_field_vocabulary_matches_the_reference():
    """The restated token layout (cardgym/games/rummy/tokens.py:87-124) against the reference's own."""

    from card_playing_gym_b200 import rummy

    data = load_golden("rummy_actor")
    assert rummy.FIELD_VOCAB == tuple(int(v) for v in data["field_vocab"])
    assert len(rummy.FIELD_VOCAB) == rummy.NUM_FIELDS == rummy.CARD_START
    assert data["tokens"].shape[-1] == rummy.CARD_START + 52
    assert int(data["tokens"][..., rummy.CARD_START:].max()) < rummy.CARD_VOCAB


@pytest.mark.gpu
@pytest.mark.parametrize("precision,kv,tol", [("fp32", torch.float32, 2e-2), ("bf16", torch.float16, 5e-2)])
def test_rummy_actor_matches_the_reference_actor(precision, kv, tol):
    """``RummyActor`` against the reference's own (cardgym/games/rummy/model.py:359-402, fp32): the
    hidden state at each row's readout after a 10-token prefill, both heads' candidate logits
    (draw with taken counts, play without) with the readout's ledger cards as context, the
    player values. Tolerance as for the piquet actor: the ledger cards are always in the
    reference's bf16-autocast rounding here."""

    from card_playing_gym_b200.rummy import RummyActor, RummyModelConfig

    data = load_golden("rummy_actor")
    config = RummyModelConfig(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    actor = RummyActor(config, {k[2:]: v for k, v in data.items() if k.startswith("w_")}, precision=precision)
    tokens = torch.from_numpy(data["tokens"].astype(np.int64)).cuda()
    batch, steps, _ = tokens.shape
    readouts = torch.from_numpy(data["readouts"]).cuda()
    cache = actor.new_cache(batch, steps + 1, kv)
    hidden = actor.forward_ragged(tokens, torch.zeros(batch, dtype=torch.int64, device="cuda"), cache, readouts,
                                  span=steps)
    context = actor.pop_context()[torch.arange(batch, device="cuda"), readouts]
    features = {name: torch.from_numpy(data[name].astype(np.int64)).cuda() for name in ("kind", "cards", "target")}

    def scaled(got, want):
        return float(np.abs(got - want).max() / np.abs(want).max())

    assert scaled(hidden.cpu().numpy(), data["hidden"]) < tol
    draw = actor.policy_logits(hidden, "draw", {**features, "taken": torch.from_numpy(data["taken"]).cuda()},
                               None, context)
    assert scaled(draw.cpu().numpy(), data["logits_draw"]) < tol
    play = actor.policy_logits(hidden, "play", features, None, context)
    assert scaled(play.cpu().numpy(), data["logits_play"]) < tol
    assert scaled(actor.player_values(hidden).cpu().numpy(), data["values"]) < tol
    with pytest.raises(ValueError):
        actor.policy_logits(hidden, "play", None, None, context)


@pytest.mark.parametrize("name", ("piquet_actor", "rummy_actor"))
def test_synthetic_actor_states_have_the_reference_names_and_shapes(name):
    """The bench's synthetic piquet and rummy actor weights carry exactly the reference actors'
    parameter names and shapes (their fixtures' state dicts), less the heads a rollout never
    reads (piquet's auxiliary head, rummy's belief heads)."""

    from card_playing_gym_b200 import piquet, rummy

    data = load_golden(name)
    module = piquet if name == "piquet_actor" else rummy
    config_cls = piquet.PiquetModelConfig if module is piquet else rummy.RummyModelConfig
    make = piquet.synthetic_piquet_actor_state if module is piquet else rummy.synthetic_rummy_actor_state
    config = config_cls(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    state = make(config, seed=1)
    reference = {k[2:]: data[k].shape for k in data if k.startswith("w_")}
    unused = {k for k in reference if k.split(".")[0] in ("auxiliary_head", "hands_head", "winner_head", "penalty_head")}
    assert set(state) == set(reference) - unused
    assert all(tuple(state[k].shape) == tuple(reference[k]) for k in state)
