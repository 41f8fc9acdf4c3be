"""Pin the CPU oracle to the reference: its golden vectors and fixtures the reference produced.

CPU only. The rl-v6 release test needs the reference checkout's checkpoint and skips
without it; every other case reads committed fixtures from tests/golden/.
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
from card_playing_gym_b200.plump_schema import PlumpSchema
from oracle import plump as oplump
from oracle import ppo as oppo
from oracle.trunk import Precision
from tests.conftest import load_golden, trunk_fixture

REFERENCE = Path(os.environ.get("CARDGYM_REFERENCE", "/root/reference"))
TRUNKS = ("tiny_div", "tiny_cat", "rlv6")


def oracle_actor(name: str, prec: Precision | None = None):
    data, config = trunk_fixture(name)
    state = synthetic_plump_actor_state(PlumpModelConfig(**config), seed=int(data["seed"]))
    return data, config, oplump.PlumpActor(state, config, prec)


def test_schema_matches_the_oracle_restatement():
    schema = PlumpSchema()
    sizes, na = oplump.schema_tables()
    assert schema.base_vocab_sizes == sizes
    assert schema.base_na_ids == na
    assert schema.field_rows() == 205


@pytest.mark.parametrize("name", TRUNKS)
def test_full_forward_matches_the_reference(name):
    data, _, actor = oracle_actor(name)
    tokens = data["tokens"].astype(np.int64)
    hidden = actor.forward_hidden(tokens)
    np.testing.assert_allclose(hidden, data["full_hidden"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(actor.heads.policy_logits(hidden, "bid"), data["full_bid"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(actor.heads.policy_logits(hidden, "play"), data["full_card"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(actor.heads.player_values(hidden), data["full_values"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", TRUNKS)
def test_prefill_and_ragged_waves_match_the_reference(name):
    data, _, actor = oracle_actor(name, Precision(kv="fp32"))
    tokens = data["tokens"].astype(np.int64)
    lengths = data["lengths"]
    prefix = int(data["prefix"])
    cache = actor.new_cache(len(lengths), int(lengths.max()) + 1)
    hidden = actor.forward_prefill(tokens[:, :prefix], cache, None)
    np.testing.assert_allclose(hidden, data["prefill_hidden"], rtol=1e-5, atol=1e-5)
    for wave in range(int(data["n_waves"])):
        counts = data[f"wave{wave}_counts"]
        hidden = actor.forward_ragged(
            data[f"wave{wave}_tokens"].astype(np.int64), data[f"wave{wave}_positions"], cache, data[f"wave{wave}_offsets"]
        )
        live = counts > 0
        np.testing.assert_allclose(hidden[live], data[f"wave{wave}_hidden"][live], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(
            actor.heads.policy_logits(hidden, "play")[live], data[f"wave{wave}_card"][live], rtol=1e-5, atol=1e-5
        )


def test_ragged_decode_equals_the_full_forward():
    """The reference's own property (tests/nn/test_trunk.py:38-78): cached steps reproduce the full forward."""

    data, _, actor = oracle_actor("tiny_cat")
    tokens = data["tokens"].astype(np.int64)
    full = actor.forward_hidden(tokens)
    lengths = data["lengths"]
    cache = actor.new_cache(len(lengths), int(lengths.max()) + 1)
    prefix = int(data["prefix"])
    actor.forward_prefill(tokens[:, :prefix], cache, None)
    cursor = np.full(len(lengths), prefix)
    for wave in range(int(data["n_waves"])):
        counts = data[f"wave{wave}_counts"]
        hidden = actor.forward_ragged(
            data[f"wave{wave}_tokens"].astype(np.int64), cursor, cache, data[f"wave{wave}_offsets"]
        )
        for row in np.flatnonzero(counts):
            np.testing.assert_allclose(hidden[row], full[row, cursor[row] + counts[row] - 1], rtol=1e-9, atol=1e-9)
        cursor = cursor + counts


@pytest.mark.skipif(
    not (REFERENCE / "checkpoints/plump/rl-v6/actor.pt").exists(), reason="needs the reference checkout's rl-v6 release"
)
def test_rl_v6_release_reproduces_the_reference_golden_vectors():
    """tests/plump/test_plump_release.py:38-49 of the reference, on the oracle."""

    import torch

    checkpoint = torch.load(REFERENCE / "checkpoints/plump/rl-v6/actor.pt", map_location="cpu", weights_only=False)
    state = {key: value.numpy() for key, value in checkpoint["state_dict"].items()}
    actor = oplump.PlumpActor(state, dict(checkpoint["model"]))
    golden = np.load(REFERENCE / "tests/fixtures/plump_rl_v6_golden.npz")
    hidden = actor.forward_hidden(golden["tokens"].astype(np.int64))
    bid = actor.heads.policy_logits(hidden, "bid")
    card = actor.heads.policy_logits(hidden, "play")
    values = actor.heads.player_values(hidden)
    for row, length in enumerate(golden["lengths"]):
        np.testing.assert_allclose(bid[row, :length], golden["bid_logits"][row, :length], atol=2e-4)
        np.testing.assert_allclose(card[row, :length], golden["card_logits"][row, :length], atol=2e-4)
        np.testing.assert_allclose(values[row, :length], golden["actor_values"][row, :length], atol=2e-4)


@pytest.mark.parametrize("width", (11, 52, 64))
def test_masked_sampling_is_bit_exact(width):
    data = load_golden("sampling")
    logits, mask, uniforms = data[f"w{width}_logits"], data[f"w{width}_mask"], data[f"w{width}_uniforms"]
    probs = oppo.masked_probabilities(logits, mask)
    assert np.array_equal(probs, data[f"w{width}_probs"])
    actions = oppo.sample_rows(probs, mask, uniforms)
    assert np.array_equal(actions, data[f"w{width}_actions"])
    assert mask[np.arange(len(actions)), actions].all()


def test_ppo_terms_and_gradient_match_autograd():
    data = load_golden("ppo")
    terms, objective, grad = oppo.policy_objective(
        data["logits"], data["old_probs"], data["actions"], data["advantages"], data["weights"],
        float(data["clip"]), float(data["alpha"]),
    )
    for key in ("losses", "divergences", "entropy", "normalized_entropy", "ratios", "log_probs"):
        np.testing.assert_allclose(terms[key], data[key], rtol=1e-5, atol=1e-6, err_msg=key)
    assert np.array_equal(terms["entropy_eligible"], data["entropy_eligible"])
    assert np.array_equal(terms["clipped"], data["clipped"])
    assert objective == pytest.approx(float(data["objective"]), rel=1e-5, abs=1e-8)
    np.testing.assert_allclose(grad, data["grad"], rtol=1e-4, atol=1e-8)


@pytest.mark.parametrize("lam", (0.0, 0.95, 1.0))
def test_segmented_gae_is_bit_exact(lam):
    data = load_golden("gae")
    adv = oppo.segmented_gae(data["values"], data["seats"], data["starts"], data["returns"], lam)
    assert np.array_equal(adv, data[f"adv_{lam}"])


def test_gae_known_answers():
    """tests/rl/test_rl.py:58-64 of the reference: lambda 1 is Monte Carlo, lambda 0 one-step TD."""

    values = np.array([[1.0, -1.0], [3.0, -3.0], [2.0, -2.0]])
    returns = np.array([5.0, -5.0])
    np.testing.assert_allclose(oppo.gae_advantages(values, returns, 1.0), returns - values)
    one_step = oppo.gae_advantages(values, returns, 0.0)
    np.testing.assert_allclose(one_step[0], values[1] - values[0])
    np.testing.assert_allclose(one_step[2], returns - values[2])


def test_value_loss_and_gradient_match_autograd():
    data = load_golden("value_loss")
    loss, squared, grad = oppo.value_loss(data["prediction"], data["players"], data["returns"], data["weight"], float(data["scale"]))
    assert loss == pytest.approx(float(data["loss"]), rel=1e-5)
    assert squared == pytest.approx(float(data["squared_error"]), rel=1e-5)
    np.testing.assert_allclose(grad, data["grad"], rtol=1e-4, atol=1e-9)
