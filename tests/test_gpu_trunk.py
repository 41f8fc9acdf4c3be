"""Model-level parity: the B200 ragged decode against the oracle and the reference's own outputs (B200 only).

The reference fixtures hold the reference's fp32 outputs for prefill + ragged waves
(tests/golden/make_golden.py), and its own bf16-autocast / fp16-KV outputs on the same
waves, whose deviation from fp32 is the accuracy bar for the B200 bf16 mode.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
from oracle import plump as oplump
from oracle import ppo as oppo
from oracle.trunk import Precision
from tests.conftest import load_golden, trunk_fixture

pytestmark = pytest.mark.gpu

TRUNKS = ("tiny_div", "tiny_cat", "rlv6")
# fp32 mode against the reference's fp32 outputs, and bf16 mode against the oracle at the kernels'
# rounding points: max |error| / max |expected| per tensor.
FP32_TOL = 1e-5
BF16_TOL = 1e-3
# The play logits of the rl-v6 fixture's bf16 waves (4 streams, prefill + 40 ragged waves) reach 1.28e-3:
# besides fp32 summation order, the attention rounds its probabilities to the cache dtype relative to the
# running maximum of its online softmax, where the reference (and the oracle) round the final softmax.
# On the benchmarked 4,096-game wave the same logits stay at 7.4e-4 (test_gpu_bench_config.py).
BF16_FIXTURE_LOGIT_TOL = 1.5e-3


def scaled(got, expected) -> float:
    return float(np.abs(got - expected).max() / max(np.abs(expected).max(), 1e-30))


def make_actor(name: str, precision: str):
    from card_playing_gym_b200.plump import PlumpActor

    data, config = trunk_fixture(name)
    model = PlumpModelConfig(**config)
    state = synthetic_plump_actor_state(model, seed=int(data["seed"]))
    return data, config, state, PlumpActor(model, state, precision=precision)


def run_waves(actor, data, kv_dtype):
    """Prefill then every ragged wave of the fixture; yields (wave, hidden, live rows)."""

    tokens = torch.from_numpy(data["tokens"].astype(np.int64)).cuda()
    lengths = data["lengths"]
    prefix = int(data["prefix"])
    cache = actor.new_cache(len(lengths), int(lengths.max()) + 1, kv_dtype)
    hidden = actor.forward_prefill(tokens[:, :prefix], cache, None)
    yield -1, hidden, np.ones(len(lengths), dtype=bool)
    for wave in range(int(data["n_waves"])):
        hidden = actor.forward_ragged(
            torch.from_numpy(data[f"wave{wave}_tokens"]).cuda(),
            torch.from_numpy(data[f"wave{wave}_positions"]).cuda(),
            cache,
            torch.from_numpy(data[f"wave{wave}_offsets"]).cuda(),
        )
        yield wave, hidden, data[f"wave{wave}_counts"] > 0


@pytest.mark.parametrize("name", TRUNKS)
def test_fp32_ragged_decode_matches_the_reference(name):
    data, _, _, actor = make_actor(name, "fp32")
    errors = {"hidden": 0.0, "card": 0.0, "values": 0.0}
    for wave, hidden, live in run_waves(actor, data, torch.float32):
        got = hidden.cpu().numpy()
        expected = data["prefill_hidden"] if wave < 0 else data[f"wave{wave}_hidden"]
        errors["hidden"] = max(errors["hidden"], scaled(got[live], expected[live]))
        if wave >= 0:
            card = actor.policy_logits(hidden, "play").cpu().numpy()
            errors["card"] = max(errors["card"], scaled(card[live], data[f"wave{wave}_card"][live]))
            values = actor.player_values(hidden).cpu().numpy()
            errors["values"] = max(errors["values"], scaled(values[live], data[f"wave{wave}_values"][live]))
    print(f"{name} fp32 against the reference: " + ", ".join(f"{k} {v:.2e}" for k, v in errors.items()))
    assert max(errors.values()) < FP32_TOL, errors


@pytest.mark.parametrize("name", TRUNKS)
def test_fp32_ragged_decode_with_gathered_rows(name):
    """Explicit ``rows`` (the continuous collector's gathered cache rows) give the same outputs."""

    data, _, _, actor = make_actor(name, "fp32")
    lengths = data["lengths"]
    batch = len(lengths)
    rows = torch.arange(batch, device="cuda") * 3 + 1  # scattered rows of a larger pool
    tokens = torch.from_numpy(data["tokens"].astype(np.int64)).cuda()
    prefix = int(data["prefix"])
    cache = actor.new_cache(3 * batch + 1, int(lengths.max()) + 1, torch.float32)
    actor.forward_prefill(tokens[:, :prefix], cache, rows)
    for wave in range(int(data["n_waves"])):
        hidden = actor.forward_ragged(
            torch.from_numpy(data[f"wave{wave}_tokens"]).cuda(), torch.from_numpy(data[f"wave{wave}_positions"]).cuda(),
            cache, torch.from_numpy(data[f"wave{wave}_offsets"]).cuda(), rows=rows,
        )
        live = data[f"wave{wave}_counts"] > 0
        assert scaled(hidden.cpu().numpy()[live], data[f"wave{wave}_hidden"][live]) < FP32_TOL


@pytest.mark.parametrize("name", TRUNKS)
@pytest.mark.parametrize("kv", ["fp16", "bf16"])
def test_bf16_ragged_decode_tracks_the_oracle_and_beats_reference_bf16_error(name, kv):
    """bf16 GEMM operands, 16-bit KV.

    (1) Against the oracle evaluated at the same rounding points (bf16 GEMM operands,
    KV/Q/probabilities in the cache dtype): max |error| / max |value| below 1e-3 on
    hidden states and play logits (the kernels differ from it only in fp32 summation
    order, which can flip a bf16 rounding).
    (2) Against the reference's fp32 outputs: no worse than twice the reference's own
    bf16-autocast / fp16-KV rollout error on the same waves.
    """

    data, config, state, actor = make_actor(name, "bf16")
    oracle = oplump.PlumpActor(state, config, Precision(gemm="bf16", kv=kv))
    tokens = data["tokens"].astype(np.int64)
    lengths = data["lengths"]
    ocache = oracle.new_cache(len(lengths), int(lengths.max()) + 1)
    prefix = int(data["prefix"])
    # The B200 prefill is a ragged append of the whole prefix at length 0; so is the oracle's here.
    oracle.forward_ragged(tokens[:, :prefix], np.zeros(len(lengths), np.int64), ocache,
                          np.full(len(lengths), prefix - 1), span=prefix)
    mine_err, ref_err = 0.0, 0.0
    for wave, hidden, live in run_waves(actor, data, getattr(torch, {"fp16": "float16", "bf16": "bfloat16"}[kv])):
        if wave < 0:
            continue
        expected = oracle.forward_ragged(data[f"wave{wave}_tokens"].astype(np.int64), data[f"wave{wave}_positions"],
                                         ocache, data[f"wave{wave}_offsets"])
        got = hidden.cpu().numpy()
        card = actor.policy_logits(hidden, "play").cpu().numpy()
        ocard = oracle.heads.policy_logits(expected, "play")
        print(f"{name} bf16/{kv} wave {wave}: hidden {scaled(got[live], expected[live]):.2e}, "
              f"play {scaled(card[live], ocard[live]):.2e}")
        assert scaled(got[live], expected[live]) < BF16_TOL
        assert scaled(card[live], ocard[live]) < BF16_FIXTURE_LOGIT_TOL
        reference = data[f"wave{wave}_card"][live]
        mine_err = max(mine_err, float(np.abs(card[live] - reference).max()))
        ref_err = max(ref_err, float(np.abs(data[f"wave{wave}_bf16_card"][live] - reference).max()))
    assert mine_err <= 2.0 * ref_err + 1e-4, (mine_err, ref_err)


@pytest.mark.parametrize("count,gather", [(4096, False), (77, True), (1, False)])
def test_decide_matches_the_oracle_heads_and_sampler(count, gather):
    """Decisions in tiles of 32: full tiles, a ragged last tile, and hidden rows picked by index."""

    from card_playing_gym_b200.plump import PlumpActor

    config = PlumpModelConfig()
    state = synthetic_plump_actor_state(config, seed=21)
    actor = PlumpActor(config, state, precision="fp32")
    heads = oplump.Heads.from_state(state)
    rng = np.random.default_rng(4 + count)
    source = rng.standard_normal((3 * count if gather else count, config.d_model)).astype(np.float32)
    pick = rng.choice(source.shape[0], count, replace=False).astype(np.int64) if gather else None
    hidden = source[pick] if gather else source
    which = rng.integers(0, 2, count).astype(np.int32)
    legal = rng.random((count, 52)) < 0.3
    legal[np.arange(count), rng.integers(0, 11, count)] = True
    legal[which == 0, 11:] = False
    uniforms = rng.random(count)
    logits, probs, actions, values = actor.decide(
        torch.from_numpy(source).cuda(), torch.from_numpy(which).cuda(), torch.from_numpy(legal).cuda(),
        torch.from_numpy(uniforms).cuda(), torch.from_numpy(pick).cuda() if gather else None,
    )
    logits, probs, actions = logits.cpu().numpy(), probs.cpu().numpy(), actions.cpu().numpy()
    assert not np.any(logits[which == 0, 11:])  # zero past a head's width
    h64 = hidden.astype(np.float64)
    for head, width in ((0, 11), (1, 52)):
        rows = which == head
        if not rows.any():
            continue
        expected = heads.policy_logits(h64[rows], ("bid", "play")[head])
        np.testing.assert_allclose(logits[rows, :width], expected, atol=2e-5, rtol=1e-5)
        # The reference samples on the host from these same logits (selfplay.py:539-548).
        mask = legal[rows, :width]
        host = oppo.masked_probabilities(logits[rows, :width], mask)
        assert np.array_equal(probs[rows, :width].view(np.uint32), host.view(np.uint32))
        assert np.array_equal(actions[rows], oppo.sample_rows(host, mask, uniforms[rows]))
        assert mask[np.arange(mask.shape[0]), actions[rows]].all()
    np.testing.assert_allclose(values.cpu().numpy(), heads.player_values(h64), atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("precision,kv", [("fp32", "fp32"), ("bf16", "fp16")])
def test_trunk_forward_ragged_from_conditioned_inputs(precision, kv):
    """Trunk.forward_ragged's own signature (trunk.py:391-429): x, ple, values from Trunk.condition."""

    from card_playing_gym_b200.trunk import B200Trunk

    data, config, state, _ = make_actor("rlv6", "fp32")
    model = PlumpModelConfig(**config)
    trunk = B200Trunk(model.trunk(), state, precision=precision)
    oracle = oplump.PlumpActor(state, config, Precision(gemm=precision, kv=kv))
    rng = np.random.default_rng(8)
    streams = data["tokens"].astype(np.int64)
    batch = streams.shape[0]
    prefix = int(data["prefix"])
    lookup = oracle.embedding.forward(streams[:, : prefix + 2])
    x, ple, values = oracle.trunk.condition(*lookup)
    dtype = {"fp32": torch.float32, "fp16": torch.float16}[kv]
    cache = trunk.new_cache(batch, 64, dtype)
    ocache = oracle.new_cache(batch, 64)
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()  # noqa: E731
    trunk.forward_ragged(cuda(x[:, :prefix]), cuda(ple[:, :prefix]), cuda(values[:, :prefix]), cache,
                         torch.zeros(batch, dtype=torch.int64, device="cuda"),
                         torch.full((batch,), prefix - 1, dtype=torch.int64, device="cuda"), span=prefix)
    oracle.trunk.forward_ragged(x[:, :prefix], ple[:, :prefix], values[:, :prefix], ocache,
                                np.zeros(batch, np.int64), np.full(batch, prefix - 1), span=prefix)
    positions = np.full(batch, prefix, np.int64)
    offsets = rng.integers(0, 2, batch)
    hidden = trunk.forward_ragged(cuda(x[:, prefix:]), cuda(ple[:, prefix:]), cuda(values[:, prefix:]), cache,
                                  torch.from_numpy(positions).cuda(), torch.from_numpy(offsets).cuda())
    expected = oracle.trunk.forward_ragged(x[:, prefix:], ple[:, prefix:], values[:, prefix:], ocache, positions,
                                           offsets)
    error = np.abs(hidden.cpu().numpy() - expected).max() / np.abs(expected).max()
    assert error < (FP32_TOL if precision == "fp32" else BF16_TOL), error


def test_wide_trunk_bf16_decode_tracks_the_oracle():
    """A d = 256 trunk (piquet-scale dims: 8 query / 2 KV heads of 32, d_ff 512; two layers)
    through the whole bf16 path: blocked field lookup, six-chunk epilogue rows, hd-32 attention."""

    from card_playing_gym_b200.config import PIQUET_SCALE
    from card_playing_gym_b200.plump import PlumpActor

    config = dataclasses.replace(PIQUET_SCALE, n_layers=2)
    state = synthetic_plump_actor_state(config, seed=31)
    actor = PlumpActor(config, state, precision="bf16")
    oracle = oplump.PlumpActor(state, dataclasses.asdict(config), Precision(gemm="bf16", kv="fp16"))
    streams = load_golden("plump_streams")["tokens"].astype(np.int64)
    batch, length = streams.shape[:2]
    prefix = length // 2
    cache = actor.new_cache(batch, length + 1, torch.float16)
    ocache = oracle.new_cache(batch, length + 1)
    tokens = torch.from_numpy(streams).cuda()
    got = actor.forward_prefill(tokens[:, :prefix], cache, None).cpu().numpy()
    expected = oracle.forward_prefill(streams[:, :prefix], ocache, None)
    assert scaled(got, expected) < BF16_TOL
    for step in range(prefix, min(length, prefix + 3)):
        positions = np.full(batch, step, np.int64)
        offsets = np.zeros(batch, np.int64)
        got = actor.forward_ragged(tokens[:, step:step + 1], torch.from_numpy(positions).cuda(), cache,
                                   torch.from_numpy(offsets).cuda()).cpu().numpy()
        expected = oracle.forward_ragged(streams[:, step:step + 1], positions, ocache, offsets)
        assert scaled(got, expected) < BF16_TOL, step
