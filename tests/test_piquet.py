"""The piquet field lookup (cardgym/games/piquet/model.py:255-264, 323-345).

CPU: the oracle against the reference's own ``_onehot_bags`` outputs (tests/golden/piquet_bags.npz),
the host module's field layout against the oracle's, and the C ABI's argument checks.
GPU: ``cg_onehot_bags`` against the same golden outputs in fp32, bf16 and fp16 (vector and
scalar paths), repeated rows counted once, out-of-range ids flagged, strided token rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import piquet as opiquet
from tests.conftest import load_golden
from tests.golden.make_golden import PIQUET_BAG_WIDTHS, piquet_bag_tables

ULP = {"bf16": 2.0 ** -8, "fp16": 2.0 ** -11}
TORCH = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def _close_to_golden(got: np.ndarray, want: np.ndarray, storage: str) -> None:
    """fp32: a few ulp of fp32 (summation order). bf16/fp16: at most one ulp of the storage
    type, and nearly everything identical (only sums within an fp32 rounding of a midpoint differ)."""

    if storage == "fp32":
        np.testing.assert_allclose(got, want, atol=1e-6, rtol=0)
        return
    diff = np.abs(got.astype(np.float64) - want.astype(np.float64))
    scale = np.maximum(np.abs(want.astype(np.float64)), 2.0 ** -14)
    assert (diff <= ULP[storage] * scale + 1e-12).all()
    assert (diff == 0).mean() > 0.99


@pytest.mark.parametrize("name", sorted(PIQUET_BAG_WIDTHS))
@pytest.mark.parametrize("storage", ("fp32", "bf16", "fp16"))
def test_oracle_matches_the_reference_lookup(name, storage):
    data = load_golden("piquet_bags")
    tables = piquet_bag_tables(PIQUET_BAG_WIDTHS[name], int(data["seed"]))
    sums = opiquet.field_sums(data["tokens"].astype(np.int64), tables, storage)
    for part, got in zip(("fields", "ple", "values"), sums):
        _close_to_golden(got, data[f"{name}_{storage}_{part}"], storage)


def test_repeated_rows_count_once_in_the_oracle():
    tables = [np.ones((opiquet.ROWS, 3), dtype=np.float32)]
    ids = np.array([[5, 5, 7], [1, 2, 3]], dtype=np.int64)
    (sums,) = opiquet.onehot_bags(ids, tables)
    assert sums[:, 0].tolist() == [2.0, 3.0]


def test_host_field_layout_matches_the_oracle():
    from card_playing_gym_b200 import piquet

    assert piquet.FIELD_VOCAB == opiquet.FIELD_VOCAB
    assert piquet.field_offsets() == opiquet.OFFSETS.tolist()
    assert piquet.FIELD_ROWS == opiquet.ROWS


def test_bags_argument_checks():
    from card_playing_gym_b200 import _native as nat

    with pytest.raises(nat.NativeError, match="fields"):
        nat.call("cg_onehot_bags", None, nat.CG_I64, 4, 40, 40, None, None, nat.CG_F32, 10, 8, None, None)
    with pytest.raises(nat.NativeError, match="stride"):
        nat.call("cg_onehot_bags", None, nat.CG_I64, 4, 2, 3, None, None, nat.CG_F32, 10, 8, None, None)
    with pytest.raises(nat.NativeError, match="dtype"):
        nat.call("cg_onehot_bags", None, nat.CG_I64, 4, 3, 3, None, None, 7, 10, 8, None, None)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(PIQUET_BAG_WIDTHS))
@pytest.mark.parametrize("storage", ("fp32", "bf16", "fp16"))
def test_field_lookup_matches_the_reference(name, storage):
    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.piquet import PiquetFieldLookup, onehot_bags

    data = load_golden("piquet_bags")
    tables = [torch.from_numpy(t).cuda() for t in piquet_bag_tables(PIQUET_BAG_WIDTHS[name], int(data["seed"]))]
    tokens = torch.from_numpy(data["tokens"]).cuda()  # int16, the collector's storage
    assert nat.fault_status() == 0
    lookup = PiquetFieldLookup(*[t.to(TORCH[storage]) for t in tables])
    sums = lookup(tokens)
    for part, got in zip(("fields", "ple", "values"), sums):
        _close_to_golden(got.float().cpu().numpy(), data[f"{name}_{storage}_{part}"], storage)
    # The reference's call form: offset ids in, one list of sums out; int64 ids give the same sums.
    ids = tokens[:, : opiquet.NUM_FIELDS].long() + torch.tensor(opiquet.OFFSETS, device="cuda")
    again = onehot_bags(ids, [t.to(TORCH[storage]) for t in tables])
    for a, b in zip(sums, again):
        assert torch.equal(a, b)
    assert nat.fault_status() == 0


@pytest.mark.gpu
def test_field_lookup_under_autocast_uses_the_autocast_dtype():
    from card_playing_gym_b200.piquet import onehot_bags

    data = load_golden("piquet_bags")
    tables = [torch.from_numpy(t).cuda() for t in piquet_bag_tables(PIQUET_BAG_WIDTHS["wide"], int(data["seed"]))]
    ids = torch.from_numpy(data["tokens"][:, : opiquet.NUM_FIELDS].astype(np.int64) + opiquet.OFFSETS).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        sums = onehot_bags(ids, tables)
    assert all(s.dtype == torch.bfloat16 for s in sums)
    for part, got in zip(("fields", "ple", "values"), sums):
        _close_to_golden(got.float().cpu().numpy(), data[f"wide_bf16_{part}"], "bf16")


@pytest.mark.gpu
def test_field_lookup_counts_repeated_rows_once_and_flags_bad_ids():
    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.piquet import onehot_bags

    table = torch.arange(40 * 8, dtype=torch.float32, device="cuda").view(40, 8) / 64
    ids = torch.tensor([[3, 3, 3, 9], [0, 1, 2, 39]], device="cuda")
    (sums,) = onehot_bags(ids, [table])
    want = torch.stack([table[3] + table[9], table[0] + table[1] + table[2] + table[39]])
    assert torch.equal(sums, want)
    assert nat.fault_status() == 0
    for bad in (40, -1, 1 << 40):
        onehot_bags(torch.tensor([[1, bad]], device="cuda"), [table])
        assert nat.fault_status() == 0x210


@pytest.mark.gpu
def test_field_lookup_at_piquet_scale_matches_the_oracle():
    """A wave's worth of tokens (4,096) against the full-width tables (d 256, PLE 16 x 64, values 8 x 64)."""

    from card_playing_gym_b200.piquet import PiquetFieldLookup

    rng = np.random.default_rng(5)
    tokens = np.zeros((4096, 64), dtype=np.int64)
    for field, vocab in enumerate(opiquet.FIELD_VOCAB):
        tokens[:, field] = rng.integers(0, vocab, tokens.shape[0])
    tables = [(rng.standard_normal((opiquet.ROWS, w)) * 0.02).astype(np.float32) for w in (256, 1024, 512)]
    lookup = PiquetFieldLookup(*[torch.from_numpy(t).cuda().to(torch.bfloat16) for t in tables])
    got = lookup(torch.from_numpy(tokens).cuda())
    sample = slice(0, 4096, 37)
    want = opiquet.field_sums(tokens[sample], tables, "bf16")
    for g, w in zip(got, want):
        _close_to_golden(g[sample].float().cpu().numpy(), w.astype(np.float32), "bf16")


def _scorer_weights(data: dict) -> dict:
    return {k[2:]: v for k, v in data.items() if k.startswith("w_")}


def test_card_scorer_oracle_matches_the_reference():
    data = load_golden("card_scorer")
    got = opiquet.card_scorer(data["hidden"], data["grid"], _scorer_weights(data))
    np.testing.assert_allclose(got, data["logits"], atol=1e-6, rtol=0)


@pytest.mark.gpu
def test_card_scorer_matches_the_reference():
    from card_playing_gym_b200.piquet import CardScorer

    data = load_golden("card_scorer")
    scorer = CardScorer(_scorer_weights(data))
    hidden = torch.from_numpy(data["hidden"]).cuda()
    grid = torch.from_numpy(data["grid"]).cuda()
    logits = scorer(hidden, grid).cpu().numpy()
    np.testing.assert_allclose(logits, data["logits"], atol=2e-6, rtol=0)
    # A bf16 grid (the card grid's output under autocast): the kernel's arithmetic stays fp32,
    # so against the reference's fp32 logits it is no worse than the reference's own bf16 autocast.
    half = scorer(hidden, grid.bfloat16()).cpu().numpy()
    want = opiquet.card_scorer(data["hidden"], grid.bfloat16().float().cpu().numpy(), _scorer_weights(data))
    np.testing.assert_allclose(half, want, atol=2e-6, rtol=0)
    assert np.abs(half - data["logits"]).max() <= np.abs(data["logits_bf16"] - data["logits"]).max()


@pytest.mark.gpu
def test_card_scorer_at_wave_size_matches_the_oracle():
    from card_playing_gym_b200.piquet import CardScorer

    data = load_golden("card_scorer")
    weights = _scorer_weights(data)
    rng = np.random.default_rng(8)
    hidden = rng.standard_normal((4096, 256)).astype(np.float32)
    grid = (rng.standard_normal((4096, 32, 32)) * 0.5).astype(np.float32)
    logits = CardScorer(weights)(torch.from_numpy(hidden).cuda(), torch.from_numpy(grid).cuda()).cpu().numpy()
    sample = slice(0, 4096, 29)
    np.testing.assert_allclose(logits[sample], opiquet.card_scorer(hidden[sample], grid[sample], weights), atol=2e-6,
                               rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ("bf16", "fp32"))
def test_piquet_decode_with_the_fused_lookup_tracks_the_oracle(precision):
    """Field sums + a card-grid summary -> Trunk.condition -> ragged decode, against the oracle
    trunk fed with the oracle's field sums (d 256 piquet trunk, two layers, empty cache, four
    one-token waves). bf16: the fused lookup writes the first tensor-core layer's inputs."""

    import dataclasses

    from card_playing_gym_b200.config import PIQUET_SCALE, synthetic_plump_actor_state
    from card_playing_gym_b200.piquet import PiquetFieldLookup, forward_ragged
    from card_playing_gym_b200.trunk import B200Trunk
    from oracle.trunk import Cache, Precision, Trunk, TrunkShape, TrunkWeights, value_layers

    config = dataclasses.replace(PIQUET_SCALE, n_layers=2)
    state = synthetic_plump_actor_state(config, seed=33)
    tc = config.trunk()
    trunk = B200Trunk(tc, state, precision=precision)
    shape = TrunkShape(d_model=tc.d_model, n_layers=tc.n_layers, n_heads=tc.n_heads, n_kv_heads=tc.n_kv_heads,
                       d_ff=tc.d_ff, per_layer_dim=tc.per_layer_dim,
                       value_layers=value_layers(tc.n_layers, config.value_embeddings))
    prec = Precision(gemm="bf16", kv="fp16") if precision == "bf16" else Precision()
    oracle = Trunk(TrunkWeights.from_state(state, shape), prec)
    rng = np.random.default_rng(12)
    batch, waves = 24, 4
    tokens = np.zeros((batch, waves, 64), dtype=np.int64)
    for field, vocab in enumerate(opiquet.FIELD_VOCAB):
        tokens[..., field] = rng.integers(0, vocab, (batch, waves))
    tables = [(rng.standard_normal((opiquet.ROWS, w)) * 0.02).astype(np.float32)
              for w in (tc.d_model, tc.ple_width, tc.value_width)]
    summary = (rng.standard_normal((batch, waves, tc.d_model)) * 0.05).astype(np.float32)
    lookup = PiquetFieldLookup(*[torch.from_numpy(t).cuda() for t in tables])
    kv = torch.float16 if precision == "bf16" else torch.float32
    cache = trunk.new_cache(batch, waves + 1, kv)
    ocache = Cache(shape.n_layers, batch, shape.n_kv_heads, waves + 1, shape.head_dim, prec)
    offsets = np.zeros(batch, np.int64)
    tol = 1e-2 if precision == "bf16" else 5e-5
    for t in range(waves):
        positions = np.full(batch, t, np.int64)
        got = forward_ragged(trunk, lookup, torch.from_numpy(tokens[:, t:t + 1]).cuda(),
                             torch.from_numpy(positions).cuda(), cache, torch.from_numpy(offsets).cuda(),
                             summary=torch.from_numpy(summary[:, t:t + 1]).cuda()).cpu().numpy()
        fields, ple, values = opiquet.field_sums(tokens[:, t:t + 1], tables)
        x, ple, values = oracle.condition(fields + summary[:, t:t + 1], ple, values)
        want = oracle.forward_ragged(x, ple, values, ocache, positions, offsets)
        err = np.abs(got - want).max()
        assert (err / np.abs(want).max() < tol) if precision == "bf16" else err < tol, (t, err)


def _grid_weights(data: dict) -> dict:
    return {k[2:]: v for k, v in data.items() if k.startswith("w_")}


def test_card_grid_oracle_matches_the_reference():
    data = load_golden("card_grid")
    cards, _ = opiquet.card_grid(data["codes"], _grid_weights(data))
    np.testing.assert_allclose(cards, data["cards"], atol=1e-5, rtol=0)
    # The bf16-autocast form: the oracle rounds where the reference does.
    cards16, _ = opiquet.card_grid(data["codes"], _grid_weights(data), storage="bf16")
    assert np.abs(cards16 - data["cards_bf16"]).max() < 2e-3 < np.abs(data["cards_bf16"] - data["cards"]).max()


@pytest.mark.gpu
def test_card_grid_matches_the_reference_autocast_form():
    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.piquet import CardGrid

    data = load_golden("card_grid")
    grid = CardGrid(_grid_weights(data))
    assert nat.fault_status() == 0
    # The codes as a slice of token rows (stride 64), the collector's int16 storage.
    tokens = np.zeros((data["codes"].shape[0], 64), dtype=np.int16)
    tokens[:, 32:] = data["codes"]
    cards = grid.cards(torch.from_numpy(tokens).cuda()[:, 32:]).cpu().numpy()
    want16, fp32 = data["cards_bf16"], data["cards"]
    # bf16 rounding points as the reference's autocast: no farther from its autocast result
    # than that result is from fp32 (an intermediate that rounds the other way at a bf16 tie
    # moves a few features by one bf16 step), and on average far closer.
    assert np.abs(cards - want16).max() <= np.abs(want16 - fp32).max()
    assert np.abs(cards - want16).mean() < 0.1 * np.abs(want16 - fp32).mean()
    assert np.abs(cards - fp32).max() <= 1.5 * np.abs(want16 - fp32).max()
    assert nat.fault_status() == 0
    # Out-of-vocabulary codes are flagged.
    bad = tokens.copy()
    bad[3, 40] = 12
    grid.cards(torch.from_numpy(bad).cuda()[:, 32:])
    assert nat.fault_status() == 0x230


@pytest.mark.gpu
def test_card_grid_at_wave_size_matches_the_oracle():
    from card_playing_gym_b200.piquet import CardGrid

    data = load_golden("card_grid")
    weights = _grid_weights(data)
    codes = np.random.default_rng(4).integers(0, 12, (4096, 32))
    cards = CardGrid(weights)(torch.from_numpy(codes).cuda())[0].cpu().numpy()
    sample = slice(0, 4096, 41)
    want, _ = opiquet.card_grid(codes[sample], weights, storage="bf16")
    diff = np.abs(cards[sample] - want)
    # Identical roundings but for the rare intermediate at a bf16 tie (fp32 sums here, exact
    # ones in the oracle), which moves a token's features by about one bf16 step.
    assert (diff > 1e-5).mean() < 0.02 and diff.mean() < 1e-4 and diff.max() < 0.04


def _piquet_actor(precision: str):
    from card_playing_gym_b200.piquet import PiquetActor, PiquetModelConfig

    data = load_golden("piquet_actor")
    config = PiquetModelConfig(**{str(k): int(v) for k, v in zip(data["config_keys"], data["config_values"])})
    state = {k[2:]: v for k, v in data.items() if k.startswith("w_")}
    return data, PiquetActor(config, state, precision=precision)


@pytest.mark.gpu
@pytest.mark.parametrize("precision,kv,tol", [("fp32", torch.float32, 2e-2), ("bf16", torch.float16, 5e-2)])
def test_piquet_actor_matches_the_reference_actor(precision, kv, tol):
    """``PiquetActor`` against the reference's own (cardgym/games/piquet/model.py:365-411, fp32):
    hidden state at each row's readout after a 12-token prefill, every head's logits with the
    readout's grid cards as context, the player values. The tolerance (max |error| / max |value|)
    covers the grid cards, which are always in the reference's bf16-autocast rounding here,
    and in bf16 mode the trunk's bf16 GEMM operands and fp16 KV."""

    data, actor = _piquet_actor(precision)
    tokens = torch.from_numpy(data["tokens"].astype(np.int64)).cuda()
    batch, steps, _ = tokens.shape
    readouts = torch.from_numpy(data["readouts"]).cuda()
    cache = actor.new_cache(batch, steps + 1, kv)
    hidden = actor.forward_ragged(tokens, torch.zeros(batch, dtype=torch.int64, device="cuda"), cache, readouts,
                                  span=steps)
    context = actor.pop_context()[torch.arange(batch, device="cuda"), readouts]
    assert actor.pop_context() is None

    def scaled(got, want):
        return float(np.abs(got - want).max() / np.abs(want).max())

    assert scaled(hidden.cpu().numpy(), data["hidden"]) < tol
    for head in actor.policy_heads:
        logits = actor.policy_logits(hidden, head, None, None, context).cpu().numpy()
        assert logits.shape == data[f"logits_{head}"].shape
        assert scaled(logits, data[f"logits_{head}"]) < tol, head
    assert scaled(actor.player_values(hidden).cpu().numpy(), data["values"]) < tol
    with pytest.raises(ValueError):
        actor.policy_logits(hidden, "bid")


@pytest.mark.gpu
def test_piquet_actor_decode_graphs_match_the_eager_wave():
    """A piquet wave captured by ``DecodeGraphs`` (card grid, fused lookup + trunk, the card
    scorers fed the readout's grid cards) replays the eager calls bit for bit."""

    from card_playing_gym_b200.graphs import DecodeGraphs

    data, actor = _piquet_actor("bf16")
    streams = data["tokens"].astype(np.int64)
    batch = streams.shape[0]
    graph_cache = actor.new_cache(batch + 1, 16, torch.float16)
    eager_cache = actor.new_cache(batch + 1, 16, torch.float16)
    graphs = DecodeGraphs(actor, graph_cache, values=True)
    cache_rows = np.arange(1, batch + 1, dtype=np.int64)
    position = 0
    for run in (4, 1, 1, 2):
        tokens = streams[:, position:position + run]
        positions = np.full(batch, position, np.int64)
        offsets = np.full(batch, run - 1, np.int64)
        got = graphs.run(tokens, positions, offsets, cache_rows, span=16).clone()
        cuda = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        hidden = actor.forward_ragged(cuda(tokens), cuda(positions), eager_cache, cuda(offsets), span=16,
                                      rows=cuda(cache_rows))
        context = actor.pop_context()[torch.arange(batch, device="cuda"), cuda(offsets)]
        want = torch.cat([actor.policy_logits(hidden, head, None, None, context) for head in actor.policy_heads]
                         + [actor.player_values(hidden)], dim=-1)
        assert torch.equal(got, want), (run, position)
        position += run
    assert graphs.columns["exchange"] == slice(0, 33) and graphs.columns["values"] == slice(67, 69)
    assert torch.equal(graph_cache.k_pool, eager_cache.k_pool)
