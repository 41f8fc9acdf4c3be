"""Op-level parity of the CUDA kernels against the CPU oracle, through the C ABI (B200 only)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import plump as oplump
from oracle import ppo as oppo
from oracle.trunk import Cache, Precision
from oracle.trunk import decode_attention as oracle_attention
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

TORCH_DTYPES = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}
# Tolerances on max |error| / max |expected|: fp32 arithmetic, then one storage rounding
# of the probabilities (fp16: 2^-11, bf16: 2^-8) that the oracle places at the final
# softmax max while the kernel's online softmax places it at the running max.
ATTN_TOL = {"fp32": 2e-5, "fp16": 2e-3, "bf16": 1.5e-2}


def scaled_error(actual: np.ndarray, expected: np.ndarray) -> float:
    return float(np.abs(actual - expected).max() / max(np.abs(expected).max(), 1e-30))


@pytest.mark.parametrize("kv", ["fp32", "fp16", "bf16"])
@pytest.mark.parametrize("heads,kv_heads,dim", [(10, 2, 24), (8, 2, 32), (5, 1, 40), (8, 4, 64)])
@pytest.mark.parametrize("steps", [1, 3, 7, 16])  # 7, 16: G*T > 16 splits a row's steps into blocks
def test_decode_attention_matches_the_oracle(kv, heads, kv_heads, dim, steps):
    rng = np.random.default_rng(heads * 100 + dim + steps)
    batch, capacity, max_len = 37, 48, 300
    k = rng.standard_normal((capacity, kv_heads, max_len, dim)).astype(np.float32)
    v = rng.standard_normal((capacity, kv_heads, max_len, dim)).astype(np.float32)
    q = rng.standard_normal((batch, heads, steps, dim)).astype(np.float32)
    rows = rng.permutation(capacity)[:batch].astype(np.int64)
    lengths = rng.integers(1, max_len - steps, batch).astype(np.int64)
    lengths[:3] = [1, 64, 65]  # one key; chunk boundaries
    span = int(lengths.max()) + steps - 1
    span -= 7  # a cap below the longest row: rows near the top see only `span` keys
    dt = TORCH_DTYPES[kv]
    kd, vd = torch.from_numpy(k).cuda().to(dt), torch.from_numpy(v).cuda().to(dt)
    k_stored, v_stored = kd.float().cpu().numpy(), vd.float().cpu().numpy()
    from card_playing_gym_b200.cuda_decode import decode_attention

    out = decode_attention(torch.from_numpy(q).cuda(), kd, vd, torch.from_numpy(rows).cuda(),
                           torch.from_numpy(lengths).cuda(), span, dim ** -0.5)
    assert out.dtype == dt and out.shape == q.shape
    expected = oracle_attention(q, k_stored, v_stored, rows, lengths, span, dim ** -0.5, kv=kv)
    assert scaled_error(out.float().cpu().numpy(), expected) < ATTN_TOL[kv]


def test_decode_attention_at_the_reference_kernel_shapes():
    """cardgym/nn/cuda_decode.py's own envelope: head_dim 32, spans <= 64, fp16, 384 rows x 3 tokens."""

    rng = np.random.default_rng(7)
    batch, heads, kv_heads, dim, steps, max_len = 384, 8, 2, 32, 3, 64
    k = rng.standard_normal((batch, kv_heads, max_len, dim)).astype(np.float16)
    v = rng.standard_normal((batch, kv_heads, max_len, dim)).astype(np.float16)
    q = rng.standard_normal((batch, heads, steps, dim)).astype(np.float32)
    lengths = rng.integers(1, max_len - steps + 1, batch).astype(np.int64)
    rows = np.arange(batch, dtype=np.int64)
    from card_playing_gym_b200.cuda_decode import decode_attention

    out = decode_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                           torch.from_numpy(rows).cuda(), torch.from_numpy(lengths).cuda(), max_len, dim ** -0.5)
    expected = oracle_attention(q, k.astype(np.float32), v.astype(np.float32), rows, lengths, max_len, dim ** -0.5,
                                kv="fp16")
    assert scaled_error(out.float().cpu().numpy(), expected) < ATTN_TOL["fp16"]


@pytest.mark.parametrize("kv", ["fp32", "fp16", "bf16"])
def test_kv_write_step_and_overlapping_copy_rows(kv):
    from card_playing_gym_b200.kv_cache import KVCache

    rng = np.random.default_rng(3)
    layers, kvh, dim, capacity, max_len = 3, 2, 24, 12, 20
    cache = KVCache(n_layers=layers, kv_heads=kvh, head_dim=dim, capacity=capacity, max_len=max_len, device="cuda",
                    dtype=TORCH_DTYPES[kv])
    ref = Cache(layers, capacity, kvh, max_len, dim, Precision(kv=kv))
    rows = np.array([5, 1, 7, 2], dtype=np.int64)
    for layer in range(layers):
        positions = rng.integers(0, max_len - 3, (4, 1)) + np.arange(3)[None, :]
        k_new = rng.standard_normal((4, kvh, 3, dim)).astype(np.float32)
        v_new = rng.standard_normal((4, kvh, 3, dim)).astype(np.float32)
        cache.write_step(layer, torch.from_numpy(rows).cuda(), torch.from_numpy(positions).cuda(),
                         torch.from_numpy(k_new).cuda(), torch.from_numpy(v_new).cuda())
        ref.write_step(layer, rows, positions, k_new, v_new)
        cache.write_range(layer, None, 2, torch.from_numpy(k_new[:2]).cuda(), torch.from_numpy(v_new[:2]).cuda())
        ref.write_range(layer, None, 2, k_new[:2], v_new[:2])
    # Survivors slide down: row 2 is both a source and a target.
    sources, targets = np.array([2, 5, 7]), np.array([1, 2, 3])
    cache.copy_rows(torch.from_numpy(sources).cuda(), torch.from_numpy(targets).cuda(), 11)
    ref.copy_rows(sources, targets, 11)
    assert np.array_equal(cache.k_pool.float().cpu().numpy(), ref.k)
    assert np.array_equal(cache.v_pool.float().cpu().numpy(), ref.v)


def test_kv_indices_outside_the_pool_are_skipped_and_reported():
    """A row or position past the pool is never read or written: the kernels skip it and set the fault word
    (0x110 writes, 0x111 row copies). The bad indices are one past the end, so a missed check would stay
    inside the allocation of the test's own stacked pool."""

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.kv_cache import KVCache

    assert nat.fault_status() == 0
    layers, kvh, dim, capacity, max_len = 2, 2, 24, 6, 16
    # The pool has one more row than the cache is told about, so index `capacity` is still memory this test
    # owns and nothing outside an allocation can be touched either way.
    backing = KVCache(n_layers=layers, kv_heads=kvh, head_dim=dim, capacity=capacity + 1, max_len=max_len,
                      device="cuda", dtype=torch.float16)
    backing.k_pool.normal_()
    backing.v_pool.normal_()
    before_k, before_v = backing.k_pool.clone(), backing.v_pool.clone()
    code = nat.DTYPE_CODES[torch.float16]
    stream = nat.stream_handle(torch.device("cuda"))
    rows = torch.tensor([1, capacity, 3], dtype=torch.int64, device="cuda")
    positions = torch.tensor([[2], [2], [max_len]], dtype=torch.int64, device="cuda")
    k_new = torch.ones((3, kvh, 1, dim), device="cuda")
    layer_k = backing.k_pool[0]
    layer_v = backing.v_pool[0]
    # cg_kv_write_step addresses one layer as [capacity, KVH, L, D]; pass the smaller capacity.
    nat.call("cg_kv_write_step", nat.ptr(layer_k), nat.ptr(layer_v), code, capacity, kvh, max_len, dim,
             nat.ptr(rows), nat.ptr(positions), 3, 1, nat.ptr(k_new), nat.ptr(k_new), nat.CG_F32, stream)
    assert nat.fault_status() == 0x110
    expected_k = before_k.clone()
    expected_k[0, 1, :, 2] = 1.0  # only the in-range entry landed
    expected_v = before_v.clone()
    expected_v[0, 1, :, 2] = 1.0
    assert torch.equal(backing.k_pool, expected_k) and torch.equal(backing.v_pool, expected_v)

    sources = torch.tensor([0, capacity, 2], dtype=torch.int64, device="cuda")
    targets = torch.tensor([4, 5, capacity], dtype=torch.int64, device="cuda")
    for name in ("cg_kv_copy_rows", "cg_kv_copy_rows_noalloc"):
        snapshot_k, snapshot_v = backing.k_pool.clone(), backing.v_pool.clone()
        # The stacked pool is addressed with capacity + 1 rows per layer, but told `capacity`: every layer's
        # rows then start `layer * capacity` rows in, all inside the allocation.
        args = [nat.ptr(backing.k_pool), nat.ptr(backing.v_pool), code, layers, capacity, kvh, max_len, dim,
                nat.ptr(sources), nat.ptr(targets), 3, 5]
        if name == "cg_kv_copy_rows":
            workspace = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
            args += [nat.ptr(workspace), workspace.numel()]
        nat.call(name, *args, stream)
        assert nat.fault_status() == 0x111
        flat_k = snapshot_k.view(-1)[: layers * capacity * kvh * max_len * dim].view(layers, capacity, kvh, max_len,
                                                                                       dim).clone()
        flat_v = snapshot_v.view(-1)[: layers * capacity * kvh * max_len * dim].view(layers, capacity, kvh, max_len,
                                                                                       dim).clone()
        flat_k[:, 4, :, :5] = flat_k[:, 0, :, :5]
        flat_v[:, 4, :, :5] = flat_v[:, 0, :, :5]
        got_k = backing.k_pool.view(-1)[: flat_k.numel()].view_as(flat_k)
        got_v = backing.v_pool.view(-1)[: flat_v.numel()].view_as(flat_v)
        assert torch.equal(got_k, flat_k) and torch.equal(got_v, flat_v)
        tail = slice(flat_k.numel(), None)
        assert torch.equal(backing.k_pool.view(-1)[tail], snapshot_k.view(-1)[tail])


def test_plump_field_lookup_matches_the_oracle():
    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    config = PlumpModelConfig()
    state = synthetic_plump_actor_state(config, seed=9)
    actor = PlumpActor(config, state, precision="fp32")
    streams = load_golden("plump_streams")["tokens"]
    tokens = torch.from_numpy(streams.astype(np.int64)).cuda()
    x, ple, values = actor.embed(tokens)
    ox, ople, ovalues = oplump.Embedding.from_state(state).forward(streams.astype(np.int64))
    np.testing.assert_allclose(x.cpu().numpy(), ox, atol=2e-6, rtol=0)
    np.testing.assert_allclose(ple.cpu().numpy(), ople, atol=2e-6, rtol=0)
    np.testing.assert_allclose(values.cpu().numpy(), ovalues, atol=2e-6, rtol=0)
    # int16 tokens (the collector's storage) give the same sums
    x16, _, _ = actor.embed(torch.from_numpy(streams).cuda())
    assert torch.equal(x16, x)


@pytest.mark.parametrize("value", (1 << 40, -(1 << 40), 1 << 31))
def test_plump_field_lookup_flags_ids_out_of_range(value):
    """An id outside its field's rows (int64 values past the int32 range included) sets the
    device fault word to 0x200, as the reference's embedding lookup raises an index error."""

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    config = PlumpModelConfig()
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=9), precision="fp32")
    streams = load_golden("plump_streams")["tokens"].astype(np.int64)
    assert nat.fault_status() == 0
    actor.embed(torch.from_numpy(streams).cuda())
    assert nat.fault_status() == 0
    bad = streams.copy()
    bad.reshape(-1, bad.shape[-1])[3, actor.schema.field_slots[0]] = value
    actor.embed(torch.from_numpy(bad).cuda())
    assert nat.fault_status() == 0x200
    assert nat.fault_status() == 0  # read and cleared


def test_plump_field_lookup_row_per_warp_kernel_matches_the_sliced_kernel():
    """A table width that is not a multiple of 4 takes the row-per-warp lookup: the same sums, bit for bit."""

    from card_playing_gym_b200 import _native as nat
    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    config = PlumpModelConfig()
    state = synthetic_plump_actor_state(config, seed=9)
    actor = PlumpActor(config, state, precision="fp32")
    streams = load_golden("plump_streams")["tokens"]
    flat = torch.from_numpy(streams.reshape(-1, streams.shape[-1]).astype(np.int64)).cuda()
    full = actor.embed_lookup(flat)
    width = actor.trunk.lookup_width - 3
    table = actor.table[:, :width].contiguous()
    out = torch.empty((flat.shape[0], width), device="cuda")
    nat.call("cg_plump_embed", actor.schema, nat.ptr(table), width, nat.ptr(flat), nat.INDEX_CODES[flat.dtype],
             flat.shape[0], nat.ptr(out), nat.stream_handle(torch.device("cuda")))
    assert torch.equal(out, full[:, :width])


@pytest.mark.parametrize("width", (11, 52, 64))
def test_masked_sampling_matches_the_reference(width):
    """The reference's own masked_probabilities / sample_rows outputs (tests/golden/sampling.npz), bit for bit."""

    from card_playing_gym_b200.sampling import masked_sample

    data = load_golden("sampling")
    logits, mask, uniforms = data[f"w{width}_logits"], data[f"w{width}_mask"], data[f"w{width}_uniforms"]
    probs, actions = masked_sample(torch.from_numpy(logits).cuda(), torch.from_numpy(mask).cuda(),
                                   torch.from_numpy(uniforms).cuda())
    probs, actions = probs.cpu().numpy(), actions.cpu().numpy()
    assert np.array_equal(probs.view(np.uint32), data[f"w{width}_probs"].astype(np.float32).view(np.uint32))
    assert np.array_equal(actions, data[f"w{width}_actions"])


def _sampling_rows(rng, rows: int, width: int):
    """Logits N(0, 2) with a few far-apart rows, Bernoulli(0.3) legality (at least one legal), U[0, 1) draws."""

    logits = (rng.standard_normal((rows, width)) * 2.0).astype(np.float32)
    logits[::97] *= 40.0  # shifted logits down to about -500: exp underflows to subnormals and zero
    mask = rng.random((rows, width)) < 0.3
    mask[np.arange(rows), rng.integers(0, width, rows)] = True
    uniforms = rng.random(rows)
    uniforms[::1009] = 1.0 - 2.0 ** -53  # draws past the last CDF step
    return logits, mask, uniforms


def _count_disagreements(width, probs, actions, logits, mask, uniforms):
    expected = oppo.masked_probabilities(logits, mask)
    drawn = oppo.sample_rows(expected, mask, uniforms)
    prob_rows = (probs.view(np.uint32) != expected.view(np.uint32)).any(axis=1)
    action_rows = actions != drawn
    # How many draws sit within 4 float32 ulp of a CDF step: where any rounding difference in
    # the probabilities would have flipped the draw. Reported, not excused.
    cdf = np.cumsum(expected, axis=1)
    near = (np.abs(cdf.astype(np.float64) - uniforms[:, None]) <= 4 * np.spacing(cdf)).any(axis=1)
    print(f"width {width}: {len(actions)} rows, probability rows differing {prob_rows.sum()}, "
          f"draws differing {action_rows.sum()}, draws within 4 ulp of a CDF step {near.sum()}")
    return prob_rows.sum(), action_rows.sum()


@pytest.mark.parametrize("width", (11, 52, 64))
def test_masked_sampling_is_bit_exact_on_a_million_rows(width):
    """cg_masked_sample against numpy's masked_probabilities + sample_rows (the reference's sampler,
    cardgym/rl/ppo.py:75-94) on 2^20 random rows: every probability bit and every draw agree."""

    from card_playing_gym_b200.sampling import masked_sample

    rng = np.random.default_rng(1000 + width)
    logits, mask, uniforms = _sampling_rows(rng, 1 << 20, width)
    probs, actions = masked_sample(torch.from_numpy(logits).cuda(), torch.from_numpy(mask).cuda(),
                                   torch.from_numpy(uniforms).cuda())
    differ = _count_disagreements(width, probs.cpu().numpy(), actions.cpu().numpy(), logits, mask, uniforms)
    assert differ == (0, 0)


def test_decide_samples_its_logits_bit_exactly():
    """The fused heads kernel samples each head's rows as the reference does: numpy's softmax and draw over the
    head's own width (11 bid actions, 52 cards), on the logits the kernel computed, 2^17 decisions."""

    from card_playing_gym_b200.config import PlumpModelConfig, synthetic_plump_actor_state
    from card_playing_gym_b200.plump import PlumpActor

    config = PlumpModelConfig()
    actor = PlumpActor(config, synthetic_plump_actor_state(config, seed=21), precision="bf16")
    rng = np.random.default_rng(21)
    count = 1 << 17
    hidden = torch.from_numpy((rng.standard_normal((count, config.d_model)) * 3).astype(np.float32)).cuda()
    heads = rng.integers(0, 2, count).astype(np.int32)
    legal = rng.random((count, 52)) < 0.3
    legal[np.arange(count), rng.integers(0, 11, count)] = True
    legal[heads == 0, 11:] = False
    uniforms = rng.random(count)
    logits, probs, actions, _ = actor.decide(hidden, torch.from_numpy(heads).cuda(), torch.from_numpy(legal).cuda(),
                                             torch.from_numpy(uniforms).cuda())
    logits, probs, actions = logits.cpu().numpy(), probs.cpu().numpy(), actions.cpu().numpy()
    for head, width in ((0, 11), (1, 52)):
        rows = heads == head
        assert (probs[rows, width:] == 0).all()
        differ = _count_disagreements(width, probs[rows, :width], actions[rows], logits[rows, :width],
                                      legal[rows, :width], uniforms[rows])
        assert differ == (0, 0)


def test_gae_segments_are_bit_exact():
    from card_playing_gym_b200.ppo import gae_advantages, segmented_gae

    data = load_golden("gae")
    for lam in (0.0, 0.95, 1.0):
        adv = segmented_gae(torch.from_numpy(data["values"]).cuda(), torch.from_numpy(data["seats"]).cuda(),
                            torch.from_numpy(data["starts"]).cuda(), torch.from_numpy(data["returns"]).cuda(), lam)
        assert np.array_equal(adv.cpu().numpy(), data[f"adv_{lam}"])
    # the reference's known answers (tests/rl/test_rl.py:58-64)
    values = torch.tensor([[1.0, -1.0], [3.0, -3.0], [2.0, -2.0]], dtype=torch.float64).cuda()
    returns = torch.tensor([5.0, -5.0], dtype=torch.float64).cuda()
    torch.testing.assert_close(gae_advantages(values, returns, 1.0), returns - values)
    one = gae_advantages(values, returns, 0.0)
    torch.testing.assert_close(one[0], values[1] - values[0])


def test_weighted_mean_std_and_normalize():
    from card_playing_gym_b200.ppo import normalize_, weighted_mean_std

    rng = np.random.default_rng(5)
    values = rng.standard_normal(100_003)
    weights = rng.random(100_003)
    mean, std = weighted_mean_std(torch.from_numpy(values).cuda(), torch.from_numpy(weights).cuda())
    emean, estd = oppo.weighted_mean_std(values, weights)
    assert mean == pytest.approx(emean, rel=1e-12, abs=1e-15) and std == pytest.approx(estd, rel=1e-12)
    device = torch.from_numpy(values.copy()).cuda()
    normalize_(device, emean, estd)
    assert np.array_equal(device.cpu().numpy(), (values - emean) / estd)
    assert weighted_mean_std(torch.zeros(4).cuda(), torch.zeros(4).cuda()) == (0.0, 1.0)


def test_normalize_without_host_reads_is_bit_identical():
    """The device-resident two passes (sums never read on the host) give the host path's values."""

    from card_playing_gym_b200.data_parallel import normalize_global_
    from card_playing_gym_b200.ppo import normalize_, weighted_mean_std

    rng = np.random.default_rng(6)
    values = rng.standard_normal(262_147) * 2.5 + 0.3
    weights = rng.random(262_147)
    x, w = torch.from_numpy(values).cuda(), torch.from_numpy(weights).cuda()
    mean, std = weighted_mean_std(x, w)
    expected = normalize_(x.clone(), mean, std)
    got = normalize_global_(x.clone(), w)
    assert torch.equal(got, expected)
    # without weight: mean 0, std 1, values unchanged
    zeros = torch.zeros(5, dtype=torch.float64, device="cuda")
    same = torch.arange(5, dtype=torch.float64, device="cuda")
    assert torch.equal(normalize_global_(same.clone(), zeros), same)


def test_ppo_objective_matches_the_reference_autograd():
    from card_playing_gym_b200.ppo import TOTAL_KEYS, policy_objective, ppo_terms

    data = load_golden("ppo")
    cuda = {k: torch.from_numpy(data[k]).cuda() for k in ("logits", "old_probs", "actions", "advantages", "weights")}
    logits = cuda["logits"].clone().requires_grad_()
    objective, totals = policy_objective(logits, cuda["old_probs"], cuda["actions"], cuda["advantages"],
                                         cuda["weights"], clip_ratio=float(data["clip"]), alpha=float(data["alpha"]))
    objective.backward()
    assert objective.item() == pytest.approx(float(data["objective"]), rel=1e-5, abs=1e-7)
    assert scaled_error(logits.grad.cpu().numpy(), data["grad"]) < 1e-5
    totals = dict(zip(TOTAL_KEYS, totals.tolist()))
    w = data["weights"].astype(np.float64)
    assert totals["policy_loss"] == pytest.approx(float((w * data["losses"]).sum()), rel=1e-5)
    assert totals["row_weight"] == pytest.approx(float(w.sum()), rel=1e-6)
    assert totals["behavior_kl"] == pytest.approx(float((w * data["divergences"]).sum()), rel=1e-5, abs=1e-9)
    terms = ppo_terms(cuda["logits"], cuda["old_probs"], cuda["actions"], cuda["advantages"],
                      clip_ratio=float(data["clip"]))
    for key in ("losses", "divergences", "entropy", "normalized_entropy", "ratios"):
        np.testing.assert_allclose(getattr(terms, key).cpu().numpy(), data[key], rtol=1e-5, atol=1e-6, err_msg=key)
    assert np.array_equal(terms.entropy_eligible.cpu().numpy(), data["entropy_eligible"])
    assert np.array_equal(terms.clipped.cpu().numpy(), data["clipped"])
    np.testing.assert_allclose(terms.log_probs.cpu().numpy(), data["log_probs"], rtol=1e-5, atol=1e-6)


def test_value_loss_matches_the_reference_autograd():
    from card_playing_gym_b200.ppo import value_loss

    data = load_golden("value_loss")
    prediction = torch.from_numpy(data["prediction"]).cuda().requires_grad_()
    loss, totals = value_loss(prediction, torch.from_numpy(data["players"]).cuda(),
                              torch.from_numpy(data["returns"]).cuda(), torch.from_numpy(data["weight"]).cuda(),
                              float(data["scale"]))
    loss.backward()
    assert loss.item() == pytest.approx(float(data["loss"]), rel=1e-5)
    assert totals[1].item() == pytest.approx(float(data["squared_error"]), rel=1e-5)
    assert scaled_error(prediction.grad.cpu().numpy(), data["grad"]) < 1e-5


@pytest.mark.parametrize("center", (False, True))
def test_seat_values_match_the_reference_baseline(center):
    """The baseline's seat gather (trainer.py:556-571) and the recorded values' centring (trainer.py:610-632),
    bit-exact with the reference's numpy arithmetic; rows read through an index, 3 to 7 players of 7 seats."""

    from card_playing_gym_b200.ppo import seat_values

    rng = np.random.default_rng(31 + center)
    n, seats, source_rows = 5000, 7, 6000
    values = rng.standard_normal((source_rows, seats)).astype(np.float32)
    flat = rng.integers(0, source_rows, n)
    players = rng.integers(3, 8, n)
    shift = rng.integers(0, 7, n)
    seat = (rng.random(n) * players).astype(np.int64)
    picked = values[flat]
    if not center:
        picked = oppo.center_zero_sum(picked.astype(np.float64), players).astype(np.float32)
        values = values.copy()
        values[flat] = picked
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    state, prediction = seat_values(cuda(values), cuda(shift), cuda(players), cuda(seat), cuda(flat), center=center)
    want_state, want_prediction = oppo.seat_values(values[flat], shift, players, seat, center=center)
    assert np.array_equal(state.cpu().numpy(), want_state)
    assert np.array_equal(prediction.cpu().numpy(), want_prediction)


def test_center_zero_sum_matches_the_oracle():
    from card_playing_gym_b200.ppo import center_zero_sum

    rng = np.random.default_rng(37)
    values = rng.standard_normal((4099, 5)).astype(np.float32)
    players = rng.integers(2, 6, 4099)
    got = center_zero_sum(torch.from_numpy(values).cuda(), torch.from_numpy(players).cuda()).cpu().numpy()
    want = oppo.center_zero_sum(values.astype(np.float64), players)
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-6)
    assert (got[np.arange(5)[None, :] >= players[:, None]] == 0).all()


def test_no_kernel_fault_was_recorded():
    from card_playing_gym_b200 import _native as nat

    assert nat.fault_status() == 0
