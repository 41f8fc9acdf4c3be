"""The library's entry points as torch custom ops (namespace ``cardgym_b200``), with fake kernels.

The reference registers its one native kernel as ``cardgym::decode_attention`` with a fake
kernel so that ``torch.compile`` and CUDA-graph capture can trace through it
(cardgym/nn/cuda_decode.py:172-181). The same is done here for every entry point a traced caller
needs: the ragged trunk decode (which writes the KV pool it is given), the fused heads + masked
sampling, masked sampling alone, segmented GAE, the baseline's seat values, the PPO objective
and the value loss. Each op calls the same C ABI as the Python wrappers in ``trunk``, ``plump``,
``sampling`` and ``ppo``; its fake kernel only allocates outputs of the right shapes, so a trace
never runs a kernel. ``decode_attention`` is registered by ``cuda_decode``.

Descriptors that are C structs in the ABI (trunk dimensions, the heads layout) are passed as int
lists in their field order.
"""

from __future__ import annotations

import torch

from . import _native as nat
from . import cuda_decode  # noqa: F401  (registers cardgym_b200::decode_attention)

_DIMS_FIELDS = ("d_model", "n_layers", "n_heads", "n_kv_heads", "d_ff", "per_layer_dim", "input_norm", "reserved",
                "value_layers")


def trunk_dims_list(dims: nat.TrunkDims) -> list[int]:
    return [int(getattr(dims, name)) for name in _DIMS_FIELDS]


def _dims(values: list[int]) -> nat.TrunkDims:
    return nat.TrunkDims(**dict(zip(_DIMS_FIELDS, values)))


def heads_desc_list(desc: nat.HeadsDesc) -> list[int]:
    return [desc.d_model, desc.n_policy, desc.value_outputs, desc.max_width, *desc.width, *desc.weight_offset,
            *desc.bias_offset, desc.value_w1, desc.value_b1, desc.value_w2, desc.value_b2]


def _heads_desc(values: list[int]) -> nat.HeadsDesc:
    desc = nat.HeadsDesc()
    desc.d_model, desc.n_policy, desc.value_outputs, desc.max_width = values[:4]
    for i in range(8):
        desc.width[i] = values[4 + i]
        desc.weight_offset[i] = values[12 + i]
        desc.bias_offset[i] = values[20 + i]
    desc.value_w1, desc.value_b1, desc.value_w2, desc.value_b2 = values[28:32]
    return desc


# -- trunk -----------------------------------------------------------------------------------------------------
@torch.library.custom_op("cardgym_b200::trunk_forward_ragged", mutates_args=("k_pool", "v_pool", "workspace"))
def trunk_forward_ragged(dims: list[int], blob: torch.Tensor, x: torch.Tensor, ple: torch.Tensor | None,
                         values: torch.Tensor | None, k_pool: torch.Tensor, v_pool: torch.Tensor,
                         positions: torch.Tensor, readout_offsets: torch.Tensor, rows: torch.Tensor | None, span: int,
                         precision: int, workspace: torch.Tensor) -> torch.Tensor:
    """Trunk.forward_ragged (cardgym/nn/trunk.py:391-429): x [B, T, d] (+ ple, values) appended to the pool
    [n_layers, capacity, kv_heads, max_len, head_dim]; returns the final-norm hidden [B, d]."""

    batch, steps, d_model = x.shape
    hidden = torch.empty((batch, d_model), device=x.device)
    nat.call("cg_trunk_forward_ragged", _dims(dims), nat.ptr(blob), nat.ptr(x.float().contiguous()),
             nat.ptr(None if ple is None else ple.float().contiguous()),
             nat.ptr(None if values is None else values.float().contiguous()), batch, steps,
             nat.ptr(positions.to(torch.int64).contiguous()), nat.ptr(readout_offsets.to(torch.int64).contiguous()),
             nat.ptr(None if rows is None else rows.to(torch.int64).contiguous()), int(span), nat.ptr(k_pool),
             nat.ptr(v_pool), nat.DTYPE_CODES[k_pool.dtype], k_pool.shape[1], k_pool.shape[3], int(precision),
             nat.ptr(workspace), workspace.numel(), nat.ptr(hidden), nat.stream_handle(x.device))
    return hidden


@trunk_forward_ragged.register_fake
def _(dims, blob, x, ple, values, k_pool, v_pool, positions, readout_offsets, rows, span, precision, workspace):
    return x.new_empty((x.shape[0], x.shape[2]), dtype=torch.float32)


# -- heads and sampling -------------------------------------------------------------------------------------------
@torch.library.custom_op("cardgym_b200::plump_decide", mutates_args=())
def plump_decide(desc: list[int], blob: torch.Tensor, hidden: torch.Tensor, hidden_rows: torch.Tensor | None,
                 heads: torch.Tensor, legal: torch.Tensor, uniforms: torch.Tensor
                 ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Heads + legal masking + inverse-CDF draws (plump/model.py:204-217, rl/ppo.py:75-94): (logits, probs fp32
    [D, max_width], actions int64 [D], values fp32 [D, value_outputs])."""

    description = _heads_desc(desc)
    count = heads.shape[0]
    width = description.max_width
    logits = torch.empty((count, width), device=hidden.device)
    probs = torch.empty((count, width), device=hidden.device)
    actions = torch.empty(count, dtype=torch.int64, device=hidden.device)
    values = torch.empty((count, description.value_outputs), device=hidden.device)
    nat.call("cg_plump_decide", description, nat.ptr(blob), nat.ptr(hidden.float().contiguous()),
             nat.ptr(None if hidden_rows is None else hidden_rows.to(torch.int64).contiguous()), count,
             nat.ptr(heads.to(torch.int32).contiguous()), nat.ptr(legal.to(torch.uint8).contiguous()),
             nat.ptr(uniforms.to(torch.float64).contiguous()), nat.ptr(logits), nat.ptr(probs), nat.ptr(actions),
             nat.ptr(values), nat.stream_handle(hidden.device))
    return logits, probs, actions, values


@plump_decide.register_fake
def _(desc, blob, hidden, hidden_rows, heads, legal, uniforms):
    count, width, outputs = heads.shape[0], desc[3], desc[2]
    return (hidden.new_empty((count, width)), hidden.new_empty((count, width)),
            hidden.new_empty(count, dtype=torch.int64), hidden.new_empty((count, outputs)))


@torch.library.custom_op("cardgym_b200::masked_sample", mutates_args=())
def masked_sample(logits: torch.Tensor, mask: torch.Tensor, uniforms: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """masked_probabilities + sample_rows (rl/ppo.py:75-94), bit-exact with numpy: (probs, actions)."""

    from .sampling import masked_sample as run

    probs, actions = run(logits, mask, uniforms)
    return probs, actions


@masked_sample.register_fake
def _(logits, mask, uniforms):
    return logits.new_empty(logits.shape, dtype=torch.float32), logits.new_empty(logits.shape[0], dtype=torch.int64)


# -- PPO -----------------------------------------------------------------------------------------------------------
@torch.library.custom_op("cardgym_b200::segmented_gae", mutates_args=())
def segmented_gae(values: torch.Tensor, seats: torch.Tensor, starts: torch.Tensor, returns: torch.Tensor,
                  gae_lambda: float) -> torch.Tensor:
    """Acting-seat GAE per game segment (rl/ppo.py:121-144, trainer.py:634-649), float64 [N]."""

    from .ppo import segmented_gae as run

    return run(values, seats, starts, returns, gae_lambda)


@segmented_gae.register_fake
def _(values, seats, starts, returns, gae_lambda):
    return values.new_empty(values.shape[0], dtype=torch.float64)


@torch.library.custom_op("cardgym_b200::seat_values", mutates_args=())
def seat_values(values: torch.Tensor, shift: torch.Tensor, players: torch.Tensor, seat: torch.Tensor,
                flat: torch.Tensor | None, center: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """The baseline's per-decision seat values and prediction (trainer.py:556-571, 610-632), float64."""

    from .ppo import seat_values as run

    return run(values, shift, players, seat, flat, center=center)


@seat_values.register_fake
def _(values, shift, players, seat, flat, center):
    count = shift.shape[0]
    return (values.new_empty((count, values.shape[1]), dtype=torch.float64),
            values.new_empty(count, dtype=torch.float64))


@torch.library.custom_op("cardgym_b200::ppo_objective", mutates_args=())
def ppo_objective(logits: torch.Tensor, old_probs: torch.Tensor, actions: torch.Tensor, advantages: torch.Tensor,
                  weights: torch.Tensor, clip_ratio: float, alpha: float
                  ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The fused per-head objective (trainer.py:733-802): (dL/dlogits fp32 [N, A], row terms fp32 [N, 8],
    totals float64 [8] in ppo.TOTAL_KEYS order)."""

    from .ppo import _run_objective

    dlogits, terms, totals = _run_objective(logits, old_probs, actions, advantages, weights, clip_ratio, alpha,
                                            want_grad=True, want_terms=True)
    return dlogits, terms, totals


@ppo_objective.register_fake
def _(logits, old_probs, actions, advantages, weights, clip_ratio, alpha):
    rows = logits.shape[0]
    return (logits.new_empty(logits.shape, dtype=torch.float32), logits.new_empty((rows, 8), dtype=torch.float32),
            logits.new_empty(8, dtype=torch.float64))


@torch.library.custom_op("cardgym_b200::value_loss", mutates_args=())
def value_loss(prediction: torch.Tensor, players: torch.Tensor, targets: torch.Tensor, weights: torch.Tensor,
               reward_scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense zero-sum value regression (trainer.py:822-850): (dloss/dprediction fp32, totals float64 [4])."""

    prediction = prediction.float().contiguous()
    rows, width = prediction.shape
    grad = torch.empty_like(prediction)
    totals = torch.empty(4, dtype=torch.float64, device=prediction.device)
    workspace = nat.Workspace.get(prediction.device, nat.query("cg_value_loss_workspace_bytes", rows), "reduce")
    nat.call("cg_value_loss", nat.ptr(prediction), nat.ptr(targets.float().contiguous()),
             nat.ptr(players.to(torch.int32).contiguous()), nat.ptr(weights.float().contiguous()), rows, width,
             float(reward_scale), nat.ptr(grad), nat.ptr(totals), nat.ptr(workspace), workspace.numel(),
             nat.stream_handle(prediction.device))
    return grad, totals


@value_loss.register_fake
def _(prediction, players, targets, weights, reward_scale):
    return prediction.new_empty(prediction.shape, dtype=torch.float32), prediction.new_empty(4, dtype=torch.float64)
