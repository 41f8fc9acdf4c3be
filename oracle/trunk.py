"""Numpy restatement of the reference trunk's three execution paths (oracle only).

Restates cardgym/nn/trunk.py (``Trunk.condition`` 285-312, ``_add_ple`` 318-333,
``forward`` 348-374, ``forward_prefill`` 376-389, ``forward_ragged`` 391-429,
``DecoderBlock._qkv`` 141-152, ``_finish`` 154-157, ``forward_ragged`` 183-223,
``_grouped_attention`` 225-256) and the KV pool of cardgym/nn/kv_cache.py
(``write_range`` 65-82, ``write_step`` 84-105, ``read`` 107-120, ``copy_rows`` 122-138).

Arithmetic is float64 by default (``Precision.dtype``), so the oracle sits closer to
exact than either float32 implementation it checks. ``Precision`` can also round at
the points where the B200 bf16 kernels round: GEMM operands (activations and
weights) to bf16, K/V/Q to the cache's storage dtype, and the attention
probabilities to the cache dtype before they multiply V. With ``gemm="fp32"`` and
``kv="fp32"`` nothing is rounded beyond the compute dtype, which is the
reference's fp32 path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from .numerics import gelu, layer_norm, rms_norm, round_bf16, round_to


@dataclass(frozen=True)
class Precision:
    gemm: str = "fp32"  # "fp32" | "bf16": GEMM operand rounding
    kv: str = "fp32"  # cache storage: "fp32" | "fp16" | "bf16"
    dtype: type = np.float64  # compute dtype of every other operation

    def operand(self, values: np.ndarray) -> np.ndarray:
        if self.gemm == "bf16":
            return round_bf16(values).astype(self.dtype)
        return values.astype(self.dtype, copy=False)

    def stored(self, values: np.ndarray) -> np.ndarray:
        if self.kv == "fp32" and self.dtype == np.float32:
            return values.astype(np.float32, copy=False)
        return round_to(values, self.kv).astype(self.dtype, copy=False)


@dataclass(frozen=True)
class TrunkShape:
    d_model: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    d_ff: int
    per_layer_dim: int
    value_layers: tuple[int, ...]
    input_norm: bool = True

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def kv_width(self) -> int:
        return self.n_kv_heads * self.head_dim


def value_layers(n_layers: int, mode: str) -> tuple[int, ...]:
    """cardgym/nn/trunk.py:58-72: the final block and every other one backward."""

    if mode == "off":
        return ()
    if mode == "all":
        return tuple(range(n_layers))
    return tuple(layer for layer in range(n_layers) if layer % 2 == (n_layers - 1) % 2)


@dataclass
class Block:
    ln_attn_w: np.ndarray
    ln_attn_b: np.ndarray
    qkv: np.ndarray  # [(H + 2 KVH) D, d]
    out: np.ndarray  # [d, d]
    ln_mlp_w: np.ndarray
    ln_mlp_b: np.ndarray
    up: np.ndarray  # [d_ff, d]
    up_b: np.ndarray
    down: np.ndarray  # [d, d_ff]
    down_b: np.ndarray


@dataclass
class TrunkWeights:
    shape: TrunkShape
    blocks: list[Block]
    input_norm: np.ndarray | None
    ple_context: np.ndarray | None  # [L * ple_dim, d]
    final_w: np.ndarray
    final_b: np.ndarray

    @classmethod
    def from_state(cls, state: dict, shape: TrunkShape, prefix: str = "trunk.") -> "TrunkWeights":
        def get(name: str) -> np.ndarray:
            return np.asarray(state[prefix + name], dtype=np.float64)

        blocks = []
        for layer in range(shape.n_layers):
            p = f"blocks.{layer}."
            blocks.append(
                Block(
                    get(p + "ln_attn.weight"), get(p + "ln_attn.bias"), get(p + "qkv_proj.weight"),
                    get(p + "out_proj.weight"), get(p + "ln_mlp.weight"), get(p + "ln_mlp.bias"),
                    get(p + "mlp.0.weight"), get(p + "mlp.0.bias"), get(p + "mlp.2.weight"), get(p + "mlp.2.bias"),
                )
            )
        return cls(
            shape=shape,
            blocks=blocks,
            input_norm=get("input_norm.weight") if shape.input_norm else None,
            ple_context=get("ple_context.weight") if shape.per_layer_dim else None,
            final_w=get("final_norm.weight"),
            final_b=get("final_norm.bias"),
        )


def _linear(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, prec: Precision) -> np.ndarray:
    y = prec.operand(x) @ prec.operand(weight).T
    if bias is not None:
        y = y + bias.astype(prec.dtype)
    return y


@dataclass
class Cache:
    """The KV pool [layers, rows, kv_heads, max_len, head_dim], zero-filled (kv_cache.py:42-59)."""

    n_layers: int
    capacity: int
    kv_heads: int
    max_len: int
    head_dim: int
    prec: Precision = field(default_factory=Precision)

    def __post_init__(self) -> None:
        shape = (self.n_layers, self.capacity, self.kv_heads, self.max_len, self.head_dim)
        self.k = np.zeros(shape, dtype=self.prec.dtype)
        self.v = np.zeros(shape, dtype=self.prec.dtype)

    def write_range(self, layer: int, rows: np.ndarray | None, start: int, k_new: np.ndarray, v_new: np.ndarray) -> None:
        """k_new/v_new [B, KVH, T, D] at a shared offset (kv_cache.py:65-82)."""

        stop = start + k_new.shape[2]
        rows = np.arange(k_new.shape[0]) if rows is None else rows
        self.k[layer, rows, :, start:stop] = self.prec.stored(k_new)
        self.v[layer, rows, :, start:stop] = self.prec.stored(v_new)

    def write_step(self, layer: int, rows: np.ndarray, positions: np.ndarray, k_new: np.ndarray, v_new: np.ndarray) -> None:
        """Per-row offsets ``positions`` [B, T] (kv_cache.py:84-105); later steps win a shared slot."""

        k_stored, v_stored = self.prec.stored(k_new), self.prec.stored(v_new)
        for t in range(positions.shape[1]):
            self.k[layer, rows, :, positions[:, t]] = k_stored[:, :, t]
            self.v[layer, rows, :, positions[:, t]] = v_stored[:, :, t]

    def copy_rows(self, sources: np.ndarray, targets: np.ndarray, length: int) -> None:
        """Copy the first ``length`` positions of ``sources`` onto ``targets`` (kv_cache.py:122-138)."""

        k = self.k[:, sources, :, :length].copy()
        v = self.v[:, sources, :, :length].copy()
        self.k[:, targets, :, :length] = k
        self.v[:, targets, :, :length] = v


class Trunk:
    """The reference Trunk's forward paths over ``TrunkWeights``."""

    def __init__(self, weights: TrunkWeights, prec: Precision | None = None) -> None:
        self.w = weights
        self.s = weights.shape
        self.prec = prec or Precision()
        self._value_index = {layer: i for i, layer in enumerate(self.s.value_layers)}

    # -- conditioning (trunk.py:285-312) -----------------------------------
    def condition(self, x: np.ndarray, ple_lookup: np.ndarray | None, value_lookup: np.ndarray | None):
        dt = self.prec.dtype
        x = x.astype(dt)
        if self.w.input_norm is not None:
            x = rms_norm(x, self.w.input_norm.astype(dt))
        lead = x.shape[:-1]
        ple = None
        if self.w.ple_context is not None:
            context = _linear(x, self.w.ple_context, None, self.prec)
            ple = ((ple_lookup.astype(dt) + context) * (1.0 / math.sqrt(2.0))).reshape(
                *lead, self.s.n_layers, self.s.per_layer_dim
            )
        values = None
        if self._value_index:
            values = value_lookup.astype(dt).reshape(*lead, len(self._value_index), self.s.kv_width)
        return x, ple, values

    def _value(self, values, layer: int):
        index = self._value_index.get(layer)
        return None if index is None or values is None else values[..., index, :]

    def add_ple(self, x: np.ndarray, ple: np.ndarray | None, layer: int) -> np.ndarray:
        """trunk.py:318-333: equal width, divisible width, or a truncated repeat."""

        if ple is None:
            return x
        update = ple[..., layer, :]
        d, p = x.shape[-1], update.shape[-1]
        if p == d:
            return x + update
        if d % p == 0:
            repeats = d // p
            shaped = x.reshape(*x.shape[:-1], repeats, p) + update[..., None, :] * (1.0 / math.sqrt(repeats))
            return shaped.reshape(x.shape)
        repeats = math.ceil(d / p)
        expanded = np.concatenate([update] * repeats, axis=-1)[..., :d]
        return x + expanded * (1.0 / math.sqrt(repeats))

    # -- block pieces ---------------------------------------------------------
    def _qkv(self, block: Block, x: np.ndarray, value_embedding):
        """DecoderBlock._qkv (trunk.py:141-152): q [B,H,T,D], k/v [B,KVH,T,D]."""

        s = self.s
        batch, length, _ = x.shape
        h = layer_norm(x, block.ln_attn_w, block.ln_attn_b)
        qkv = _linear(h, block.qkv, None, self.prec)
        q_w, kv_w = s.n_heads * s.head_dim, s.kv_width
        q = qkv[..., :q_w].reshape(batch, length, s.n_heads, s.head_dim).transpose(0, 2, 1, 3)
        k = qkv[..., q_w : q_w + kv_w].reshape(batch, length, s.n_kv_heads, s.head_dim).transpose(0, 2, 1, 3)
        v = qkv[..., q_w + kv_w :].reshape(batch, length, s.n_kv_heads, s.head_dim)
        if value_embedding is not None:
            v = v + value_embedding.reshape(v.shape)
        return q, k, v.transpose(0, 2, 1, 3)

    def _finish(self, block: Block, x: np.ndarray, attn: np.ndarray) -> np.ndarray:
        """DecoderBlock._finish (trunk.py:154-157)."""

        batch, _, length, _ = attn.shape
        merged = attn.transpose(0, 2, 1, 3).reshape(batch, length, -1)
        x = x + _linear(merged, block.out, None, self.prec)
        h = layer_norm(x, block.ln_mlp_w, block.ln_mlp_b)
        hidden = gelu(_linear(h, block.up, block.up_b, self.prec))
        return x + _linear(hidden, block.down, block.down_b, self.prec)

    def _attend(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, limits: np.ndarray) -> np.ndarray:
        """Grouped masked attention (trunk.py:225-256).

        q [B,H,T,D]; k/v [B,KVH,S,D]; ``limits`` [B,T]: query t of row b sees keys
        below ``limits[b, t]``. Softmax runs at the compute dtype; the weights that
        multiply V are rounded to the cache dtype, as the reference's ``.to(v.dtype)``.
        """

        s = self.s
        batch, _, length, dim = q.shape
        grouped = q.reshape(batch, s.n_kv_heads, s.group * length, dim)
        scores = np.matmul(grouped, k.transpose(0, 1, 3, 2)) * (1.0 / math.sqrt(dim))
        keys = np.arange(k.shape[2])
        # Row g * T + t of the merged axis is query t of group g.
        limit = np.tile(limits, (1, s.group))  # [B, G*T]
        blocked = keys[None, None, :] >= limit[:, :, None]
        scores = np.where(blocked[:, None], -np.inf, scores)
        peak = scores.max(axis=-1, keepdims=True)
        weights = np.exp(scores - peak)
        total = weights.sum(axis=-1, keepdims=True)
        if self.prec.kv != "fp32":
            # The B200 tensor-core path multiplies V by probabilities held in the cache dtype
            # and divides by the float32 row sum afterwards.
            out = np.matmul(self.prec.stored(weights), v) / total
        else:
            out = np.matmul(weights / total, v)
        return out.reshape(batch, s.n_heads, length, dim)

    # -- full causal forward (trunk.py:348-374) ----------------------------
    def forward(self, x: np.ndarray, ple, values) -> np.ndarray:
        length = x.shape[1]
        causal = np.tile(np.arange(1, length + 1)[None, :], (x.shape[0], 1))
        for layer, block in enumerate(self.w.blocks):
            q, k, v = self._qkv(block, x, self._value(values, layer))
            # The full forward attends at the compute dtype (SDPA): no cache rounding.
            prec, self.prec = self.prec, Precision(self.prec.gemm, "fp32", self.prec.dtype)
            try:
                attn = self._attend(q, k, v, causal)
            finally:
                self.prec = prec
            x = self._finish(block, x, attn)
            x = self.add_ple(x, ple, layer)
        return layer_norm(x, self.w.final_w, self.w.final_b)

    # -- prefill (trunk.py:376-389) ------------------------------------------
    def forward_prefill(self, x: np.ndarray, ple, values, cache: Cache, rows: np.ndarray | None) -> np.ndarray:
        length = x.shape[1]
        causal = np.tile(np.arange(1, length + 1)[None, :], (x.shape[0], 1))
        for layer, block in enumerate(self.w.blocks):
            q, k, v = self._qkv(block, x, self._value(values, layer))
            cache.write_range(layer, rows, 0, k, v)
            prec, self.prec = self.prec, Precision(self.prec.gemm, "fp32", self.prec.dtype)
            try:
                attn = self._attend(q, k, v, causal)
            finally:
                self.prec = prec
            x = self._finish(block, x, attn)
            x = self.add_ple(x, ple, layer)
        return layer_norm(x[:, -1], self.w.final_w, self.w.final_b)

    # -- ragged cached step (trunk.py:391-429, 183-223) -----------------------
    def forward_ragged(
        self,
        x: np.ndarray,
        ple,
        values,
        cache: Cache,
        positions: np.ndarray,
        readout_offsets: np.ndarray,
        span: int | None = None,
        rows: np.ndarray | None = None,
    ) -> np.ndarray:
        batch, length, _ = x.shape
        positions = np.asarray(positions, dtype=np.int64)
        write_positions = np.minimum(positions[:, None] + np.arange(length)[None, :], cache.max_len - 1)
        if span is None:
            span = int(positions.max()) + length
        span = min(span, cache.max_len)
        key_lengths = positions + 1
        limits = np.minimum(key_lengths[:, None] + np.arange(length)[None, :], span)
        row_ids = np.arange(batch) if rows is None else np.asarray(rows, dtype=np.int64)
        for layer, block in enumerate(self.w.blocks):
            q, k, v = self._qkv(block, x, self._value(values, layer))
            cache.write_step(layer, row_ids, write_positions, k, v)
            k_all = cache.k[layer, row_ids, :, :span]
            v_all = cache.v[layer, row_ids, :, :span]
            attn = self._attend(self.prec.stored(q), k_all, v_all, limits)
            x = self._finish(block, x, attn)
            x = self.add_ple(x, ple, layer)
        readout = x[np.arange(batch), np.asarray(readout_offsets, dtype=np.int64)]
        return layer_norm(readout, self.w.final_w, self.w.final_b)


def decode_attention(q, k_cache, v_cache, rows, key_lengths, span: int, scale: float, kv: str = "fp32",
                     dtype=np.float64) -> np.ndarray:
    """The reference op's contract (cardgym/nn/cuda_decode.py:188-202, trunk.py:225-256).

    q [B, H, T, D]; k/v [R, KVH, L, D]; query t of row b sees keys < min(key_lengths[b] + t, span).
    ``kv`` names the cache dtype: q is rounded to it (cuda_decode.py:202), and with a
    16-bit cache the probabilities multiplying V are rounded to it as well.
    """

    prec = Precision(kv=kv, dtype=dtype)
    q = prec.stored(np.asarray(q, np.float64))
    batch, heads, steps, dim = q.shape
    kv_heads = k_cache.shape[1]
    group = heads // kv_heads
    out = np.zeros((batch, heads, steps, dim), dtype=dtype)
    for b in range(batch):
        row = int(rows[b])
        for h in range(heads):
            kvh = h // group
            keys = np.asarray(k_cache[row, kvh], np.float64)
            values = np.asarray(v_cache[row, kvh], np.float64)
            for t in range(steps):
                limit = min(int(key_lengths[b]) + t, span)
                if limit <= 0:
                    continue
                scores = keys[:limit] @ q[b, h, t] * scale
                weights = np.exp(scores - scores.max())
                total = weights.sum()
                if kv != "fp32":
                    out[b, h, t] = prec.stored(weights) @ values[:limit] / total
                else:
                    out[b, h, t] = (weights / total) @ values[:limit]
    return out
