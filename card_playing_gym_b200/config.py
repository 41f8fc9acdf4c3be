"""Trunk and plump-actor configuration, and seeded synthetic weights.

``TrunkConfig`` keeps the field names and derived properties of the reference's
``cardgym/nn/trunk.py:39-90`` so that a reference ``[model]`` section maps onto it
one to one; ``PlumpModelConfig`` mirrors ``cardgym/games/plump/model.py:59-91``.
``synthetic_plump_actor_state`` produces a state dict with the reference
``PlumpActor`` parameter names (``cardgym/games/plump/model.py:170-196``), so
the same arrays load into the reference model (golden fixtures) and into the
B200 trunk (tests, bench) without any checkpoint on disk.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .plump_schema import NUM_CARDS, NUM_NA_PATTERNS, NUM_RANKS, NUM_SUITS, PlumpSchema


@dataclass(frozen=True)
class TrunkConfig:
    d_model: int = 256
    n_layers: int = 6
    n_heads: int = 8
    n_kv_heads: int = 2
    d_ff: int = 768
    per_layer_dim: int = 0
    value_embeddings: str = "off"
    input_norm: bool = True

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def head_group(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def kv_width(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_width(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    @property
    def value_layers(self) -> tuple[int, ...]:
        """Blocks whose V receives a value embedding (trunk.py:58-72 placement)."""

        if self.value_embeddings == "off":
            return ()
        if self.value_embeddings == "all":
            return tuple(range(self.n_layers))
        return tuple(layer for layer in range(self.n_layers) if layer % 2 == (self.n_layers - 1) % 2)

    @property
    def ple_width(self) -> int:
        return self.n_layers * self.per_layer_dim

    @property
    def value_width(self) -> int:
        return len(self.value_layers) * self.kv_width

    def validate(self) -> None:
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads.")
        if self.n_kv_heads > self.n_heads or self.n_heads % self.n_kv_heads:
            raise ValueError("n_kv_heads must divide n_heads.")
        if self.per_layer_dim < 0:
            raise ValueError("per_layer_dim must be non-negative.")
        if self.value_embeddings not in ("off", "alternating", "all"):
            raise ValueError(f"Unknown value_embeddings mode {self.value_embeddings!r}.")


@dataclass(frozen=True)
class PlumpModelConfig:
    """The reference's [model] section; defaults are the rl-v6 architecture."""

    max_players: int = 5
    max_hand_size: int = 10
    d_model: int = 240
    n_layers: int = 16
    n_heads: int = 10
    n_kv_heads: int = 2
    d_ff: int = 720
    per_layer_dim: int = 64
    value_embeddings: str = "alternating"

    def trunk(self) -> TrunkConfig:
        return TrunkConfig(
            d_model=self.d_model,
            n_layers=self.n_layers,
            n_heads=self.n_heads,
            n_kv_heads=self.n_kv_heads,
            d_ff=self.d_ff,
            per_layer_dim=self.per_layer_dim,
            value_embeddings=self.value_embeddings,
            input_norm=True,
        )

    def schema(self) -> PlumpSchema:
        return PlumpSchema(max_players=self.max_players, max_hand_size=self.max_hand_size)


RL_V6 = PlumpModelConfig()
# The piquet-scale trunk's dimensions (d 256, 16 layers, 8 query / 2 KV heads of 32, d_ff 512)
# with the plump field lookup and heads standing in for piquet's card grid and scorers.
PIQUET_SCALE = PlumpModelConfig(d_model=256, n_layers=16, n_heads=8, n_kv_heads=2, d_ff=512, per_layer_dim=64)
# configs/plump/smoke.toml [model]
SMOKE = PlumpModelConfig(d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, per_layer_dim=8)


def synthetic_plump_actor_state(config: PlumpModelConfig, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """Seeded float32 weights under the reference PlumpActor's parameter names.

    Every matrix and embedding is N(0, std); norm gains are 1 + N(0, std) and
    biases N(0, std), so every term of the forward carries signal (the
    reference starts its conditioning tables at zero, cardgym/games/plump/model.py:128-133;
    a test of them needs them non-zero). Row 0 of each NA-pattern table stays
    zero: the padding pattern contributes nothing (model.py:129).
    """

    rng = np.random.default_rng(seed)
    trunk = config.trunk()
    trunk.validate()
    schema = config.schema()
    d, f = trunk.d_model, trunk.d_ff
    rows = schema.field_rows()

    def normal(*shape: int) -> np.ndarray:
        return (std * rng.standard_normal(shape)).astype(np.float32)

    def gain(n: int) -> np.ndarray:
        return (1.0 + std * rng.standard_normal(n)).astype(np.float32)

    state: dict[str, np.ndarray] = {}
    state["card_rank_bias"] = normal(NUM_RANKS)
    state["card_suit_bias"] = normal(NUM_SUITS)
    state["trunk.input_norm.weight"] = gain(d)
    if trunk.per_layer_dim:
        state["trunk.ple_context.weight"] = normal(trunk.ple_width, d)
    for layer in range(trunk.n_layers):
        prefix = f"trunk.blocks.{layer}."
        state[prefix + "ln_attn.weight"] = gain(d)
        state[prefix + "ln_attn.bias"] = normal(d)
        state[prefix + "qkv_proj.weight"] = normal(trunk.qkv_width, d)
        state[prefix + "out_proj.weight"] = normal(d, d)
        state[prefix + "ln_mlp.weight"] = gain(d)
        state[prefix + "ln_mlp.bias"] = normal(d)
        state[prefix + "mlp.0.weight"] = normal(f, d)
        state[prefix + "mlp.0.bias"] = normal(f)
        state[prefix + "mlp.2.weight"] = normal(d, f)
        state[prefix + "mlp.2.bias"] = normal(d)
    state["trunk.final_norm.weight"] = gain(d)
    state["trunk.final_norm.bias"] = normal(d)
    for name, width in (("", d), ("ple_", trunk.ple_width), ("value_", trunk.value_width)):
        if not width:
            continue
        state[f"embedding.{name}fields.weight"] = normal(rows, width)
        pattern = normal(NUM_NA_PATTERNS, width)
        pattern[0] = 0.0
        state[f"embedding.{name}na_pattern.weight"] = pattern
    bids = schema.bid_count
    state["bid_head.weight"] = normal(bids, d)
    state["bid_head.bias"] = normal(bids)
    state["card_rank.weight"] = normal(NUM_RANKS, d)
    state["card_suit.weight"] = normal(NUM_SUITS, d)
    state["value_head.0.weight"] = normal(d, d)
    state["value_head.0.bias"] = normal(d)
    state["value_head.2.weight"] = normal(config.max_players, d)
    state["value_head.2.bias"] = normal(config.max_players)
    return state


def card_head_tables(state: dict[str, np.ndarray]) -> tuple[np.ndarray, np.ndarray]:
    """The 52 play-head rows and biases: rank[r] + suit[s] (cardgym/games/plump/model.py:204-207)."""

    cards = np.arange(NUM_CARDS)
    ranks, suits = cards % NUM_RANKS, cards // NUM_RANKS
    weight = (state["card_rank.weight"][ranks] + state["card_suit.weight"][suits]).astype(np.float32)
    bias = (state["card_rank_bias"][ranks] + state["card_suit_bias"][suits]).astype(np.float32)
    return weight, bias
