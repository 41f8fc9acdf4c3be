"""The plump actor's rollout path on the B200: field lookup -> trunk decode -> heads -> sampling.

Mirrors the reference ``PlumpActor`` surface used by the collectors
(cardgym/games/plump/model.py:170-217 and cardgym/nn/model.py:60-106):
``forward_ragged(tokens, positions, cache, readout_offsets, span, rows)``,
``forward_prefill(tokens, cache, rows)``, ``policy_logits(hidden, head)``,
``player_values(hidden)``, ``new_cache(capacity, max_len, dtype)``, plus ``decide``,
the fused heads + legal masking + sampling step that replaces
``launch_policies`` + ``sample_decisions`` (cardgym/rl/selfplay.py:486-567).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _native as nat
from .config import PlumpModelConfig, card_head_tables
from .kv_cache import KVCache
from .plump_schema import (
    FIELDS, NUM_CARDS, NUM_NA_PATTERNS, NUM_RANKS, REMAINING_HAND_SLOTS, SLOT_NA_PATTERN, SLOT_REMAINING_HAND,
    SLOT_TYPE, TOKEN_TRICK_WIN, TOKEN_WIDTH,
)
from .trunk import B200Trunk, _as_numpy

POLICY_HEADS = ("bid", "play")


def schema_struct(config: PlumpModelConfig) -> nat.PlumpSchemaC:
    schema = config.schema()
    sc = nat.PlumpSchemaC()
    sc.field_count = len(FIELDS)
    for i, (slot, offset, na) in enumerate(zip(FIELDS, schema.field_offsets(), schema.field_na_ids())):
        sc.field_slots[i] = slot
        sc.field_offsets[i] = offset
        sc.field_na[i] = na
    sc.field_rows = schema.field_rows()
    sc.pattern_rows = NUM_NA_PATTERNS
    sc.token_width = TOKEN_WIDTH
    sc.slot_type = SLOT_TYPE
    sc.slot_pattern = SLOT_NA_PATTERN
    sc.slot_hand = SLOT_REMAINING_HAND
    sc.hand_slots = REMAINING_HAND_SLOTS
    sc.trick_win_type = TOKEN_TRICK_WIN
    sc.rank_offset = schema.rank_offset
    sc.suit_offset = schema.suit_offset
    sc.num_cards = NUM_CARDS
    sc.num_ranks = NUM_RANKS
    return sc


def lookup_table(config: PlumpModelConfig, state: dict) -> np.ndarray:
    """[field rows + pattern rows, d | ple | value] fp32: the three embedders side by side."""

    trunk = config.trunk()
    rows = config.schema().field_rows()
    parts = []
    for name, width in (("", trunk.d_model), ("ple_", trunk.ple_width), ("value_", trunk.value_width)):
        if not width:
            continue
        fields = _as_numpy(state[f"embedding.{name}fields.weight"])
        patterns = _as_numpy(state[f"embedding.{name}na_pattern.weight"])
        assert fields.shape == (rows, width) and patterns.shape == (NUM_NA_PATTERNS, width)
        parts.append(np.concatenate([fields, patterns], axis=0))
    return np.ascontiguousarray(np.concatenate(parts, axis=1), dtype=np.float32)


def heads_blob(config: PlumpModelConfig, state: dict) -> tuple[np.ndarray, nat.HeadsDesc]:
    d = config.d_model
    card_w, card_b = card_head_tables({k: _as_numpy(v) for k, v in state.items() if k.startswith("card_")})
    pieces = [
        _as_numpy(state["bid_head.weight"]), _as_numpy(state["bid_head.bias"]), card_w, card_b,
        _as_numpy(state["value_head.0.weight"]), _as_numpy(state["value_head.0.bias"]),
        _as_numpy(state["value_head.2.weight"]), _as_numpy(state["value_head.2.bias"]),
    ]
    offsets, at = [], 0
    for piece in pieces:
        offsets.append(at)
        at += (piece.size + 63) // 64 * 64
    blob = np.zeros(at, dtype=np.float32)
    for piece, offset in zip(pieces, offsets):
        blob[offset : offset + piece.size] = piece.reshape(-1)
    desc = nat.HeadsDesc()
    desc.d_model = d
    desc.n_policy = 2
    desc.value_outputs = config.max_players
    widths = (config.schema().bid_count, NUM_CARDS)
    desc.max_width = max(widths)
    for head, width in enumerate(widths):
        desc.width[head] = width
        desc.weight_offset[head] = offsets[2 * head]
        desc.bias_offset[head] = offsets[2 * head + 1]
    desc.value_w1, desc.value_b1, desc.value_w2, desc.value_b2 = offsets[4:8]
    return blob, desc


class PlumpActor:
    """Rollout-side plump actor over reference-named weights (actor.pt ``state_dict`` or synthetic)."""

    policy_heads = POLICY_HEADS
    # The heads read only the readout state and the lookup has no host synchronisation, so a
    # wave can be captured whole (graphs.DecodeGraphs).
    graphable_heads = True

    def __init__(self, config: PlumpModelConfig, state: dict, device: torch.device | str = "cuda", precision: str = "bf16") -> None:
        self.config = config
        self.device = torch.device(device)
        self.precision = precision
        self.trunk = B200Trunk(config.trunk(), state, self.device, precision)
        self.schema = schema_struct(config)
        self.table = torch.from_numpy(lookup_table(config, state)).to(self.device)
        blob, self.heads_desc = heads_blob(config, state)
        self.heads = torch.from_numpy(blob).to(self.device)
        self.head_index = {name: i for i, name in enumerate(POLICY_HEADS)}

    @property
    def trunk_config(self):
        return self.trunk.config

    def new_cache(self, capacity: int, max_len: int, dtype: torch.dtype = torch.float16) -> KVCache:
        return self.trunk.new_cache(capacity, max_len, dtype)

    # -- embedding ----------------------------------------------------------------
    def embed_lookup(self, tokens: torch.Tensor) -> torch.Tensor:
        """Raw field-lookup sums [..., d | ple | value] (PlumpEmbedding.forward, model.py:135-167)."""

        lead = tokens.shape[:-1]
        flat = tokens.reshape(-1, tokens.shape[-1]).contiguous()
        out = torch.empty((flat.shape[0], self.trunk.lookup_width), device=self.device)
        nat.call("cg_plump_embed", self.schema, nat.ptr(self.table), self.trunk.lookup_width, nat.ptr(flat),
                 nat.INDEX_CODES[flat.dtype], flat.shape[0], nat.ptr(out), nat.stream_handle(self.device))
        return out.view(*lead, self.trunk.lookup_width)

    def embed(self, tokens: torch.Tensor):
        c = self.trunk.config
        lookup = self.embed_lookup(tokens)
        x = lookup[..., : c.d_model]
        ple = lookup[..., c.d_model : c.d_model + c.ple_width] if c.ple_width else None
        values = lookup[..., c.d_model + c.ple_width :] if c.value_width else None
        return x, ple, values

    def prepare(self, tokens: torch.Tensor):
        return self.trunk.condition_lookup(self.embed_lookup(tokens))

    # -- trunk --------------------------------------------------------------------
    def forward_ragged(
        self,
        tokens: torch.Tensor,
        positions: torch.Tensor,
        cache: KVCache,
        readout_offsets: torch.Tensor,
        span: int | None = None,
        rows: torch.Tensor | None = None,
        workspace: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Append a padded run per cache row 0..B-1 (or ``rows``); hidden at each readout [B, d] (model.py:76-89).

        ``workspace`` (uint8, at least ``step_workspace_bytes``) pins the step's scratch memory,
        for callers that capture the step in a CUDA graph; by default a shared buffer is used.
        """

        batch, steps, _ = tokens.shape
        if span is None:
            span = int(positions.max()) + steps
        span = min(span, cache.max_len)
        tokens = tokens.contiguous()
        precision = nat.PRECISIONS[self.precision]
        need = self.step_workspace_bytes(batch, steps)
        if workspace is None:
            workspace = nat.Workspace.get(self.device, need)
        elif workspace.numel() < need:
            raise ValueError(f"workspace of {workspace.numel()} bytes < {need} needed")
        hidden = torch.empty((batch, self.config.d_model), device=self.device)
        nat.call(
            "cg_plump_forward_ragged", self.trunk.dims, nat.ptr(self.trunk.blob), self.schema, nat.ptr(self.table),
            nat.ptr(tokens), nat.INDEX_CODES[tokens.dtype], batch, steps, nat.ptr(positions.to(torch.int64).contiguous()),
            nat.ptr(readout_offsets.to(torch.int64).contiguous()),
            nat.ptr(None if rows is None else rows.to(torch.int64).contiguous()), int(span), nat.ptr(cache.k_pool),
            nat.ptr(cache.v_pool), nat.DTYPE_CODES[cache.dtype], cache.capacity, cache.max_len, precision,
            nat.ptr(workspace), workspace.numel(), nat.ptr(hidden), nat.stream_handle(self.device),
        )
        return hidden

    def step_workspace_bytes(self, batch: int, steps: int) -> int:
        return nat.query("cg_plump_step_workspace_bytes", self.trunk.dims, batch, steps, nat.PRECISIONS[self.precision])

    def forward_prefill(self, tokens: torch.Tensor, cache: KVCache, rows: torch.Tensor | None) -> torch.Tensor:
        """Encode fresh prefixes [B, T, W] at positions 0..T-1; hidden at the last position (trunk.py:376-389).

        The same arithmetic as a ragged append of the whole prefix at length 0.
        """

        batch, steps, _ = tokens.shape
        positions = torch.zeros(batch, dtype=torch.int64, device=self.device)
        offsets = torch.full((batch,), steps - 1, dtype=torch.int64, device=self.device)
        return self.forward_ragged(tokens, positions, cache, offsets, span=steps, rows=rows)

    # -- heads --------------------------------------------------------------------
    def decide(
        self,
        hidden: torch.Tensor,
        heads: torch.Tensor,
        legal: torch.Tensor,
        uniforms: torch.Tensor,
        hidden_rows: torch.Tensor | None = None,
        *,
        logits: bool = True,
        values: bool = True,
    ):
        """Heads + masked softmax + inverse-CDF draw for each decision.

        ``heads`` int32 [D] (0 bid, 1 play), ``legal`` bool/uint8 [D, max_width],
        ``uniforms`` float64 [D] (one draw per decision from the game's own RNG,
        selfplay.py:547). Returns (logits, probs, actions int64, values) with
        logits/probs fp32 [D, max_width] (zero past a head's width).
        """

        count = heads.shape[0] if hidden_rows is None else hidden_rows.shape[0]
        width = self.heads_desc.max_width
        legal = legal.to(torch.uint8).contiguous()
        if legal.shape != (count, width):
            raise ValueError(f"legal must be [{count}, {width}]")
        out_logits = torch.empty((count, width), device=self.device) if logits else None
        probs = torch.empty((count, width), device=self.device)
        actions = torch.empty(count, dtype=torch.int64, device=self.device)
        out_values = torch.empty((count, self.config.max_players), device=self.device) if values else None
        nat.call(
            "cg_plump_decide", self.heads_desc, nat.ptr(self.heads), nat.ptr(hidden.float().contiguous()),
            nat.ptr(None if hidden_rows is None else hidden_rows.to(torch.int64).contiguous()), count,
            nat.ptr(heads.to(torch.int32).contiguous()), nat.ptr(legal), nat.ptr(uniforms.to(torch.float64).contiguous()),
            nat.ptr(out_logits), nat.ptr(probs), nat.ptr(actions), nat.ptr(out_values), nat.stream_handle(self.device),
        )
        return out_logits, probs, actions, out_values

    def policy_logits(self, hidden: torch.Tensor, head: str, features=None, tokens=None, context=None) -> torch.Tensor:
        if head not in self.head_index:
            raise ValueError(f"Unknown plump policy head {head!r}.")
        flat = hidden.reshape(-1, hidden.shape[-1])
        count = flat.shape[0]
        heads = torch.full((count,), self.head_index[head], dtype=torch.int32, device=self.device)
        legal = torch.ones((count, self.heads_desc.max_width), dtype=torch.uint8, device=self.device)
        uniforms = torch.zeros(count, dtype=torch.float64, device=self.device)
        logits, *_ = self.decide(flat, heads, legal, uniforms, values=False)
        width = self.heads_desc.width[self.head_index[head]]
        return logits[:, :width].reshape(*hidden.shape[:-1], width)

    def player_values(self, hidden: torch.Tensor) -> torch.Tensor:
        flat = hidden.reshape(-1, hidden.shape[-1])
        count = flat.shape[0]
        heads = torch.zeros(count, dtype=torch.int32, device=self.device)
        legal = torch.ones((count, self.heads_desc.max_width), dtype=torch.uint8, device=self.device)
        uniforms = torch.zeros(count, dtype=torch.float64, device=self.device)
        *_, values = self.decide(flat, heads, legal, uniforms, logits=False)
        return values.reshape(*hidden.shape[:-1], self.config.max_players)
