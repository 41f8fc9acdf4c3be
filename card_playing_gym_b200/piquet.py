"""Piquet field lookup and card pointer heads on the device.

Reference: cardgym/games/piquet/model.py:255-264 (``_onehot_bags``) and the field part of
``PiquetEmbedding.forward`` 323-345: ids = tokens[..., :NUM_FIELDS] + offsets, and every
table's field sums as one product of one-hot token rows with the tables side by side, in
the autocast dtype (fp32 accumulation, each sum rounded once) or the tables' own. Here the
product is a gather-sum of each distinct selected row (``cg_onehot_bags``). The card-grid
summary that ``PiquetEmbedding.forward`` adds to the first sum stays with the caller.

``CardGrid`` mirrors cardgym/games/piquet/model.py:180-240 (``cards`` and ``forward``): the
per-card features of a token's 32 card codes (``cg_card_grid``, in the reference's bf16
autocast form) and their summary projection (a plain GEMM, left to torch).

``CardScorer`` mirrors cardgym/games/piquet/model.py:348-363: one logit per card from the
readout state and the card's grid features (``cg_card_scorer``), as PiquetActor.policy_logits
(399-411) calls it for the exchange and play heads.

``PiquetActor`` puts them together as the reference's rollout model (model.py:365-411).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from .config import TrunkConfig
from .kv_cache import KVCache
from .trunk import B200Trunk

NUM_FIELDS = 32
CARD_START = NUM_FIELDS
# cardgym/games/piquet/tokens.py:121-128, evaluated: rows of each field in the tables.
FIELD_VOCAB = (8, 4, 3, 2, 33, 9, 9, 4, 4, 9, 76, 9, 3, 4, 64, 5, 3, 13, 3, 5, 13, 13, 100, 100, 141, 141, 6, 2,
               9, 16, 4, 149)
FIELD_ROWS = sum(FIELD_VOCAB)


def field_offsets(vocab: tuple[int, ...] = FIELD_VOCAB) -> list[int]:
    """First table row of each field (``PiquetEmbedding.offsets``; rummy's with its vocabulary)."""

    return [sum(vocab[:i]) for i in range(len(vocab))]


def _lookup_dtype(tables: list[torch.Tensor]) -> torch.dtype:
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return tables[0].dtype


def _bags(ids: torch.Tensor, id_stride: int, fields: int, offsets: list[int] | None, table: torch.Tensor,
          lead: tuple[int, ...]) -> torch.Tensor:
    if table.dtype not in nat.DTYPE_CODES:
        raise TypeError(f"field tables in {table.dtype} are not supported")
    count = ids.shape[0]
    out = torch.empty((count, table.shape[1]), dtype=table.dtype, device=table.device)
    offs = None
    if offsets is not None:
        offs = (nat._i64 * fields)(*offsets)
    nat.call("cg_onehot_bags", nat.ptr(ids), nat.INDEX_CODES[ids.dtype], count, id_stride, fields, offs,
             nat.ptr(table), nat.DTYPE_CODES[table.dtype], table.shape[0], table.shape[1], nat.ptr(out),
             nat.stream_handle(table.device))
    return out.view(*lead, table.shape[1])


def onehot_bags(ids: torch.Tensor, tables: list[torch.Tensor]) -> list[torch.Tensor]:
    """``_onehot_bags(ids, tables)``: ids [..., F] row ids, tables [rows, w_i] -> sums [..., w_i]."""

    dtype = _lookup_dtype(tables)
    flat = ids.reshape(-1, ids.shape[-1])
    if flat.dtype not in nat.INDEX_CODES:
        flat = flat.long()
    flat = flat.contiguous()
    table = torch.cat(tables, dim=1).to(dtype).contiguous()
    sums = _bags(flat, flat.shape[1], flat.shape[1], None, table, tuple(ids.shape[:-1]))
    widths = [t.shape[1] for t in tables]
    return list(sums.split(widths, dim=-1))


class PiquetFieldLookup:
    """The field sums of ``PiquetEmbedding.forward`` with the tables packed once per dtype.

    ``fields`` is ``embedding.fields.weight`` [FIELD_ROWS, d]; ``ple`` and ``values`` the
    optional ``ple_fields``/``value_fields`` tables. Calling it with tokens [..., 64]
    (int16/int32/int64) returns (fields, ple or None, values or None) sums in the lookup
    dtype (the autocast dtype on CUDA, else the tables').
    """

    def __init__(self, fields: torch.Tensor, ple: torch.Tensor | None = None, values: torch.Tensor | None = None,
                 vocab: tuple[int, ...] = FIELD_VOCAB):
        self.parts = [fields] + [t for t in (ple, values) if t is not None]
        self.has = (ple is not None, values is not None)
        # Each field's ids live in their own rows, so no two fields of a token select the same row:
        # the one-hot product (piquet) and the bag sum (rummy's F.embedding_bag) agree.
        self.fields = len(vocab)
        self.offsets = field_offsets(vocab)
        self._packed: dict[torch.dtype, torch.Tensor] = {}

    def table(self, dtype: torch.dtype) -> torch.Tensor:
        packed = self._packed.get(dtype)
        if packed is None:
            packed = torch.cat(self.parts, dim=1).to(dtype).contiguous()
            self._packed[dtype] = packed
        return packed

    def __call__(self, tokens: torch.Tensor):
        dtype = _lookup_dtype(self.parts)
        flat = tokens.reshape(-1, tokens.shape[-1])
        if flat.dtype not in nat.INDEX_CODES:
            flat = flat.long()
        flat = flat.contiguous()
        sums = _bags(flat, flat.shape[1], self.fields, self.offsets, self.table(dtype), tuple(tokens.shape[:-1]))
        parts = iter(sums.split([t.shape[1] for t in self.parts], dim=-1))
        first = next(parts)
        ple = next(parts) if self.has[0] else None
        values = next(parts) if self.has[1] else None
        return first, ple, values


class CardScorer:
    """``CardScorer.forward(hidden [N, d], grid [N, 32, card_width]) -> logits fp32 [N, 32]``.

    Built from the reference module's parameters (``state`` holds ``prefix + "query.weight"``
    and the rest, as in a PiquetActor ``state_dict`` with prefix ``"play_scorer."`` or
    ``"exchange_scorer."``). fp32 arithmetic whatever the grid's dtype.
    """

    NAMES = ("query.weight", "query.bias", "card.weight", "card_id.weight", "norm.weight", "norm.bias",
             "hidden.weight", "hidden.bias", "out.weight", "out.bias")

    def __init__(self, state: dict, prefix: str = "", device: torch.device | str = "cuda"):
        self.params = {
            name: torch.as_tensor(state[prefix + name]).detach().to(device=device, dtype=torch.float32).contiguous()
            for name in self.NAMES
        }
        p = self.params
        dim, d = p["query.weight"].shape
        self.weights = nat.CardScorerWeights(
            d, p["card.weight"].shape[1], dim, p["card_id.weight"].shape[0],
            *[nat.ptr(p[name]) for name in self.NAMES[:8]], nat.ptr(p["out.weight"]), nat.ptr(p["out.bias"]),
        )

    def __call__(self, hidden: torch.Tensor, grid: torch.Tensor) -> torch.Tensor:
        hidden = hidden.float().contiguous()
        if grid.dtype not in nat.DTYPE_CODES:
            grid = grid.float()
        grid = grid.contiguous()
        count = hidden.shape[0]
        logits = torch.empty((count, self.weights.cards), dtype=torch.float32, device=hidden.device)
        nat.call("cg_card_scorer", self.weights, nat.ptr(hidden), count, nat.ptr(grid), nat.DTYPE_CODES[grid.dtype],
                 nat.ptr(logits), nat.stream_handle(hidden.device))
        return logits


def forward_ragged(trunk, lookup: PiquetFieldLookup, tokens: torch.Tensor, positions: torch.Tensor, cache,
                   readout_offsets: torch.Tensor, span: int | None = None, rows: torch.Tensor | None = None,
                   summary: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``SequenceModel.forward_ragged`` (cardgym/nn/model.py:76-89) with the piquet field sums:
    tokens [B, T, 64] -> (field sums + ``summary``, the card-grid summary [B, T, d] if given) ->
    Trunk.condition -> the ragged trunk decode -> final-normed hidden [B, d] at each readout.

    With a bf16 trunk the lookup writes straight into the first tensor-core layer's inputs
    (``cg_bags_forward_ragged``); an fp32 trunk runs lookup, condition and decode as three calls.
    ``workspace`` as in ``B200Trunk.forward_ragged``.
    """

    batch, steps, _ = tokens.shape
    if span is None:
        span = int(positions.max()) + steps
    span = min(span, cache.max_len)
    if trunk.precision != "bf16":
        fields, ple, values = lookup(tokens)
        if summary is not None:
            fields = fields + summary
        x, ple, values = trunk.condition(fields, ple, values)
        return trunk.forward_ragged(x, ple, values, cache, positions, readout_offsets, span=span, rows=rows,
                                    workspace=workspace)
    flat = tokens.reshape(-1, tokens.shape[-1])
    if flat.dtype not in nat.INDEX_CODES:
        flat = flat.long()
    flat = flat.contiguous()
    table = lookup.table(torch.float32)
    extra = None if summary is None else summary.reshape(-1, summary.shape[-1]).float().contiguous()
    workspace = trunk.workspace(batch, steps, workspace)
    hidden = torch.empty((batch, trunk.config.d_model), device=trunk.device)
    offsets = (nat._i64 * lookup.fields)(*lookup.offsets)
    nat.call("cg_bags_forward_ragged", trunk.dims, nat.ptr(trunk.blob), nat.ptr(flat), nat.INDEX_CODES[flat.dtype],
             flat.shape[1], lookup.fields, offsets, nat.ptr(table), table.shape[0], nat.ptr(extra), batch, steps,
             nat.ptr(positions.to(torch.int64).contiguous()), nat.ptr(readout_offsets.to(torch.int64).contiguous()),
             nat.ptr(None if rows is None else rows.to(torch.int64).contiguous()), int(span), nat.ptr(cache.k_pool),
             nat.ptr(cache.v_pool), nat.DTYPE_CODES[cache.dtype], cache.capacity, cache.max_len,
             nat.PRECISIONS[trunk.precision], nat.ptr(workspace), workspace.numel(), nat.ptr(hidden),
             nat.stream_handle(trunk.device))
    return hidden


class CardGrid:
    """``CardGrid``: card codes [..., 32] -> (cards fp32 [..., 32, width], summary [..., d]).

    Rummy's ledger grid (cardgym/games/rummy/model.py:166-230: 52 codes, 13 ranks, a circular
    5-tap convolution) is the same class built from that module's parameters.

    Built from the reference module's parameters (``prefix + "code.weight"`` etc., as in a
    PiquetActor ``state_dict`` with prefix ``"embedding.grid."``). ``cards`` is computed as the
    reference computes it under bf16 autocast (its rollout precision); ``forward`` adds the
    summary projection with torch, honouring the caller's autocast state like the reference.
    """

    def __init__(self, state: dict, prefix: str = "", device: torch.device | str = "cuda", blocks: int | None = None,
                 circular: bool | None = None):
        get = lambda name: torch.as_tensor(state[prefix + name]).detach().to(device=device, dtype=torch.float32).contiguous()  # noqa: E731
        if blocks is None:
            blocks = 0
            while f"{prefix}blocks.{blocks}.norm.weight" in state:
                blocks += 1
        self.params = {"code": get("code.weight"), "rank": get("rank.weight"), "norm": get("norm.weight")}
        self.summary = get("summary.weight") if prefix + "summary.weight" in state else None
        names = ("norm.weight", "along_rank.weight", "along_rank.bias", "across_suits.weight", "out.weight", "out.bias")
        self.blocks = [{n: get(f"blocks.{b}.{n}") for n in names} for b in range(blocks)]
        width = self.params["code"].shape[1]
        hidden, _, taps = self.blocks[0]["along_rank.weight"].shape if blocks else (64, width, 3)
        ranks = self.params["rank"].shape[0]
        w = nat.CardGridWeights()
        w.width, w.hidden, w.kernel, w.blocks, w.codes = width, hidden, taps, blocks, self.params["code"].shape[0]
        # Piquet's 8-rank grid pads with zeros; rummy's 13-rank ledger grid wraps around.
        w.ranks, w.circular = ranks, int(ranks == 13 if circular is None else circular)
        self.cards_per_token = 4 * ranks
        w.code_emb, w.rank_emb, w.final_norm = (nat.ptr(self.params[k]) for k in ("code", "rank", "norm"))
        for b, blk in enumerate(self.blocks):
            w.norm_w[b] = nat.ptr(blk["norm.weight"])
            w.conv_w[b] = nat.ptr(blk["along_rank.weight"])
            w.conv_b[b] = nat.ptr(blk["along_rank.bias"])
            w.across_w[b] = nat.ptr(blk["across_suits.weight"])
            w.out_w[b] = nat.ptr(blk["out.weight"])
            w.out_b[b] = nat.ptr(blk["out.bias"])
        self.weights = w
        self.width = width

    def cards(self, codes: torch.Tensor) -> torch.Tensor:
        """Per-card features [..., cards, width] of card codes [..., cards] (any view of token rows)."""

        lead = codes.shape[:-1]
        flat = codes.reshape(-1, codes.shape[-1])
        if flat.dtype not in nat.INDEX_CODES:
            flat = flat.long()
        if flat.stride(-1) != 1:
            flat = flat.contiguous()
        count = flat.shape[0]
        cards = self.cards_per_token
        out = torch.empty((count, cards, self.width), dtype=torch.float32, device=flat.device)
        nat.call("cg_card_grid", self.weights, nat.ptr(flat), nat.INDEX_CODES[flat.dtype], count, flat.stride(0),
                 nat.ptr(out), nat.stream_handle(flat.device))
        return out.view(*lead, cards, self.width)

    def __call__(self, codes: torch.Tensor):
        cards = self.cards(codes)
        if self.summary is None:
            return cards, None
        return cards, torch.nn.functional.linear(cards.flatten(-2), self.summary)


HEADS = ("exchange", "declare", "play")  # cardgym/games/piquet/engine.py:56
PLAYERS = 2


@dataclass(frozen=True)
class PiquetModelConfig:
    """The reference's piquet ``[model]`` section (cardgym/games/piquet/model.py:79-108): the
    16-layer actor by default."""

    d_model: int = 256
    n_layers: int = 16
    n_heads: int = 8
    n_kv_heads: int = 2
    d_ff: int = 512
    per_layer_dim: int = 64
    value_embeddings: str = "alternating"
    card_width: int = 32
    card_hidden: int = 64
    card_layers: int = 2
    card_kernel: int = 3
    score_dim: int = 64

    def trunk(self) -> TrunkConfig:
        return TrunkConfig(d_model=self.d_model, n_layers=self.n_layers, n_heads=self.n_heads,
                           n_kv_heads=self.n_kv_heads, d_ff=self.d_ff, per_layer_dim=self.per_layer_dim,
                           value_embeddings=self.value_embeddings, input_norm=True)


class PiquetActor:
    """The rollout side of ``PiquetActor`` (cardgym/games/piquet/model.py:365-411) over its
    ``state_dict`` names: ``forward_ragged`` runs the card grid over every appended token, adds
    its summary to the one-hot field sums, and decodes them through the trunk (fused into the
    first tensor-core layer with a bf16 trunk); ``pop_context`` hands back the grid cards of
    those tokens, which ``policy_logits`` scores for the exchange and play heads
    (``CardScorer``; the exchange head appends the stop logit) while the declare head and the
    player values are plain projections of the readout state.

    ``precision = "bf16"`` is the reference's rollout form (bf16 autocast): the card grid in its
    autocast rounding (always: ``CardGrid.cards``), the summary projection under bf16 autocast,
    bf16 trunk GEMM operands. The scorers, the declare and stop heads and the value MLP run in
    fp32 in both precisions (the reference runs those few small projections in bf16 under
    autocast). The heads read only the readout state and its grid cards, so a wave can be
    captured by ``graphs.DecodeGraphs``.
    """

    policy_heads = HEADS
    # Every head reads only the readout state and its grid cards (model.py:367-370).
    graphable_heads = True

    def __init__(self, config: PiquetModelConfig, state: dict, device: torch.device | str = "cuda",
                 precision: str = "bf16") -> None:
        self.config = config
        self.device = torch.device(device)
        self.precision = precision
        self.trunk = B200Trunk(config.trunk(), state, self.device, precision)

        def get(name: str) -> torch.Tensor | None:
            if name not in state:
                return None
            return torch.as_tensor(state[name]).detach().to(device=self.device, dtype=torch.float32).contiguous()

        self.lookup = PiquetFieldLookup(get("embedding.fields.weight"), get("embedding.ple_fields.weight"),
                                        get("embedding.value_fields.weight"))
        self.grid = CardGrid(state, "embedding.grid.", self.device, blocks=config.card_layers, circular=False)
        self.exchange_scorer = CardScorer(state, "exchange_scorer.", self.device)
        self.play_scorer = CardScorer(state, "play_scorer.", self.device)
        self.linear = {name: (get(f"{name}.weight"), get(f"{name}.bias"))
                       for name in ("stop_head", "declare_head", "value_head.0", "value_head.2")}
        self.kept: torch.Tensor | None = None

    @property
    def trunk_config(self) -> TrunkConfig:
        return self.trunk.config

    def new_cache(self, capacity: int, max_len: int, dtype: torch.dtype = torch.float16) -> KVCache:
        return self.trunk.new_cache(capacity, max_len, dtype)

    def step_workspace_bytes(self, batch: int, steps: int) -> int:
        return self.trunk.step_workspace_bytes(batch, steps)

    def _grid(self, tokens: torch.Tensor):
        codes = tokens[..., CARD_START:]
        if self.precision == "bf16":
            with torch.autocast("cuda", dtype=torch.bfloat16):
                return self.grid(codes)
        return self.grid(codes)

    def forward_ragged(self, tokens: torch.Tensor, positions: torch.Tensor, cache: KVCache,
                       readout_offsets: torch.Tensor, span: int | None = None, rows: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
        """Append a padded run per cache row 0..B-1 (or ``rows``); hidden at each readout [B, d]
        (cardgym/nn/model.py:76-89). Keeps the appended tokens' grid cards for ``pop_context``."""

        cards, summary = self._grid(tokens)
        self.kept = cards
        return forward_ragged(self.trunk, self.lookup, tokens, positions, cache, readout_offsets, span=span,
                              rows=rows, summary=summary, workspace=workspace)

    def forward_prefill(self, tokens: torch.Tensor, cache: KVCache, rows: torch.Tensor | None) -> torch.Tensor:
        """Fresh prefixes [B, T, 64] at positions 0..T-1; hidden at the last position."""

        batch, steps, _ = tokens.shape
        positions = torch.zeros(batch, dtype=torch.int64, device=self.device)
        offsets = torch.full((batch,), steps - 1, dtype=torch.int64, device=self.device)
        return self.forward_ragged(tokens, positions, cache, offsets, span=steps, rows=rows)

    def pop_context(self) -> torch.Tensor | None:
        """The grid cards [B, T, 32, card_width] of the last forward's tokens (model.py:389-391)."""

        cards, self.kept = self.kept, None
        return cards

    def _project(self, name: str, x: torch.Tensor) -> torch.Tensor:
        weight, bias = self.linear[name]
        return torch.nn.functional.linear(x.float(), weight, bias)

    def policy_logits(self, hidden: torch.Tensor, head: str, features=None, tokens=None, context=None) -> torch.Tensor:
        """fp32 logits of ``head`` at each readout (model.py:393-406)."""

        if head == "declare":
            return self._project("declare_head", hidden)
        if head not in ("exchange", "play"):
            raise ValueError(f"Unknown piquet policy head {head!r}.")
        if context is None:
            if tokens is None:
                raise ValueError("Card heads need the readout tokens or their grid features.")
            context = self.grid.cards(tokens[..., CARD_START:])
        if head == "play":
            return self.play_scorer(hidden, context)
        return torch.cat([self.exchange_scorer(hidden, context), self._project("stop_head", hidden)], dim=-1)

    def player_values(self, hidden: torch.Tensor) -> torch.Tensor:
        """value_head: Linear -> exact GELU -> Linear, fp32 [N, 2] (cardgym/nn/model.py:12-17)."""

        inner = torch.nn.functional.gelu(self._project("value_head.0", hidden))
        return self._project("value_head.2", inner)


def synthetic_actor_parts(trunk: TrunkConfig, rows: int, seed: int, std: float = 0.02):
    """(state, normal, gain) for a synthetic actor: the trunk's parameters and the field tables
    under the reference's names, plus the seeded draw helpers for the rest. Matrices and
    embeddings are N(0, std), norm gains 1 + N(0, std), biases N(0, std)."""

    import numpy as np

    from .config import PlumpModelConfig, synthetic_plump_actor_state

    plump = PlumpModelConfig(d_model=trunk.d_model, n_layers=trunk.n_layers, n_heads=trunk.n_heads,
                             n_kv_heads=trunk.n_kv_heads, d_ff=trunk.d_ff, per_layer_dim=trunk.per_layer_dim,
                             value_embeddings=trunk.value_embeddings)
    state = {k: v for k, v in synthetic_plump_actor_state(plump, seed=seed, std=std).items() if k.startswith("trunk.")}
    rng = np.random.default_rng(seed + 1)

    def normal(*shape: int):
        return (std * rng.standard_normal(shape)).astype(np.float32)

    def gain(n: int):
        return (1.0 + std * rng.standard_normal(n)).astype(np.float32)

    state["embedding.fields.weight"] = normal(rows, trunk.d_model)
    if trunk.ple_width:
        state["embedding.ple_fields.weight"] = normal(rows, trunk.ple_width)
    if trunk.value_width:
        state["embedding.value_fields.weight"] = normal(rows, trunk.value_width)
    return state, normal, gain


def synthetic_grid_state(state: dict, normal, gain, *, d: int, codes: int, ranks: int, cards: int, width: int,
                         hidden: int, blocks: int, kernel: int, prefix: str = "embedding.grid.") -> None:
    """A card grid's parameters (``CardGrid``, piquet/model.py:180-240) added to ``state``."""

    state[prefix + "code.weight"] = normal(codes, width)
    state[prefix + "rank.weight"] = normal(ranks, width)
    for b in range(blocks):
        p = f"{prefix}blocks.{b}."
        state[p + "norm.weight"] = gain(width)
        state[p + "along_rank.weight"] = normal(hidden, width, kernel)
        state[p + "along_rank.bias"] = normal(hidden)
        state[p + "across_suits.weight"] = normal(hidden, width)
        state[p + "out.weight"] = normal(width, hidden)
        state[p + "out.bias"] = normal(width)
    state[prefix + "norm.weight"] = gain(width)
    state[prefix + "summary.weight"] = normal(d, cards * width)


def synthetic_piquet_actor_state(config: PiquetModelConfig, seed: int = 0) -> dict:
    """Seeded float32 weights under the reference ``PiquetActor``'s parameter names and shapes
    (the heads it rolls out with; the auxiliary head is left out)."""

    trunk = config.trunk()
    d, s, w = config.d_model, config.score_dim, config.card_width
    state, normal, gain = synthetic_actor_parts(trunk, FIELD_ROWS, seed)
    synthetic_grid_state(state, normal, gain, d=d, codes=12, ranks=8, cards=32, width=w, hidden=config.card_hidden,
                         blocks=config.card_layers, kernel=config.card_kernel)
    for scorer in ("exchange_scorer.", "play_scorer."):
        state.update({scorer + "query.weight": normal(s, d), scorer + "query.bias": normal(s),
                      scorer + "card.weight": normal(s, w), scorer + "card_id.weight": normal(32, s),
                      scorer + "norm.weight": gain(s), scorer + "norm.bias": normal(s),
                      scorer + "hidden.weight": normal(s, s), scorer + "hidden.bias": normal(s),
                      scorer + "out.weight": normal(1, s), scorer + "out.bias": normal(1)})
    state.update({"stop_head.weight": normal(1, d), "stop_head.bias": normal(1),
                  "declare_head.weight": normal(2, d), "declare_head.bias": normal(2),
                  "value_head.0.weight": normal(d, d), "value_head.0.bias": normal(d),
                  "value_head.2.weight": normal(PLAYERS, d), "value_head.2.bias": normal(PLAYERS)})
    return state
