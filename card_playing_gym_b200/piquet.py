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
"""

from __future__ import annotations

import torch

from . import _native as nat

NUM_FIELDS = 32
CARD_START = NUM_FIELDS
# cardgym/games/piquet/tokens.py:121-128, evaluated: rows of each field in the tables.
FIELD_VOCAB = (8, 4, 3, 2, 33, 9, 9, 4, 4, 9, 76, 9, 3, 4, 64, 5, 3, 13, 3, 5, 13, 13, 100, 100, 141, 141, 6, 2,
               9, 16, 4, 149)
FIELD_ROWS = sum(FIELD_VOCAB)


def field_offsets() -> list[int]:
    """First table row of each field (``PiquetEmbedding.offsets``)."""

    return [sum(FIELD_VOCAB[:i]) for i in range(NUM_FIELDS)]


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

    def __init__(self, fields: torch.Tensor, ple: torch.Tensor | None = None, values: torch.Tensor | None = None):
        self.parts = [fields] + [t for t in (ple, values) if t is not None]
        self.has = (ple is not None, values is not None)
        self.offsets = field_offsets()
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
        sums = _bags(flat, flat.shape[1], NUM_FIELDS, self.offsets, self.table(dtype), tuple(tokens.shape[:-1]))
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
                   summary: torch.Tensor | None = None) -> torch.Tensor:
    """``SequenceModel.forward_ragged`` (cardgym/nn/model.py:76-89) with the piquet field sums:
    tokens [B, T, 64] -> (field sums + ``summary``, the card-grid summary [B, T, d] if given) ->
    Trunk.condition -> the ragged trunk decode -> final-normed hidden [B, d] at each readout.

    With a bf16 trunk the lookup writes straight into the first tensor-core layer's inputs
    (``cg_bags_forward_ragged``); an fp32 trunk runs lookup, condition and decode as three calls.
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
        return trunk.forward_ragged(x, ple, values, cache, positions, readout_offsets, span=span, rows=rows)
    flat = tokens.reshape(-1, tokens.shape[-1])
    if flat.dtype not in nat.INDEX_CODES:
        flat = flat.long()
    flat = flat.contiguous()
    table = lookup.table(torch.float32)
    extra = None if summary is None else summary.reshape(-1, summary.shape[-1]).float().contiguous()
    need = nat.query("cg_trunk_step_workspace_bytes", trunk.dims, batch, steps, nat.PRECISIONS[trunk.precision])
    workspace = nat.Workspace.get(trunk.device, need)
    hidden = torch.empty((batch, trunk.config.d_model), device=trunk.device)
    offsets = (nat._i64 * NUM_FIELDS)(*lookup.offsets)
    nat.call("cg_bags_forward_ragged", trunk.dims, nat.ptr(trunk.blob), nat.ptr(flat), nat.INDEX_CODES[flat.dtype],
             flat.shape[1], NUM_FIELDS, offsets, nat.ptr(table), table.shape[0], nat.ptr(extra), batch, steps,
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
