"""Rummy candidate pointer head on the device.

Reference: cardgym/games/rummy/model.py:292-357 (``CandidateScorer.forward``), called by
``RummyActor.policy_logits`` (391-399) with the candidate features that
cardgym/games/rummy/selfplay.py:28-50 builds: per candidate its kind, the cards it moves
(``cards``), a lay-off's target meld (``target``), NO_CARD-padded to MAX_MELD_CARDS, and for
draw decisions the counts of each card type it takes from the pile (``taken``).

``RummyActor`` is the reference's rollout model around it (model.py:359-402).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from .config import TrunkConfig
from .kv_cache import KVCache
from .trunk import B200Trunk

NUM_CARDS = 52
NO_CARD = NUM_CARDS
MAX_MELD_CARDS = 13


class CandidateScorer:
    """``CandidateScorer.forward(hidden, grid, kind, cards, target, taken=None) -> logits fp32 [N, K]``.

    Built from the reference module's parameters (``prefix + "query.weight"`` etc., as in a
    RummyActor ``state_dict`` with prefix ``"scorer."``). fp32 arithmetic.
    """

    NAMES = ("query.weight", "query.bias", "card.weight", "target.weight", "taken.weight", "card_id.weight",
             "target_id.weight", "taken_id.weight", "kind.weight", "size.weight", "norm.weight", "norm.bias",
             "hidden.weight", "hidden.bias", "out.weight", "out.bias")

    def __init__(self, state: dict, prefix: str = "", device: torch.device | str = "cuda"):
        self.params = {
            name: torch.as_tensor(state[prefix + name]).detach().to(device=device, dtype=torch.float32).contiguous()
            for name in self.NAMES
        }
        p = self.params
        dim, d = p["query.weight"].shape
        self.weights = nat.CandidateScorerWeights(
            d, p["card.weight"].shape[1], dim, p["card_id.weight"].shape[0], p["kind.weight"].shape[0],
            p["size.weight"].shape[0], *[nat.ptr(p[name]) for name in self.NAMES],
        )

    def __call__(self, hidden: torch.Tensor, grid: torch.Tensor, kind: torch.Tensor, cards: torch.Tensor,
                 target: torch.Tensor, taken: torch.Tensor | None = None) -> torch.Tensor:
        count, candidates = kind.shape
        if cards.shape[-1] != target.shape[-1]:
            raise ValueError("cards and target lists must have the same length (the reference's slot layout)")
        hidden = hidden.float().contiguous()
        if grid.dtype not in nat.DTYPE_CODES:
            grid = grid.float()
        grid = grid.contiguous()
        kind = kind.long().contiguous()
        cards = cards.long().contiguous()
        target = target.long().contiguous()
        if taken is not None:
            taken = taken.float().contiguous()
        logits = torch.empty((count, candidates), dtype=torch.float32, device=hidden.device)
        nat.call("cg_candidate_scorer", self.weights, nat.ptr(hidden), count, candidates, cards.shape[-1],
                 nat.ptr(grid), nat.DTYPE_CODES[grid.dtype], nat.ptr(kind), nat.ptr(cards), nat.ptr(target),
                 nat.ptr(taken), nat.ptr(logits), nat.stream_handle(hidden.device))
        return logits


# cardgym/games/rummy/tokens.py:87-124: a token's 26 field ids (each within its vocabulary),
# then a 52-code ledger (CARD_START = 26, codes < CARD_VOCAB = 570).
NUM_FIELDS = 26
CARD_START = NUM_FIELDS
FIELD_VOCAB = (2, 3, 7, 53, 3, 14, 30, 53, 4, 4, 53, 63, 53, 8, 16, 105, 63, 64, 64, 64, 64, 16, 5, 3, 64, 53)
CARD_VOCAB = 570
MAX_PLAYERS = 4  # cardgym/games/rummy/engine.py:65
HEADS = ("draw", "play")


@dataclass(frozen=True)
class RummyModelConfig:
    """The reference's rummy ``[model]`` section (cardgym/games/rummy/model.py:55-84)."""

    d_model: int = 256
    n_layers: int = 8
    n_heads: int = 8
    n_kv_heads: int = 2
    d_ff: int = 768
    per_layer_dim: int = 64
    value_embeddings: str = "alternating"
    ledger_width: int = 32
    ledger_hidden: int = 64
    ledger_layers: int = 2
    ledger_kernel: int = 5
    score_dim: int = 64

    def trunk(self) -> TrunkConfig:
        return TrunkConfig(d_model=self.d_model, n_layers=self.n_layers, n_heads=self.n_heads,
                           n_kv_heads=self.n_kv_heads, d_ff=self.d_ff, per_layer_dim=self.per_layer_dim,
                           value_embeddings=self.value_embeddings, input_norm=True)


class RummyActor:
    """The rollout side of ``RummyActor`` (cardgym/games/rummy/model.py:359-402) over its
    ``state_dict`` names: the ledger grid (13 ranks, circular convolution) over every appended
    token, its summary added to the field sums (``RummyEmbedding.forward`` 264-290) inside the
    fused first trunk layer, the trunk, ``pop_context`` with the appended tokens' ledger cards,
    and ``CandidateScorer`` over each decision's candidate features for both heads.

    Rummy's field sums are ``F.embedding_bag`` sums; every field's ids live in their own table
    rows, so they equal the one-hot product the piquet lookup computes (``PiquetFieldLookup``
    with rummy's vocabulary). Precision as ``piquet.PiquetActor``. The heads need per-decision
    candidate features, so, as in the reference, rummy waves are not graph-captured.
    """

    policy_heads = HEADS
    graphable_heads = False

    def __init__(self, config: RummyModelConfig, state: dict, device: torch.device | str = "cuda",
                 precision: str = "bf16") -> None:
        from .piquet import CardGrid, PiquetFieldLookup

        self.config = config
        self.device = torch.device(device)
        self.precision = precision
        self.trunk = B200Trunk(config.trunk(), state, self.device, precision)

        def get(name: str) -> torch.Tensor | None:
            if name not in state:
                return None
            return torch.as_tensor(state[name]).detach().to(device=self.device, dtype=torch.float32).contiguous()

        self.lookup = PiquetFieldLookup(get("embedding.fields.weight"), get("embedding.ple_fields.weight"),
                                        get("embedding.value_fields.weight"), vocab=FIELD_VOCAB)
        self.grid = CardGrid(state, "embedding.grid.", self.device, blocks=config.ledger_layers, circular=True)
        self.scorer = CandidateScorer(state, "scorer.", self.device)
        self.value = [get(f"value_head.{i}.{kind}") for i in (0, 2) for kind in ("weight", "bias")]
        self.kept: torch.Tensor | None = None

    def new_cache(self, capacity: int, max_len: int, dtype: torch.dtype = torch.float16) -> KVCache:
        return self.trunk.new_cache(capacity, max_len, dtype)

    def step_workspace_bytes(self, batch: int, steps: int) -> int:
        return self.trunk.step_workspace_bytes(batch, steps)

    def forward_ragged(self, tokens: torch.Tensor, positions: torch.Tensor, cache: KVCache,
                       readout_offsets: torch.Tensor, span: int | None = None, rows: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
        """Append a padded run per cache row 0..B-1 (or ``rows``); hidden at each readout [B, d]."""

        from .piquet import forward_ragged

        codes = tokens[..., CARD_START:]
        if self.precision == "bf16":
            with torch.autocast("cuda", dtype=torch.bfloat16):
                cards, summary = self.grid(codes)
        else:
            cards, summary = self.grid(codes)
        self.kept = cards
        return forward_ragged(self.trunk, self.lookup, tokens, positions, cache, readout_offsets, span=span,
                              rows=rows, summary=summary, workspace=workspace)

    def forward_prefill(self, tokens: torch.Tensor, cache: KVCache, rows: torch.Tensor | None) -> torch.Tensor:
        batch, steps, _ = tokens.shape
        positions = torch.zeros(batch, dtype=torch.int64, device=self.device)
        offsets = torch.full((batch,), steps - 1, dtype=torch.int64, device=self.device)
        return self.forward_ragged(tokens, positions, cache, offsets, span=steps, rows=rows)

    def pop_context(self) -> torch.Tensor | None:
        """The ledger cards [B, T, 52, ledger_width] of the last forward's tokens (model.py:387-389)."""

        cards, self.kept = self.kept, None
        return cards

    def policy_logits(self, hidden: torch.Tensor, head: str, features=None, tokens=None, context=None) -> torch.Tensor:
        """fp32 candidate logits [N, K] (model.py:391-399); ``features`` holds ``kind`` [N, K],
        ``cards`` and ``target`` [N, K, 13] (NO_CARD-padded) and, for draws, ``taken`` [N, K, 52]."""

        if features is None or (tokens is None and context is None):
            raise ValueError("Rummy policy heads score candidate lists at a readout token.")
        if head not in self.policy_heads:
            raise ValueError(f"Unknown rummy policy head {head!r}.")
        grid = self.grid.cards(tokens[..., CARD_START:]) if context is None else context
        return self.scorer(hidden, grid, features["kind"], features["cards"], features["target"],
                           features.get("taken"))

    def player_values(self, hidden: torch.Tensor) -> torch.Tensor:
        """value_head: Linear -> exact GELU -> Linear, fp32 [N, 4] (cardgym/nn/model.py:12-17)."""

        w0, b0, w2, b2 = self.value
        inner = torch.nn.functional.gelu(torch.nn.functional.linear(hidden.float(), w0, b0))
        return torch.nn.functional.linear(inner, w2, b2)


def synthetic_rummy_actor_state(config: RummyModelConfig, seed: int = 0) -> dict:
    """Seeded float32 weights under the reference ``RummyActor``'s parameter names and shapes
    (the heads it rolls out with; the belief heads are left out)."""

    from .piquet import synthetic_actor_parts, synthetic_grid_state

    trunk = config.trunk()
    d, s, w = config.d_model, config.score_dim, config.ledger_width
    state, normal, gain = synthetic_actor_parts(trunk, sum(FIELD_VOCAB), seed)
    synthetic_grid_state(state, normal, gain, d=d, codes=CARD_VOCAB, ranks=13, cards=NUM_CARDS, width=w,
                         hidden=config.ledger_hidden, blocks=config.ledger_layers, kernel=config.ledger_kernel)
    p = "scorer."
    state.update({p + "query.weight": normal(s, d), p + "query.bias": normal(s), p + "card.weight": normal(s, w),
                  p + "target.weight": normal(s, w), p + "taken.weight": normal(s, w),
                  p + "card_id.weight": normal(NUM_CARDS, s), p + "target_id.weight": normal(NUM_CARDS, s),
                  p + "taken_id.weight": normal(NUM_CARDS, s), p + "kind.weight": normal(7, s),
                  p + "size.weight": normal(MAX_MELD_CARDS + 1, s), p + "norm.weight": gain(s),
                  p + "norm.bias": normal(s), p + "hidden.weight": normal(s, s), p + "hidden.bias": normal(s),
                  p + "out.weight": normal(1, s), p + "out.bias": normal(1)})
    state.update({"value_head.0.weight": normal(d, d), "value_head.0.bias": normal(d),
                  "value_head.2.weight": normal(MAX_PLAYERS, d), "value_head.2.bias": normal(MAX_PLAYERS)})
    return state
