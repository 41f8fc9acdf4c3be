"""The decoder trunk on the B200: a device weight blob and the reference Trunk's decode entry points.

``B200Trunk`` mirrors the reference ``Trunk`` (cardgym/nn/trunk.py:259-429) for the
rollout path: ``condition(x, ple_lookup, value_lookup)`` (285-312) and
``forward_ragged(x, ple, values, cache, positions, readout_offsets, span, rows)``
(391-429). Weights come from a reference-named state dict (``trunk.*`` keys); they
are packed once into one device blob (fp32 master copies + bf16 tensor-core copies).

Precision ``"fp32"`` runs every GEMM in fp32 on CUDA cores (the strict-parity mode);
``"bf16"`` feeds bf16 operands to the GEMMs with fp32 accumulation, keeps the
residual stream, norms, softmax and GELU in fp32, and is the rollout mode.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import _native as nat
from .config import TrunkConfig
from .kv_cache import KVCache


def trunk_dims(config: TrunkConfig) -> nat.TrunkDims:
    mask = 0
    for layer in config.value_layers:
        mask |= 1 << layer
    return nat.TrunkDims(
        d_model=config.d_model, n_layers=config.n_layers, n_heads=config.n_heads, n_kv_heads=config.n_kv_heads,
        d_ff=config.d_ff, per_layer_dim=config.per_layer_dim, input_norm=1 if config.input_norm else 0,
        reserved=0, value_layers=mask,
    )


def _as_numpy(value) -> np.ndarray:
    if isinstance(value, torch.Tensor):
        return value.detach().to("cpu", torch.float32).numpy()
    return np.asarray(value, dtype=np.float32)


_PARTS = {
    nat.CG_PART_LN_ATTN_W: "ln_attn.weight", nat.CG_PART_LN_ATTN_B: "ln_attn.bias",
    nat.CG_PART_QKV: "qkv_proj.weight", nat.CG_PART_OUT: "out_proj.weight",
    nat.CG_PART_LN_MLP_W: "ln_mlp.weight", nat.CG_PART_LN_MLP_B: "ln_mlp.bias",
    nat.CG_PART_UP: "mlp.0.weight", nat.CG_PART_UP_B: "mlp.0.bias",
    nat.CG_PART_DOWN: "mlp.2.weight", nat.CG_PART_DOWN_B: "mlp.2.bias",
}


def build_blob(config: TrunkConfig, state: dict, device: torch.device, prefix: str = "trunk.") -> torch.Tensor:
    """Pack ``trunk.*`` parameters into the native weight blob on ``device``."""

    config.validate()
    dims = trunk_dims(config)
    total = nat.query("cg_trunk_blob_bytes", dims)
    host = np.zeros(total, dtype=np.uint8)

    def put(which: int, layer: int, name: str) -> None:
        offset = nat.lib().cg_trunk_part_offset(dims, which, layer)
        if offset < 0:
            return
        array = np.ascontiguousarray(_as_numpy(state[prefix + name]).reshape(-1))
        host[offset : offset + array.nbytes] = array.view(np.uint8)

    if config.input_norm:
        put(nat.CG_PART_INPUT_NORM, 0, "input_norm.weight")
    if config.per_layer_dim:
        put(nat.CG_PART_PLE_CONTEXT, 0, "ple_context.weight")
    put(nat.CG_PART_FINAL_W, 0, "final_norm.weight")
    put(nat.CG_PART_FINAL_B, 0, "final_norm.bias")
    for layer in range(config.n_layers):
        for which, name in _PARTS.items():
            put(which, layer, f"blocks.{layer}.{name}")
    blob = torch.from_numpy(host).to(device)
    with torch.cuda.device(device):
        nat.call("cg_trunk_prepare", dims, nat.ptr(blob), nat.stream_handle(device))
    return blob


class B200Trunk:
    """Reference ``Trunk`` decode path over a packed device blob."""

    def __init__(self, config: TrunkConfig, state: dict, device: torch.device | str = "cuda", precision: str = "bf16") -> None:
        if precision not in nat.PRECISIONS:
            raise ValueError(f"precision must be one of {sorted(nat.PRECISIONS)}")
        self.config = config
        self.device = torch.device(device)
        self.precision = precision
        self.dims = trunk_dims(config)
        self.blob = build_blob(config, state, self.device)

    @property
    def lookup_width(self) -> int:
        c = self.config
        return c.d_model + c.ple_width + c.value_width

    def new_cache(self, capacity: int, max_len: int, dtype: torch.dtype = torch.float16) -> KVCache:
        c = self.config
        return KVCache(n_layers=c.n_layers, kv_heads=c.n_kv_heads, head_dim=c.head_dim, capacity=capacity,
                       max_len=max_len, device=self.device, dtype=dtype)

    def condition_lookup(self, lookup: torch.Tensor):
        """Trunk.condition on the packed lookup [..., d | ple | value] (trunk.py:285-312)."""

        c = self.config
        lead = lookup.shape[:-1]
        flat = lookup.reshape(-1, lookup.shape[-1]).float().contiguous()
        n = flat.shape[0]
        x = torch.empty((n, c.d_model), device=self.device)
        ple = torch.empty((n, c.ple_width), device=self.device) if c.ple_width else None
        values = torch.empty((n, c.value_width), device=self.device) if c.value_width else None
        nat.call("cg_trunk_condition", self.dims, nat.ptr(self.blob), nat.ptr(flat), n, nat.ptr(x), nat.ptr(ple),
                 nat.ptr(values), nat.PRECISIONS[self.precision], nat.stream_handle(self.device))
        x = x.view(*lead, c.d_model)
        if ple is not None:
            ple = ple.view(*lead, c.n_layers, c.per_layer_dim)
        if values is not None:
            values = values.view(*lead, len(c.value_layers), c.kv_width)
        return x, ple, values

    def condition(self, x: torch.Tensor, ple_lookup: torch.Tensor | None, value_lookup: torch.Tensor | None):
        parts = [x.float()]
        if self.config.ple_width:
            if ple_lookup is None:
                raise ValueError("This trunk expects a per-layer embedding lookup.")
            parts.append(ple_lookup.float())
        if self.config.value_width:
            if value_lookup is None:
                raise ValueError("This trunk expects a value-embedding lookup.")
            parts.append(value_lookup.float())
        return self.condition_lookup(torch.cat(parts, dim=-1))

    def forward_ragged(
        self,
        x: torch.Tensor,
        ple: torch.Tensor | None,
        values: torch.Tensor | None,
        cache: KVCache,
        positions: torch.Tensor,
        readout_offsets: torch.Tensor,
        span: int | None = None,
        rows: torch.Tensor | None = None,
        workspace: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Append a padded run of tokens per row; final-norm hidden at each readout [B, d] (trunk.py:391-429).

        ``workspace`` (uint8, at least ``step_workspace_bytes``) pins the step's scratch memory,
        for callers that capture the step in a CUDA graph; by default a shared buffer is used.
        """

        batch, steps, _ = x.shape
        if span is None:
            span = int(positions.max()) + steps
        span = min(span, cache.max_len)
        x = x.float().contiguous()
        workspace = self.workspace(batch, steps, workspace)
        hidden = torch.empty((batch, self.config.d_model), device=self.device)
        nat.call(
            "cg_trunk_forward_ragged", self.dims, nat.ptr(self.blob), nat.ptr(x),
            nat.ptr(None if ple is None else ple.float().contiguous()),
            nat.ptr(None if values is None else values.float().contiguous()), batch, steps,
            nat.ptr(positions.to(torch.int64).contiguous()), nat.ptr(readout_offsets.to(torch.int64).contiguous()),
            nat.ptr(None if rows is None else rows.to(torch.int64).contiguous()), int(span), nat.ptr(cache.k_pool),
            nat.ptr(cache.v_pool), nat.DTYPE_CODES[cache.dtype], cache.capacity, cache.max_len,
            nat.PRECISIONS[self.precision], nat.ptr(workspace), workspace.numel(), nat.ptr(hidden),
            nat.stream_handle(self.device),
        )
        return hidden

    def step_workspace_bytes(self, batch: int, steps: int) -> int:
        return nat.query("cg_trunk_step_workspace_bytes", self.dims, batch, steps, nat.PRECISIONS[self.precision])

    def workspace(self, batch: int, steps: int, given: torch.Tensor | None = None) -> torch.Tensor:
        """The caller's scratch buffer (checked for size) or the shared one."""

        need = self.step_workspace_bytes(batch, steps)
        if given is None:
            return nat.Workspace.get(self.device, need)
        if given.numel() < need:
            raise ValueError(f"workspace of {given.numel()} bytes < {need} needed")
        return given

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.config.head_dim)
