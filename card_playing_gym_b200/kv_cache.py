"""Device KV pool with the reference KVCache interface (cardgym/nn/kv_cache.py:19-138).

One stacked ``[n_layers, capacity, kv_heads, max_len, head_dim]`` tensor per K and V,
zero-filled (masked NaNs must not poison sums, kv_cache.py:42-44); ``k[layer]`` and
``v[layer]`` are views. Writes and row copies run as native kernels; ``read`` keeps
the reference's tensor-view semantics.
"""

from __future__ import annotations

import torch

from . import _native as nat


class KVCache:
    def __init__(
        self,
        *,
        n_layers: int,
        kv_heads: int,
        head_dim: int,
        capacity: int,
        max_len: int,
        device: torch.device | str,
        dtype: torch.dtype = torch.float32,
    ) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("card_playing_gym_b200.KVCache lives on a CUDA device")
        if dtype not in nat.DTYPE_CODES:
            raise ValueError(f"Unsupported KV dtype {dtype}.")
        self.n_layers = n_layers
        self.kv_heads = kv_heads
        self.head_dim = head_dim
        self.capacity = capacity
        self.max_len = max_len
        self.dtype = dtype
        self._row_shape = (kv_heads, max_len, head_dim)
        self.stacked = True
        self._base_k = torch.zeros((n_layers, capacity, *self._row_shape), device=self.device, dtype=dtype)
        self._base_v = torch.zeros_like(self._base_k)
        self.k = list(self._base_k.unbind(0))
        self.v = list(self._base_v.unbind(0))

    @staticmethod
    def bytes_per_row(n_layers: int, kv_heads: int, head_dim: int, max_len: int, dtype: torch.dtype) -> int:
        return n_layers * kv_heads * max_len * head_dim * 2 * dtype.itemsize

    @property
    def k_pool(self) -> torch.Tensor:
        return self._base_k

    @property
    def v_pool(self) -> torch.Tensor:
        return self._base_v

    def _write(self, layer: int, rows: torch.Tensor | None, positions: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        batch, _, steps, _ = k_new.shape
        if rows is None:
            rows = torch.arange(batch, device=self.device)
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
        if k_new.dtype not in nat.DTYPE_CODES or v_new.dtype != k_new.dtype:
            raise ValueError("k_new/v_new must share a float dtype")
        nat.call(
            "cg_kv_write_step", nat.ptr(self.k[layer]), nat.ptr(self.v[layer]), nat.DTYPE_CODES[self.dtype],
            self.capacity, self.kv_heads, self.max_len, self.head_dim, nat.ptr(rows.to(torch.int64).contiguous()),
            nat.ptr(positions.to(torch.int64).contiguous()), batch, steps, nat.ptr(k_new), nat.ptr(v_new),
            nat.DTYPE_CODES[k_new.dtype], nat.stream_handle(self.device),
        )

    def write_range(self, layer: int, rows: torch.Tensor | None, start: int, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Write [B, kv_heads, T, head_dim] at a shared offset; ``rows=None`` is 0..B-1 (kv_cache.py:65-82)."""

        batch, _, steps, _ = k_new.shape
        positions = (start + torch.arange(steps, device=self.device))[None, :].expand(batch, steps)
        self._write(layer, rows, positions, k_new, v_new)

    def write_step(self, layer: int, rows: torch.Tensor, positions: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Write K/V at a per-row offset: ``positions`` is [B] or [B, T] (kv_cache.py:84-105)."""

        steps = k_new.shape[2]
        if positions.dim() == 1:
            if steps != 1:
                raise ValueError("A [B] position vector writes exactly one position per row.")
            positions = positions[:, None]
        if positions.shape[1] != steps:
            raise ValueError("positions must carry one offset per written step.")
        self._write(layer, rows, positions, k_new, v_new)

    def read(self, layer: int, rows: torch.Tensor | None, length: int, count: int | None = None):
        """Cached K/V [B, kv_heads, length, head_dim]; ``rows=None`` is a zero-copy 0..count-1 view."""

        if rows is None:
            if count is None:
                raise ValueError("A dense read requires an explicit row count.")
            return self.k[layer][:count, :, :length], self.v[layer][:count, :, :length]
        return self.k[layer][rows, :, :length], self.v[layer][rows, :, :length]

    def copy_rows(self, sources: torch.Tensor, targets: torch.Tensor, length: int) -> None:
        """Copy the first ``length`` positions of ``sources`` rows onto ``targets`` (kv_cache.py:122-138)."""

        count = int(sources.shape[0])
        if count == 0 or length == 0:
            return
        code = nat.DTYPE_CODES[self.dtype]
        need = nat.query("cg_kv_copy_rows_workspace_bytes", self.n_layers, self.kv_heads, length, self.head_dim, code, count)
        workspace = nat.Workspace.get(self.device, need, "kv_copy")
        nat.call(
            "cg_kv_copy_rows", nat.ptr(self._base_k), nat.ptr(self._base_v), code, self.n_layers, self.capacity,
            self.kv_heads, self.max_len, self.head_dim, nat.ptr(sources.to(torch.int64).contiguous()),
            nat.ptr(targets.to(torch.int64).contiguous()), count, int(length), nat.ptr(workspace), workspace.numel(),
            nat.stream_handle(self.device),
        )
