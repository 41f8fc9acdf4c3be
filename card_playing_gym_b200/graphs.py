"""CUDA graphs of a rollout decode wave: one replay per wave shape.

Reference: cardgym/rl/graphs.py:66-151 (``DecodeGraphs``). For each wave shape (rows, tokens
per row, token width, attention span) the whole wave — the field lookup and ragged trunk
decode into the KV cache, every policy head's logits at each row's readout and, with
``values``, the per-seat values — is captured once and replayed with one launch. The output
is one fp32 [rows, columns] device tensor (``columns`` names each head's slice), valid until
the next ``run``. A model with ``pop_context`` (piquet's card grid) hands each head the
context of its row's readout token, as graphs.py:88-95 does.

The step's scratch memory belongs to this object: captured graphs hold its address, so when
a larger shape needs more, the buffer is replaced and every earlier graph is dropped (and
recaptured on its next use). The KV cache and the weights must keep their storage.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class _Graph:
    graph: torch.cuda.CUDAGraph
    inputs: torch.Tensor  # int64 [rows * run * width + 3 * rows]: tokens, positions, offsets, cache rows
    output: torch.Tensor  # fp32 [rows, columns]


class DecodeGraphs:
    def __init__(self, model, cache, *, precision: str | None = None, values: bool = True) -> None:
        if precision is not None and precision != model.precision:
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.cache = cache
        self.values = values
        self.heads: tuple[str, ...] = tuple(model.policy_heads)
        self.pool = torch.cuda.graph_pool_handle()
        self._graphs: dict[tuple[int, int, int, int], _Graph] = {}
        self._workspace: torch.Tensor | None = None
        self.columns: dict[str, slice] = {}

    def __len__(self) -> int:
        return len(self._graphs)

    def _body(self, inputs: torch.Tensor, rows: int, run: int, width: int, span: int) -> torch.Tensor:
        cells = rows * run * width
        tokens = inputs[:cells].view(rows, run, width)
        positions, offsets, cache_rows = inputs[cells:].view(3, rows)
        hidden = self.model.forward_ragged(tokens, positions, self.cache, offsets, span=span, rows=cache_rows,
                                           workspace=self._workspace)
        # Pointer heads (piquet's card scorers) read the readout token's grid cards.
        pop = getattr(self.model, "pop_context", None)
        context = pop() if pop is not None else None
        if context is not None:
            context = context[torch.arange(rows, device=inputs.device), offsets]
        outputs = [self.model.policy_logits(hidden, head, None, None, context) for head in self.heads]
        if self.values:
            outputs.append(self.model.player_values(hidden))
        if not self.columns:
            names = [*self.heads, "values"] if self.values else list(self.heads)
            start = 0
            for name, output in zip(names, outputs):
                self.columns[name] = slice(start, start + output.shape[-1])
                start += output.shape[-1]
        return torch.cat([output.float() for output in outputs], dim=-1)

    def run(self, tokens: np.ndarray, positions: np.ndarray, offsets: np.ndarray, cache_rows: np.ndarray,
            span: int) -> torch.Tensor:
        """Decode one wave; returns the device output [rows, columns] (copy it before the next run)."""

        rows, run, width = tokens.shape
        span = min(span, self.cache.max_len)
        key = (rows, run, width, span)
        host = torch.from_numpy(
            np.concatenate([tokens.reshape(-1), positions, offsets, cache_rows]).astype(np.int64, copy=False)
        ).pin_memory()
        need = self.model.step_workspace_bytes(rows, run)
        if self._workspace is None or self._workspace.numel() < need:
            self._graphs.clear()  # they hold the old scratch buffer's address
            self._workspace = torch.empty(need, dtype=torch.uint8, device=self.cache.device)
        entry = self._graphs.get(key)
        if entry is None:
            return self._capture(key, host)
        entry.inputs.copy_(host, non_blocking=True)
        entry.graph.replay()
        return entry.output

    def _capture(self, key: tuple[int, int, int, int], host: torch.Tensor) -> torch.Tensor:
        rows, run, width, span = key
        inputs = torch.empty(host.shape, dtype=host.dtype, device=self.cache.device)
        inputs.copy_(host, non_blocking=True)
        # A warm-up run of the same wave (it writes the same K/V the replay writes again)
        # configures every kernel before the capture.
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._body(inputs, rows, run, width, span)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self.pool):
            output = self._body(inputs, rows, run, width, span)
        self._graphs[key] = _Graph(graph, inputs, output)
        graph.replay()
        return output
