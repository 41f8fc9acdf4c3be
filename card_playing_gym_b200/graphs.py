"""CUDA graphs of a rollout decode wave, upload included: one graph launch per wave.

Drop-in for ``DecodeGraphs`` (cardgym/rl/graphs.py:66-151): ``DecodeGraphs(model, cache,
precision=, values=).run(tokens, positions, offsets, cache_rows, span)`` returns one fp32
[rows, columns] device tensor holding, for every row, each policy head's logits at the row's
readout and (with ``values``) the per-seat values; ``columns`` names each head's slice. A model
with ``pop_context`` (piquet's card grid) hands every head the context of its row's readout
token, as the reference's graphed body does (graphs.py:88-95).

Each wave shape (rows, tokens per row, token width, span) gets one ``_Replay``: a pinned host
staging buffer, its device twin, the graph and the graph's output. The graph starts with the
copy of the staging buffer to the device, so a wave is: write the packed inputs into the
staging buffer, launch the graph. Before the buffer is written again, the event recorded after
the previous launch of that shape is waited on, so an upload still reading it is never
overwritten. The output stays valid until the next ``run`` of the same shape.

The trunk's step scratch belongs to this object: graphs hold its address, so when a larger
shape needs more, every graph is dropped (and recaptured on its next use) before the buffer is
replaced. The KV cache and the weights must keep their storage.
"""

from __future__ import annotations

import numpy as np
import torch


class _Replay:
    """One captured wave shape."""

    def __init__(self, host: torch.Tensor, device_inputs: torch.Tensor) -> None:
        self.host = host  # pinned int64 [rows * run * width + 3 * rows]
        self.view = host.numpy()
        self.device_inputs = device_inputs
        self.graph: torch.cuda.CUDAGraph | None = None
        self.output: torch.Tensor | None = None
        self.done = torch.cuda.Event()


class DecodeGraphs:
    def __init__(self, model, cache, *, precision: str | None = None, values: bool = True) -> None:
        if precision is not None and precision != model.precision:
            raise ValueError(f"the model runs in {model.precision}, not {precision}")
        self.model = model
        self.cache = cache
        self.values = values
        self.heads: tuple[str, ...] = tuple(model.policy_heads)
        self.columns: dict[str, slice] = {}
        self._replays: dict[tuple[int, int, int, int], _Replay] = {}
        self._scratch: torch.Tensor | None = None
        self._pool = torch.cuda.graph_pool_handle()

    def __len__(self) -> int:
        return len(self._replays)

    def run(self, tokens: np.ndarray, positions: np.ndarray, offsets: np.ndarray, cache_rows: np.ndarray,
            span: int) -> torch.Tensor:
        """Decode one wave; returns the device output [rows, columns] (read it before this shape runs again)."""

        rows, run, width = tokens.shape
        key = (rows, run, width, min(span, self.cache.max_len))
        self._fit_scratch(rows, run)
        replay = self._replays.get(key)
        fresh = replay is None
        if fresh:
            cells = rows * run * width + 3 * rows
            replay = _Replay(torch.empty(cells, dtype=torch.int64, pin_memory=True),
                             torch.empty(cells, dtype=torch.int64, device=self.cache.device))
            self._replays[key] = replay
        else:
            replay.done.synchronize()  # the last upload from this buffer has been read
        cells = rows * run * width
        view = replay.view
        view[:cells] = tokens.reshape(-1)
        view[cells:cells + rows] = positions
        view[cells + rows:cells + 2 * rows] = offsets
        view[cells + 2 * rows:] = cache_rows
        if fresh:
            self._capture(replay, key)
        replay.graph.replay()
        replay.done.record()
        return replay.output

    # ------------------------------------------------------------------------------------------------
    def _fit_scratch(self, rows: int, run: int) -> None:
        need = self.model.step_workspace_bytes(rows, run)
        if self._scratch is not None and self._scratch.numel() >= need:
            return
        self._replays.clear()  # every graph holds the old buffer's address
        self._scratch = None
        self._scratch = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=self.cache.device)

    def _wave(self, replay: _Replay, key) -> torch.Tensor:
        rows, run, width, span = key
        replay.device_inputs.copy_(replay.host, non_blocking=True)
        cells = rows * run * width
        tokens = replay.device_inputs[:cells].view(rows, run, width)
        positions, offsets, cache_rows = replay.device_inputs[cells:].view(3, rows)
        hidden = self.model.forward_ragged(tokens, positions, self.cache, offsets, span=span, rows=cache_rows,
                                           workspace=self._scratch)
        pop = getattr(self.model, "pop_context", None)
        context = pop() if pop is not None else None
        if context is not None:
            context = context[torch.arange(rows, device=hidden.device), offsets]
        outputs = [self.model.policy_logits(hidden, head, None, None, context).float() for head in self.heads]
        if self.values:
            outputs.append(self.model.player_values(hidden).float())
        if not self.columns:
            names = [*self.heads, "values"] if self.values else list(self.heads)
            ends = np.cumsum([output.shape[-1] for output in outputs])
            self.columns = {name: slice(int(end - output.shape[-1]), int(end))
                            for name, output, end in zip(names, outputs, ends)}
        return torch.cat(outputs, dim=-1)

    def _capture(self, replay: _Replay, key) -> None:
        """A warm-up wave on a side stream (it configures every kernel and writes the K/V the graph writes
        again), then the capture."""

        stream = torch.cuda.current_stream(self.cache.device)
        side = torch.cuda.Stream(self.cache.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            self._wave(replay, key)
        stream.wait_stream(side)
        replay.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(replay.graph, pool=self._pool):
            replay.output = self._wave(replay, key)
