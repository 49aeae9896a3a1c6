"""CUDA-graph replay of ticks (packed mixed ticks and uniform decode ticks).

A tick has a host half and a device half. The host half stays eager every tick:
page acquisition, the tick descriptor upload and the tick-pack kernel
(``PackedBatchCache.prepare_packed`` or ``PagedBatchCache.prepare``), which rewrite
the tick's metadata in place.
The device half is the same for every tick of one shape: the embedding gather, the
36 decoder layers (about ten launches each: projections, fused norm + RoPE + KV
append, attention, residual norms, SwiGLU) and the final norm + lm_head. It is
captured once per shape into a CUDA graph and replayed, which removes the gaps
between ~400 small launches that an eager tick pays.

What makes one graph serve many ticks: the cache runs in capacity mode, so its
metadata buffers and the attention launches are sized to work capacities (with
headroom) and the attention kernels read the tick's real work counts from the
device; the token ids are copied into the graph's own input buffer. A tick whose
shape or buffers differ from every captured graph (batch rows, token and logit
counts, split size, block-table width, capacities, reallocated buffers) gets a new
capture; the least recently used graphs beyond ``max_graphs`` are released.

The reference has no counterpart: its engine runs every tick eagerly
(src/helios/runtime/engine.py:406-530). Results are identical to the eager path.
"""

from __future__ import annotations

from collections import OrderedDict

import torch


class TickGraphs:
    def __init__(self, model, max_graphs: int = 4) -> None:
        self.model = model
        self.max_graphs = max_graphs
        self._graphs: OrderedDict[tuple, tuple] = OrderedDict()
        self._pool = None
        self.captures = 0
        self.replays = 0

    @staticmethod
    def _key(cache) -> tuple:
        ws = cache.workspace
        return (cache.batch_size, cache.total_tokens, int(cache.logit_rows.numel()), cache.split_keys,
                int(cache.block_table.shape[1]), cache.work_capacity, cache._i32.data_ptr(), cache._i64.data_ptr(),
                0 if ws is None else ws.data_ptr(), int(cache.logit_rows.data_ptr()))

    def run(self, ids: torch.Tensor, cache, *, greedy: bool = False) -> torch.Tensor:
        """Logits ``[logit rows, V]`` of a prepared tick (``greedy``: their argmax ids). The
        returned tensor is the graph's own output buffer: it holds this tick's result until
        the next replay of the same graph."""
        flat = ids.reshape(-1)
        if not cache.capacity_mode:
            # From the next prepare on, this cache lays out its buffers by capacity; this
            # tick (prepared without capacities) runs eagerly.
            cache.capacity_mode = True
            return self.model._packed_logits(flat, cache, greedy=greedy)
        key = self._key(cache) + (greedy,)
        entry = self._graphs.get(key)
        if entry is None:
            entry = self._capture(flat, cache, greedy)
            self._graphs[key] = entry
            while len(self._graphs) > self.max_graphs:
                self._graphs.popitem(last=False)
        else:
            self._graphs.move_to_end(key)
        graph, static_ids, logits = entry
        static_ids.copy_(flat)
        graph.replay()
        self.replays += 1
        return logits

    def _capture(self, flat: torch.Tensor, cache, greedy: bool) -> tuple:
        device = flat.device
        static_ids = flat.clone()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            # One eager pass first: library handles, kernel attributes and the caching
            # allocator's blocks are set up outside the capture. It writes the same K/V
            # rows the replay will write, so it changes nothing.
            self.model._packed_logits(static_ids, cache, greedy=greedy)
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(graph, pool=self._pool):
            logits = self.model._packed_logits(static_ids, cache, greedy=greedy)
        self.captures += 1
        return graph, static_ids, logits
