"""Steady-state streaming through one captured CUDA graph per cache layout.

Contract kept from the reference's StreamRunner (src/sinkcache/graphs.py:28-86): `step(ids)`
returns the logits of a [batch, q] token step; a one-token step on a steady cache is replayed
from a captured graph, everything else runs the model eagerly; a change of the cache's
layout (reallocated buffers, a different attention length) makes the next steady step
capture again; the cache's host-side counters, which no replay can move, are advanced after
each replay.

How it is built here.  The cache itself answers the three questions a replay depends on:
`is_steady` (is every further one-token step the same kernel sequence?),
`graph_signature()` (the pointers and sizes a captured step has baked in) and
`note_replayed_step()` (advance the counters a replay did not run).  A cache that counts
positions from the start of the stream rather than inside its buffer (SinkCacheV2:
`absolute_positions`) also gets the step's position ids from a static device tensor that is
refilled before each replay.  Every kernel of the sink-cache path takes its decisions on the
host before the step or reads them from device memory, so the graph never goes stale inside
one layout.

Each runner keeps at most one captured step (a layout change frees the old one) and warms
the model up once on a side stream before its first capture, so that libraries the model
calls finish their lazy set-up outside the capture.
"""

from __future__ import annotations

import torch

from . import _lib


class _CapturedStep:
    """One captured one-token step: the graph, the static tensors it reads (token ids,
    position ids) and writes (logits), and the cache layout it was captured against."""

    __slots__ = ("graph", "ids", "positions", "logits", "signature", "cache_kernels")

    def __init__(self, signature, ids: torch.Tensor, positions: torch.Tensor | None):
        self.graph = torch.cuda.CUDAGraph()
        self.signature = signature
        self.ids = ids
        self.positions = positions
        self.logits = None
        self.cache_kernels = 0  # the sink-cache library's kernels in the graph

    def run(self, ids: torch.Tensor, position: int) -> torch.Tensor:
        self.ids.copy_(ids)
        if self.positions is not None:
            self.positions.fill_(position)
        self.graph.replay()
        return self.logits


class StreamRunner:
    """Feeds a model token steps over a sink cache, replaying steady one-token steps from a
    CUDA graph.

        runner = StreamRunner(model, cache)
        logits = runner.step(ids)     # ids [batch, q]; logits [batch, q, vocab]

    A replayed step's logits tensor is overwritten by the next replay: consume it first.
    `replays` counts the steps served by a replay."""

    def __init__(self, model, cache, use_graph: bool = True):
        self.model, self.cache = model, cache
        self.use_graph = (bool(use_graph) and torch.cuda.is_available()
                          and callable(getattr(cache, "graph_signature", None)))
        self.replays = 0
        self._captured: _CapturedStep | None = None
        self._warmed = False

    @property
    def graph(self) -> torch.cuda.CUDAGraph | None:
        """The graph of the current layout, if one has been captured."""
        return None if self._captured is None else self._captured.graph

    @property
    def cache_kernels_per_replay(self) -> int | None:
        """How many of the sink-cache library's kernels one replay launches (counted by the
        library while the step was captured), if a step has been captured."""
        return None if self._captured is None else self._captured.cache_kernels

    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        if not (self.use_graph and ids.shape[-1] == 1 and self.cache.is_steady):
            return self.model(ids, past_key_values=self.cache, use_cache=True).logits
        signature = self.cache.graph_signature()
        captured = self._captured
        if captured is None or captured.signature != signature:
            self._captured = None  # free the old layout's graph before capturing the new one
            return self._capture_and_run(ids, signature)
        logits = captured.run(ids, self.cache.tokens_seen)
        self.cache.note_replayed_step()
        self.replays += 1
        return logits

    def _warm_up(self, ids: torch.Tensor) -> None:
        """One forward without the cache on a side stream (the cache is left untouched)."""
        side = torch.cuda.Stream(device=ids.device)
        side.wait_stream(torch.cuda.current_stream(ids.device))
        with torch.cuda.stream(side):
            self.model(ids, use_cache=False)
        torch.cuda.current_stream(ids.device).wait_stream(side)
        torch.cuda.synchronize(ids.device)
        self._warmed = True

    def _capture_and_run(self, ids: torch.Tensor, signature) -> torch.Tensor:
        """Capture this step and run it.  The capture executes the step's host code (the
        cache's counters advance once, as in an eager step) but none of its kernels; the
        replay that follows runs them."""
        if not self._warmed:
            self._warm_up(ids)
        positions = None
        kwargs = {}
        if getattr(self.cache, "absolute_positions", False):
            positions = torch.full((ids.shape[0], 1), self.cache.tokens_seen, dtype=torch.long, device=ids.device)
            kwargs["position_ids"] = positions
        captured = _CapturedStep(signature, ids.clone(), positions)
        torch.cuda.synchronize(ids.device)
        launched = _lib.launch_count()
        with torch.cuda.graph(captured.graph):
            captured.logits = self.model(captured.ids, past_key_values=self.cache, use_cache=True, **kwargs).logits
        captured.cache_kernels = _lib.launch_count() - launched
        captured.graph.replay()
        self._captured = captured
        return captured.logits
