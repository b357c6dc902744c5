"""One-token streaming with a CUDA graph for the steady state (src/sinkcache/graphs.py:1-86).

SinkCache (v1): once full, every decode step is the same computation -- same shapes, same
position (n_sink + window), same buffers, drop == 1.  One captured step (every kernel of
the model forward including the sink-cache kernels, which take no host-side decisions
inside a step) is replayed for every later token.

SinkCacheV2: shapes and buffers are fixed too, but the position grows.  The ring slot and
the region rotation come from a device-side position inside each layer (read and advanced
by the place kernel), and position_ids are fed from a static device tensor, so one captured
step still serves every later token.  A step that moves a pinned token into the region
runs eagerly, and a change of region size (attention length) triggers a recapture.

Python-side counters do not advance inside a replay, so the runner advances them.
"""

import torch

from .cache import SinkCache
from .cache_v2 import SinkCacheV2


class StreamRunner:
    def __init__(self, model, cache, use_graph: bool = True):
        self.model, self.cache = model, cache
        self.v2 = isinstance(cache, SinkCacheV2)
        self.use_graph = use_graph and isinstance(cache, (SinkCache, SinkCacheV2)) and torch.cuda.is_available()
        self.graph = None
        self.static_ids = self.static_logits = self.static_pos = None
        self._key = None
        self.replays = 0
        self._warmed = False

    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """Feed ids [batch, q]; returns logits [batch, q, vocab].  One-token steps on a steady
        cache are graph-replayed; anything else runs eagerly (and may reallocate the cache or
        resize the region, which invalidates the graph: it is then recaptured).  When graphed,
        the returned tensor is overwritten by the next step: consume it first."""
        one = ids.shape[-1] == 1
        if self.graph is not None and self._layout() != self._key:
            self.graph = None
        if self.graph is not None and one and self.cache.is_steady:
            self.static_ids.copy_(ids)
            if self.v2:
                self.static_pos.fill_(self.cache.tokens_seen)
            self.graph.replay()
            self._advance()
            self.replays += 1
            return self.static_logits
        if self.use_graph and one and self.cache.is_steady:
            self._capture(ids)
            self.graph.replay()  # capture records but does not execute: run this step now
            return self.static_logits
        return self.model(ids, past_key_values=self.cache, use_cache=True).logits

    def _advance(self):
        if self.v2:
            self.cache.advance_after_replay()
            return
        for layer in self.cache.layers:
            layer.tokens_seen += 1
            layer.tokens_evicted += 1

    def _layout(self):
        ws = self.cache.workspace.buf
        return ([(l._kbuf.data_ptr(), l._vbuf.data_ptr()) for l in self.cache.layers],
                ws.data_ptr() if ws is not None else None,
                self.cache.layout_key() if self.v2 else None)

    def _capture(self, ids):
        if not self._warmed:
            # Libraries the model calls set themselves up on first use (cuBLAS handles,
            # lazily loaded kernels), which cannot happen inside a capture.  A v2 cache is
            # steady right after its fill, so the first step may be a capture: run one
            # forward without the cache first (it leaves the cache untouched).
            self.model(ids, use_cache=False)
            torch.cuda.synchronize()
            self._warmed = True
        self._key = self._layout()
        self.static_ids = ids.clone()
        kwargs = {}
        if self.v2:
            self.static_pos = torch.full((ids.shape[0], 1), self.cache.tokens_seen, dtype=torch.long,
                                         device=ids.device)
            kwargs["position_ids"] = self.static_pos
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(self.graph):
            self.static_logits = self.model(self.static_ids, past_key_values=self.cache, use_cache=True,
                                            **kwargs).logits
