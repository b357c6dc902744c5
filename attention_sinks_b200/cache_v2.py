"""Ring-buffer attention-sink cache ("v2"): the sinks move forward, the window stays put
(the algorithm of src/sinkcache/cache_v2.py:1-50).

RoPE attention depends only on relative position.  So instead of re-rotating every window
key each step (v1), window keys keep the rotation the model gave them at their absolute
positions, the query sits at its absolute position t, and only the few *region* tokens --
the sinks, plus pinned tokens that have left the window -- are rotated, from their stored
original keys and with fp64 angles, to sit just before the window.  Keys are stored in the
model dtype: a window key is never rounded again.

Layout of one layer (what the kernels read): K and V buffers of `ring + region_cap` rows,
ring = window + 1.  The token at absolute position p >= n_sink lives in ring slot
(p - n_sink) mod ring; the region's rows follow the ring (rotated keys in K, values in V),
in region order: sinks first, then pinned tokens in the order they left the window.  The
region's original keys sit in a separate buffer with their positions on the device.

Host state is small: the next position `t`, the region's positions, how far pins have been
looked for (`moved_upto`) and how many the pin budget dropped.  The device keeps the
position too ({t, arrival counter}), read and advanced by the steady-step kernel, so one
captured CUDA graph serves every later steady token.

Device work goes through the sm_100a library: the steady one-token step is sink_v2_place
(or, when the model uses the registered attention backend, sink_v2_decode_step: the same
step fused with its attention); chunk steps and kept() rotate the region with
sink_v2_place into a fresh tensor and gather the window out of the ring, in position order,
with sink_v2_gather (one launch, 16-byte copies).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _lib
from .cache import _BY_BUFFER, find_inv_freq, uses_sink_attention


def _pins_between(pinned, lo: int, hi: int) -> list[int]:
    """Pinned positions p with lo <= p < hi, ascending.  Probes the range when it is shorter
    than the pin set (a steady step asks about one position), else filters the set."""
    if hi <= lo or not pinned:
        return []
    if hi - lo <= len(pinned):
        return [p for p in range(lo, hi) if p in pinned]
    return sorted(p for p in pinned if lo <= p < hi)


class _Region:
    """The rows placed just before the window.

    Entry j has an original key (`keys[:, :, j]`, at the rotation of its own position
    `positions[j]`, mirrored on the device in `pos_dev[j]`) and a value (`values[:, :, j]`,
    a view into the layer's V buffer right after the ring, where attention reads it).
    Entries 0..n_sink-1 are the sinks; after them come pins.  When the region is full, a
    new pin pushes out the oldest pin (entry n_sink) and the pins after it move up a row;
    with no pin budget a full region is an error."""

    def __init__(self, n_sink: int, max_pinned: int):
        self.n_sink, self.max_pinned = n_sink, max_pinned
        self.capacity = n_sink + max_pinned
        self.positions: list[int] = []
        self.dropped = 0
        self.keys = self.values = self.pos_dev = None

    def bind(self, keys: torch.Tensor, values: torch.Tensor, pos_dev: torch.Tensor) -> None:
        self.keys, self.values, self.pos_dev = keys, values, pos_dev

    def __len__(self) -> int:
        return len(self.positions)

    def add(self, k_row: torch.Tensor, v_row: torch.Tensor, position: int) -> None:
        """k_row, v_row: [b, h, 1, d]; the key at the rotation of `position`."""
        if len(self.positions) >= self.capacity:
            if self.max_pinned == 0:
                raise RuntimeError("region full")
            self._drop_oldest_pin()
        j = len(self.positions)
        self.keys[:, :, j:j + 1].copy_(k_row)
        self.values[:, :, j:j + 1].copy_(v_row)
        self.pos_dev[j] = position
        self.positions.append(position)

    def _drop_oldest_pin(self) -> None:
        first, n = self.n_sink, len(self.positions)
        for rows in (self.keys, self.values, self.pos_dev.view(1, 1, -1, 1)):
            rows[:, :, first:n - 1] = rows[:, :, first + 1:n].clone()  # overlapping move: copy first
        del self.positions[first]
        self.dropped += 1


@dataclass
class _LayerState:
    """Everything restore() writes back into a layer (device copies plus host counters)."""
    k: torch.Tensor
    v: torch.Tensor
    region_keys: torch.Tensor
    region_pos: torch.Tensor
    t: int
    positions: list[int]
    moved_upto: int


@dataclass
class V2Snapshot:
    """SinkCacheV2.snapshot(): per-layer states and the pinned positions."""
    layers: list[_LayerState]
    pinned: frozenset


class SinkLayerV2(CacheLayerMixin):
    """One layer of the ring-buffer cache (the interface of src/sinkcache/cache_v2.py:59-248)."""

    is_sliding = False
    is_croppable = False

    def __init__(self, n_sink: int, window: int, inv_freq: torch.Tensor, max_pinned: int = 0,
                 pinned: set[int] | None = None, fused: bool = False,
                 workspace: "_lib.Workspace | None" = None):
        super().__init__()
        if n_sink < 0 or window < 1 or max_pinned < 0:
            raise ValueError(f"need n_sink >= 0, window >= 1, max_pinned >= 0; got {n_sink}, {window}, {max_pinned}")
        self.n_sink, self.window, self.max_pinned = n_sink, window, max_pinned
        self.ring = window + 1
        self.region_cap = n_sink + max_pinned
        self.inv_freq = inv_freq
        self.pinned = pinned if pinned is not None else set()  # shared with the cache's pin()
        self.t = 0               # absolute position of the next token (= tokens seen)
        self.moved_upto = 0      # pins below this position have been looked for
        self.fused = fused
        self._region = _Region(n_sink, max_pinned)
        self._kbuf = self._vbuf = None
        self._pending = None     # (k, v, region size) of a deferred steady step
        self._ws = workspace if workspace is not None else _lib.Workspace()

    @property
    def region_pos(self) -> list[int]:
        """Original positions of the region entries (sinks, then pins)."""
        return self._region.positions

    @property
    def pins_dropped(self) -> int:
        return self._region.dropped

    # ------------------------------------------------------------------ storage

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        _lib.check_device(self.device)
        _lib.prepare_device(self.device)  # before any graph capture of this layer's steps
        b, h, _, d = key_states.shape
        if 2 * self.inv_freq.numel() > d:
            raise ValueError(f"rotary dims {2 * self.inv_freq.numel()} exceed head_dim {d}")
        rows = self.ring + self.region_cap
        self._kbuf = torch.zeros(b, h, rows, d, dtype=self.dtype, device=self.device)
        self._vbuf = torch.zeros(b, h, rows, d, dtype=self.dtype, device=self.device)
        cap = max(self.region_cap, 1)
        self._reg_k = torch.zeros(b, h, cap, d, dtype=self.dtype, device=self.device)
        self._reg_pos = torch.zeros(cap, dtype=torch.long, device=self.device)
        self._region.bind(self._reg_k, self._vbuf[:, :, self.ring:], self._reg_pos)
        # {t, arrival counter}: the steady-step kernel reads t and advances it
        self._position = torch.zeros(2, dtype=torch.long, device=self.device)
        self._t_dev = self._position[0]
        self.inv_freq = self.inv_freq.to(self.device, torch.float64).contiguous()
        _BY_BUFFER[self._kbuf.data_ptr()] = self
        self._size_workspace(b, h, d)
        self.is_initialized = True

    def _size_workspace(self, b, h, d):
        """Workspace for the fused steady step at every region size (a captured step keeps
        the pointer, so it must not grow later).  The size only changes with the number of
        pipeline chunks, so one query per 8 rows covers every region size."""
        sms = _lib.sm_count(self.device)
        need = 256
        for R in list(range(0, self.region_cap + 1, 8)) + [self.region_cap]:
            need = max(need, _lib.workspace_bytes(_lib.OP_ATTEND, b, h, h * 8, d, self.dtype, self.dtype,
                                                  self.ring + R, 0, 1, 0, sms))
        self._ws.get(need, self.device)

    # ------------------------------------------------------------------ positions

    def _window_start(self, t: int) -> int:
        """First window position when the next token is t (positions below n_sink count as
        sinks, not window)."""
        return max(min(t, self.n_sink), t - self.window)

    def _window_span(self, t: int) -> tuple[int, int]:
        """Window positions [lo, hi) held in the ring when the next token is t (empty while
        t <= n_sink)."""
        return max(self._window_start(t), self.n_sink), t

    def _ring_views(self, buf: torch.Tensor, lo: int, hi: int) -> list[torch.Tensor]:
        """Ring rows of positions [lo, hi) (all >= n_sink, at most a ring's worth) in position
        order: one contiguous view, or two when the span wraps around the ring's end."""
        n = hi - lo
        if n <= 0:
            return []
        s = (lo - self.n_sink) % self.ring
        head = min(n, self.ring - s)
        views = [buf[:, :, s:s + head]]
        if head < n:
            views.append(buf[:, :, :n - head])
        return views

    def _logical(self, t: int, chunk: tuple[torch.Tensor, torch.Tensor] | None = None):
        """(keys, values) of [region rotated to sit before the window, window by position,
        chunk] for a query at position t: the window rows and the region's values gathered by
        one kernel launch (16-byte copies from the ring slots), the region's keys rotated
        straight into the new tensor's first rows by the place kernel."""
        R = len(self._region)
        lo, hi = self._window_span(t)
        n = chunk[0].shape[-2] if chunk is not None else 0
        b, h, _, d = self._kbuf.shape
        rows = R + max(0, hi - lo) + n
        keys = torch.empty(b, h, rows, d, dtype=self.dtype, device=self.device)
        values = torch.empty(b, h, rows, d, dtype=self.dtype, device=self.device)
        if R:
            _lib.v2_place(self._kbuf, self._vbuf, None, None, self._reg_k, self._reg_pos, R, keys[:, :, :R], None,
                          t, self.n_sink, self.window, self.inv_freq)
        k_new, v_new = chunk if chunk is not None else (None, None)
        if n and (not self._gatherable(k_new) or not self._gatherable(v_new)):
            k_new, v_new = k_new.contiguous(), v_new.contiguous()
        _lib.v2_gather(self._kbuf, self._vbuf, self.n_sink, self.window, R, lo, hi, k_new if n else None,
                       v_new if n else None, keys, values)
        return keys, values

    @staticmethod
    def _gatherable(x: torch.Tensor) -> bool:
        """Rows the gather kernel reads with 16-byte copies: unit last stride, 16-byte aligned."""
        es = x.element_size()
        return (x.stride(-1) == 1 and x.data_ptr() % 16 == 0
                and all((st * es) % 16 == 0 for st in x.stride()[:-1]))

    # ------------------------------------------------------------------ pins

    def next_step_moves_pin(self) -> bool:
        """Would a one-token step at the current position move a pin into the region?"""
        p = self.t - self.window
        return p >= self.n_sink and p in self.pinned

    def _pins_leave(self, bound: int, chunk=None) -> None:
        """Pins below `bound` have left the window: each joins the region, its rows taken
        from its ring slot or, for a position of the chunk being stored (chunk = (k, v,
        first position)), from the chunk."""
        if bound <= self.moved_upto:
            return
        for p in _pins_between(self.pinned, max(self.moved_upto, self.n_sink), bound):
            if chunk is not None and p >= chunk[2]:
                i = p - chunk[2]
                self._region.add(chunk[0][:, :, i:i + 1], chunk[1][:, :, i:i + 1], p)
            else:
                s = (p - self.n_sink) % self.ring
                self._region.add(self._kbuf[:, :, s:s + 1], self._vbuf[:, :, s:s + 1], p)
        self.moved_upto = bound

    # ------------------------------------------------------------------ cache API

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.materialize()
        if key_states.shape[-2] == 1 and self.t >= self.n_sink + self.window:
            return self._steady_step(key_states, value_states)
        return self._chunk_step(key_states, value_states)

    def _steady_step(self, k, v):
        """A one-token step on a full window: the token overwrites the ring slot of the one
        that left the window last step, and the region is re-placed before the new window --
        device-side slot and position only, so the step can be captured in a CUDA graph.
        Fused mode leaves the kernel to the attention backend, unless this step moves a pin
        (the region then changes before attention runs, so the step is placed now)."""
        R = len(self._region)
        if self.fused and not self.next_step_moves_pin():
            self._pending = (k, v, R)
        else:
            self._place(k, v, R)
        self.t += 1
        self._pins_leave(self.t - self.window)
        rows = self.ring + R
        self.keys, self.values = self._kbuf[:, :, :rows], self._vbuf[:, :, :rows]
        return self.keys, self.values

    def _place(self, k, v, R):
        _lib.v2_place(self._kbuf, self._vbuf, k, v, self._reg_k, self._reg_pos, R, None, self._position, 0,
                      self.n_sink, self.window, self.inv_freq)

    def run_pending(self, query: torch.Tensor, scale: float, mask: torch.Tensor | None = None) -> torch.Tensor:
        """The deferred steady step fused with its attention; returns [B, 1, Hq, D]."""
        k, v, R = self._pending
        self._pending = None
        b, hq, _, d = query.shape
        out = torch.empty(b, 1, hq, d, dtype=query.dtype, device=query.device)
        return _lib.v2_decode_step(self._kbuf, self._vbuf, k, v, self._reg_k, self._reg_pos, R, self._position,
                                   self.n_sink, self.window, self.inv_freq, query, scale, out, self._ws, mask)

    def materialize(self) -> None:
        """Apply a deferred step without its attention."""
        if self._pending is not None:
            k, v, R = self._pending
            self._pending = None
            self._place(k, v, R)

    def _chunk_step(self, k, v):
        """Any chunk, the warm-up, or a one-token step before the window is full: attention
        gets a fresh [region, window, chunk] tensor; then the chunk is stored -- positions
        below n_sink join the region, pins that the chunk pushes out of the window join it
        next, and the chunk's positions that stay within a ring's reach go to their slots."""
        t, n = self.t, k.shape[-2]
        keys, values = self._logical(t, (k, v))
        end = t + n
        for p in range(t, min(end, self.n_sink)):
            self._region.add(k[:, :, p - t:p - t + 1], v[:, :, p - t:p - t + 1], p)
        self._pins_leave(end - self.window, chunk=(k, v, t))
        first = max(self.n_sink, end - self.ring, t)
        if first < end:
            done = first - t
            for buf, src in ((self._kbuf, k), (self._vbuf, v)):
                at = done
                for view in self._ring_views(buf, first, end):
                    view.copy_(src[:, :, at:at + view.shape[-2]])
                    at += view.shape[-2]
        self.t = end
        self._t_dev.fill_(end)
        self.keys, self.values = keys, values
        return keys, values

    def get_seq_length(self) -> int:
        """Absolute position of the next token (Transformers builds position_ids from it)."""
        return self.t

    def in_cache_length(self) -> int:
        """Rows a new query attends to besides itself: region + current window."""
        lo, hi = self._window_span(self.t)
        return len(self._region) + max(0, hi - lo)

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        """(kv_length, kv_offset) of the attention mask over [region, window, chunk].
        Transformers places the chunk's queries at get_seq_length() (the absolute position);
        kv_offset = t - in_cache_length lines the chunk's own keys up with them, so chunk
        query i sees chunk keys 0..i and every cached key -- the causal mask the reference
        gets from SinkCacheV2.get_query_offset (cache_v2.py:274-276)."""
        n = self.in_cache_length()
        return n + query_length, self.t - n

    def get_max_length(self) -> int:
        return self.region_cap + self.window

    def get_max_cache_shape(self) -> int:
        return self.region_cap + self.window

    def kept(self) -> tuple[torch.Tensor, torch.Tensor, list[int]]:
        """The logical cache for the next query: keys and values in the order [region,
        window by position], and the position each key is rotated at (region entries just
        before the window, window tokens at their own)."""
        self.materialize()
        t = self.t
        keys, values = self._logical(t)
        lo, hi = self._window_span(t)
        R, ws = len(self._region), self._window_start(t)
        return keys, values, list(range(ws - R, ws)) + list(range(lo, hi))

    def reset(self) -> None:
        self.t = self.moved_upto = 0
        self._region = _Region(self.n_sink, self.max_pinned)
        self.keys = self.values = None
        self._pending = None
        self.is_initialized = False

    def crop(self, tokens_to_remove: int) -> None:
        raise NotImplementedError("evicted tokens are gone; use snapshot()/restore() on the cache")

    def reorder_cache(self, beam_idx):
        raise NotImplementedError("beam search is not supported")

    # ------------------------------------------------------------------ snapshots

    def _state(self) -> _LayerState:
        self.materialize()
        return _LayerState(self._kbuf.clone(), self._vbuf.clone(), self._reg_k.clone(), self._reg_pos.clone(),
                           self.t, list(self._region.positions), self.moved_upto)

    def _load(self, s: _LayerState) -> None:
        """Write a saved state back into the same buffers (pointers kept, so a captured graph
        stays valid)."""
        self._pending = None
        for dst, src in ((self._kbuf, s.k), (self._vbuf, s.v), (self._reg_k, s.region_keys),
                         (self._reg_pos, s.region_pos)):
            dst.copy_(src)
        self.t, self.moved_upto = s.t, s.moved_upto
        self._region.positions[:] = s.positions
        self._position.copy_(torch.tensor([s.t, 0], dtype=torch.long))


class SinkCacheV2(Cache):
    """Attention sinks with the sinks moved forward and the window left alone (the interface
    of src/sinkcache/cache_v2.py:251-328).

        cache = SinkCacheV2.from_model(model, n_sink=4, window=1020)
        out = model(input_ids, past_key_values=cache, use_cache=True)

    `max_pinned`: extra region slots for pinned tokens (`cache.pin(start, end)`).  `fused`
    (default: whether the model uses the registered attention backend) runs steady
    one-token steps fused with their attention.
    """

    # position ids of a steady step come from the stream start, not from the buffer: a
    # graph-replayed step needs them fed from a device tensor (StreamRunner)
    absolute_positions = True

    def __init__(self, n_sink: int, window: int, inv_freq: torch.Tensor, num_layers: int, max_pinned: int = 0,
                 fused: bool = False):
        self.pinned: set[int] = set()  # one set for every layer
        self.workspace = _lib.Workspace()  # one for all layers: they run in order on one stream
        super().__init__(layers=[SinkLayerV2(n_sink, window, inv_freq, max_pinned, self.pinned, fused=fused,
                                             workspace=self.workspace) for _ in range(num_layers)])
        self.n_sink, self.window, self.max_pinned = n_sink, window, max_pinned

    @classmethod
    def from_model(cls, model, n_sink: int = 4, window: int = 1020, **kwargs) -> "SinkCacheV2":
        config = model.config.get_text_config(decoder=True)
        kinds = set(getattr(config, "layer_types", None) or ["full_attention"])
        if kinds != {"full_attention"}:
            raise ValueError(f"SinkCacheV2 supports full-attention models only, got {kinds}")
        kwargs.setdefault("fused", uses_sink_attention(model))
        return cls(n_sink, window, find_inv_freq(model), config.num_hidden_layers, **kwargs)

    def get_query_offset(self, layer_idx: int = 0) -> int:
        return self.layers[layer_idx].in_cache_length()

    def pin(self, start: int, end: int) -> None:
        """Keep absolute positions [start, end) when they leave the window (they move into
        the region).  Positions already past the window cannot be pinned."""
        if self.max_pinned == 0:
            raise ValueError("cache was built with max_pinned=0")
        gone = self.layers[0].moved_upto
        if start < gone:
            raise ValueError(f"positions before {gone} have already been evicted")
        self.pinned.update(range(start, end))

    @property
    def tokens_seen(self) -> int:
        return self.layers[0].t

    @property
    def tokens_evicted(self) -> int:
        first = self.layers[0]
        return first.t - first.in_cache_length()

    @property
    def region_size(self) -> int:
        return len(self.layers[0].region_pos)

    @property
    def is_steady(self) -> bool:
        """The next one-token step is the device-only steady step and moves no pin: it can
        be captured once and replayed."""
        first = self.layers[0]
        return (first.is_initialized and first.t >= self.n_sink + self.window
                and not first.next_step_moves_pin())

    def check_status(self) -> None:
        """Raise RuntimeError if one of this cache's kernels reported a failure since the
        last check; synchronises the stream."""
        self.workspace.check()

    # what a captured steady step depends on, and what a replay cannot advance

    def graph_signature(self):
        """Buffers and workspace the kernels were captured with, and the region size (the
        attention length)."""
        ws = self.workspace.buf
        return (tuple((l._kbuf.data_ptr(), l._vbuf.data_ptr()) for l in self.layers),
                None if ws is None else ws.data_ptr(), self.region_size)

    def note_replayed_step(self) -> None:
        """Host counters of one replayed steady step (the device position advanced itself)."""
        for layer in self.layers:
            layer.t += 1
            layer.moved_upto = max(layer.moved_upto, layer.t - layer.window)

    # the reference's names for the two (src/sinkcache/cache_v2.py:302-313)
    def layout_key(self):
        return self.region_size

    def advance_after_replay(self) -> None:
        self.note_replayed_step()

    def snapshot(self) -> V2Snapshot:
        """Device copies of every layer's state and the pinned positions; restore() writes
        them back in place (buffer pointers kept, so a captured CUDA graph stays valid)."""
        return V2Snapshot([layer._state() for layer in self.layers], frozenset(self.pinned))

    def restore(self, snap: V2Snapshot) -> None:
        for layer, state in zip(self.layers, snap.layers, strict=True):
            layer._load(state)
        self.pinned.clear()
        self.pinned.update(snap.pinned)
