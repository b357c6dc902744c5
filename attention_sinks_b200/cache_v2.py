"""Ring-buffer attention-sink cache ("v2"): the sinks move forward, the window stays put
(src/sinkcache/cache_v2.py:1-50).

RoPE attention depends only on relative position, so instead of re-rotating every window
key each step (v1), window keys keep the rotation the model gave them at their absolute
positions, the query sits at its absolute position t, and only the few region tokens (the
sinks, plus pinned tokens) are rotated -- from stored originals, with fp64 angles -- to sit
just before the window.  Keys are stored in the model dtype (no drift: window keys are never
rounded again).

Storage per layer: a ring of window + 1 slots (position p >= n_sink in slot
(p - n_sink) mod (window + 1)) followed by the region slots; attention reads one contiguous
view, ring then region.

Device work goes through the sm_100a library:
  * steady one-token step: sink_v2_place (ring write + region rotation + device position
    advance) and, when the model uses the registered attention backend, the same step fused
    with split-K decode attention (sink_v2_decode_step);
  * the region rotation of chunk steps and kept(): sink_v2_place into a gathered tensor.
The general (chunk) step's gather of the window in position order and its stores are
device tensor copies, as in the reference.  A steady step reads t from a device tensor,
so one captured CUDA graph serves every later token (StreamRunner).
"""

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _lib
from .cache import _BY_BUFFER, find_inv_freq, uses_sink_attention


class SinkLayerV2(CacheLayerMixin):
    """One layer of the ring-buffer cache (src/sinkcache/cache_v2.py:59-248)."""

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
        self.pinned = pinned if pinned is not None else set()
        self.t = 0                       # absolute position of the next token = tokens seen
        self.region_pos: list[int] = []  # original positions of region tokens (sinks, then pinned)
        self.moved_upto = 0              # pinned positions below this have been handled
        self.pins_dropped = 0
        self.fused = fused
        self._kbuf = self._vbuf = None
        self._pending = None             # (k, v, R) of a deferred steady step
        self._ws = workspace if workspace is not None else _lib.Workspace()

    # ------------------------------------------------------------------ storage

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        _lib.check_device(self.device)
        _lib.prepare_device(self.device)  # before any graph capture of this layer's steps
        b, h, _, d = key_states.shape
        if 2 * self.inv_freq.numel() > d:
            raise ValueError(f"rotary dims {2 * self.inv_freq.numel()} exceed head_dim {d}")
        n = self.ring + self.region_cap
        self._kbuf = torch.zeros(b, h, n, d, dtype=self.dtype, device=self.device)
        self._vbuf = torch.zeros(b, h, n, d, dtype=self.dtype, device=self.device)
        self._reg_k = torch.zeros(b, h, max(self.region_cap, 1), d, dtype=self.dtype, device=self.device)
        self._reg_pos = torch.zeros(max(self.region_cap, 1), dtype=torch.long, device=self.device)
        # {t, arrival counter}: t is read and advanced by the steady-step kernel
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

    def _slot(self, p: int) -> int:
        return (p - self.n_sink) % self.ring

    def _slots(self, lo: int, hi: int) -> torch.Tensor:
        """Ring slots of positions [lo, hi) (all >= n_sink) as a device index tensor, computed
        on the device (cache_v2.py:190, 202 build them as host lists)."""
        return (torch.arange(lo, max(lo, hi), device=self.device) - self.n_sink) % self.ring

    def _window_start(self, t: int) -> int:
        return max(min(t, self.n_sink), t - self.window)

    def _assemble(self, R: int, window: list[torch.Tensor], chunk: torch.Tensor | None,
                  region: torch.Tensor | None = None) -> torch.Tensor:
        """[region (R rows), window rows, chunk] in one new tensor, filled by slice copies
        (torch.cat of these strided views runs far below the copy bandwidth).  Region rows
        are copied from `region`, or left for the caller to write when it is None."""
        b, h, _, d = self._kbuf.shape
        n = R + sum(x.shape[-2] for x in window) + (chunk.shape[-2] if chunk is not None else 0)
        out = torch.empty(b, h, n, d, dtype=self.dtype, device=self.device)
        if region is not None and R:
            out[:, :, :R].copy_(region)
        o = R
        for x in window + ([chunk] if chunk is not None else []):
            out[:, :, o:o + x.shape[-2]].copy_(x)
            o += x.shape[-2]
        return out

    def _ring_rows(self, buf: torch.Tensor, lo: int, hi: int) -> list[torch.Tensor]:
        """Rows of positions [lo, hi) (all >= n_sink, fewer than a ring) in position order, as
        at most two contiguous views of the ring: the same rows the reference gathers with an
        index list (cache_v2.py:189-193), without the gather."""
        n = hi - lo
        if n <= 0:
            return []
        s0 = (lo - self.n_sink) % self.ring
        if s0 + n <= self.ring:
            return [buf[:, :, s0:s0 + n]]
        return [buf[:, :, s0:self.ring], buf[:, :, :s0 + n - self.ring]]

    # ------------------------------------------------------------------ rotation

    def _rotate_region(self, t: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Region keys rotated from their originals to positions ws-R..ws-1, ws the window
        start when the next token is t (cache_v2.py:101-116), by the place kernel."""
        R = len(self.region_pos)
        b, h, _, d = self._kbuf.shape
        if out is None:
            out = torch.empty(b, h, R, d, dtype=self.dtype, device=self.device)
        if R:
            _lib.v2_place(self._kbuf, self._vbuf, None, None, self._reg_k, self._reg_pos, R, out, None, t,
                          self.n_sink, self.window, self.inv_freq)
        return out

    # ------------------------------------------------------------------ region bookkeeping

    def _region_append(self, k: torch.Tensor, v: torch.Tensor, p: int):
        """k, v: [b, h, 1, d]; k at its original rotation (position p) (cache_v2.py:120-130)."""
        if len(self.region_pos) == self.region_cap:
            if self.max_pinned == 0:
                raise RuntimeError("region full")
            self._region_drop_oldest_pin()
        j = len(self.region_pos)
        self._reg_k[:, :, j:j + 1].copy_(k)
        self._vbuf[:, :, self.ring + j:self.ring + j + 1].copy_(v)
        self._reg_pos[j] = p
        self.region_pos.append(p)

    def _region_drop_oldest_pin(self):
        """cache_v2.py:132-138"""
        s, R, r = self.n_sink, len(self.region_pos), self.ring
        self._reg_k[:, :, s:R - 1] = self._reg_k[:, :, s + 1:R].clone()
        self._vbuf[:, :, r + s:r + R - 1] = self._vbuf[:, :, r + s + 1:r + R].clone()
        self._reg_pos[s:R - 1] = self._reg_pos[s + 1:R].clone()
        del self.region_pos[s]
        self.pins_dropped += 1

    def _move_pins(self, bound: int, chunk=None):
        """Pinned positions in [moved_upto, bound) have left the window: into the region
        (cache_v2.py:140-151)."""
        if self.pinned and bound > self.moved_upto:
            for p in sorted(p for p in self.pinned if self.moved_upto <= p < bound and p >= self.n_sink):
                if chunk is not None and p >= chunk[2]:
                    i = p - chunk[2]
                    self._region_append(chunk[0][:, :, i:i + 1], chunk[1][:, :, i:i + 1], p)
                else:
                    sl = self._slot(p)
                    self._region_append(self._kbuf[:, :, sl:sl + 1], self._vbuf[:, :, sl:sl + 1], p)
        self.moved_upto = max(self.moved_upto, bound)

    def next_step_moves_pin(self) -> bool:
        """Would a one-token step at the current position move a pin afterwards?"""
        return (self.t - self.window) in self.pinned and self.t - self.window >= self.n_sink

    # ------------------------------------------------------------------ cache API

    def update(self, key_states, value_states, *args, **kwargs):
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.materialize()
        q = key_states.shape[-2]
        if q == 1 and self.t >= self.n_sink + self.window:
            return self._decode_step(key_states, value_states)
        return self._general_step(key_states, value_states)

    def _decode_step(self, k, v):
        """Steady state (cache_v2.py:167-181): device-side slot and position only, so the step
        can be captured in a CUDA graph.  Fused mode defers the place kernel to the attention
        backend, unless this step moves a pin (then the region changes before attention
        runs, exactly as in the reference, so the step is placed now)."""
        R = len(self.region_pos)
        if self.fused and not self.next_step_moves_pin():
            self._pending = (k, v, R)
        else:
            self._place(k, v, R)
        self.t += 1
        self._move_pins(self.t - self.window)
        n = self.ring + R
        self.keys, self.values = self._kbuf[:, :, :n], self._vbuf[:, :, :n]
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
        if self._pending is None:
            return
        k, v, R = self._pending
        self._pending = None
        self._place(k, v, R)

    def _general_step(self, k, v):
        """Any chunk, warm-up, or a one-token step before the window is full
        (cache_v2.py:183-208): attention gets [region (rotated), window in position order,
        new chunk]; then the new tokens are stored."""
        t, q = self.t, k.shape[-2]
        ws = self._window_start(t)
        R = len(self.region_pos)
        lo = max(ws, self.n_sink)
        r = self.ring
        keys = self._assemble(R, self._ring_rows(self._kbuf, lo, t), k)
        self._rotate_region(t, keys[:, :, :R])
        values = self._assemble(R, self._ring_rows(self._vbuf, lo, t), v, self._vbuf[:, :, r:r + R])

        for i in range(q):
            if t + i < self.n_sink:
                self._region_append(k[:, :, i:i + 1], v[:, :, i:i + 1], t + i)
        self._move_pins(t + q - self.window, chunk=(k, v, t))
        lo = max(self.n_sink, t + q - self.ring, t)
        if lo < t + q:
            idx = self._slots(lo, t + q)
            self._kbuf.index_copy_(2, idx, k[:, :, lo - t:])
            self._vbuf.index_copy_(2, idx, v[:, :, lo - t:])
        self.t = t + q
        self._t_dev.fill_(self.t)
        self.keys, self.values = keys, values
        return keys, values

    def get_seq_length(self) -> int:
        """Absolute position of the next token (Transformers builds position_ids from this)."""
        return self.t

    def in_cache_length(self) -> int:
        """Tokens a new query attends to besides itself: region + current window."""
        return len(self.region_pos) + (self.t - max(self._window_start(self.t), self.n_sink)
                                       if self.t > self.n_sink else 0)

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
        """Logical cache for the next query: keys/values in order [region, window by
        position], and the positions they are rotated at (cache_v2.py:225-236)."""
        self.materialize()
        t = self.t
        ws = self._window_start(t)
        R = len(self.region_pos)
        win = list(range(max(ws, self.n_sink), t))
        r = self.ring
        lo = win[0] if win else t
        k = self._assemble(R, self._ring_rows(self._kbuf, lo, t), None)
        self._rotate_region(t, k[:, :, :R])
        v = self._assemble(R, self._ring_rows(self._vbuf, lo, t), None, self._vbuf[:, :, r:r + R])
        return k, v, [ws - R + j for j in range(R)] + win

    def reset(self) -> None:
        self.t = self.moved_upto = self.pins_dropped = 0
        self.region_pos = []
        self.keys = self.values = None
        self._pending = None
        self.is_initialized = False

    def crop(self, tokens_to_remove: int) -> None:
        raise NotImplementedError("evicted tokens are gone; use snapshot()/restore() on the cache")

    def reorder_cache(self, beam_idx):
        raise NotImplementedError("beam search is not supported")


class SinkCacheV2(Cache):
    """Attention sinks with the sinks moved forward and the window left alone
    (src/sinkcache/cache_v2.py:251-328).

        cache = SinkCacheV2.from_model(model, n_sink=4, window=1020)
        out = model(input_ids, past_key_values=cache, use_cache=True)

    `max_pinned`: extra region slots for pinned tokens (`cache.pin(start, end)`).  `fused`
    (default: whether the model uses the registered attention backend) runs steady
    one-token steps fused with their attention.
    """

    def __init__(self, n_sink: int, window: int, inv_freq: torch.Tensor, num_layers: int, max_pinned: int = 0,
                 fused: bool = False):
        self.pinned: set[int] = set()
        self.workspace = _lib.Workspace()  # one for all layers: they run in order on one stream
        layers = [SinkLayerV2(n_sink, window, inv_freq, max_pinned, self.pinned, fused=fused,
                              workspace=self.workspace) for _ in range(num_layers)]
        super().__init__(layers=layers)
        self.n_sink, self.window, self.max_pinned = n_sink, window, max_pinned

    @classmethod
    def from_model(cls, model, n_sink: int = 4, window: int = 1020, **kwargs) -> "SinkCacheV2":
        config = model.config.get_text_config(decoder=True)
        layer_types = getattr(config, "layer_types", None) or ["full_attention"] * config.num_hidden_layers
        if any(t != "full_attention" for t in layer_types):
            raise ValueError(f"SinkCacheV2 supports full-attention models only, got {set(layer_types)}")
        kwargs.setdefault("fused", uses_sink_attention(model))
        return cls(n_sink, window, find_inv_freq(model), config.num_hidden_layers, **kwargs)

    def get_query_offset(self, layer_idx: int = 0) -> int:
        return self.layers[layer_idx].in_cache_length()

    def pin(self, start: int, end: int) -> None:
        """Pin absolute positions [start, end).  Must be called before they leave the window."""
        if self.max_pinned == 0:
            raise ValueError("cache was built with max_pinned=0")
        if start < self.layers[0].moved_upto:
            raise ValueError(f"positions before {self.layers[0].moved_upto} have already been evicted")
        self.pinned.update(range(start, end))

    @property
    def tokens_seen(self) -> int:
        return self.layers[0].t

    @property
    def tokens_evicted(self) -> int:
        layer = self.layers[0]
        return layer.t - layer.in_cache_length()

    @property
    def region_size(self) -> int:
        return len(self.layers[0].region_pos)

    @property
    def is_steady(self) -> bool:
        """The next one-token step takes the device-only path and moves no pin: safe to
        capture/replay."""
        layer = self.layers[0]
        return (layer.is_initialized and layer.t >= self.n_sink + self.window
                and not layer.next_step_moves_pin())

    def layout_key(self):
        """What changes the captured computation: the region size (attention length)."""
        return self.region_size

    def advance_after_replay(self):
        for layer in self.layers:
            layer.t += 1
            layer.moved_upto = max(layer.moved_upto, layer.t - layer.window)

    def snapshot(self):
        """Device copies of all state; restore() writes them back in place (buffer pointers
        kept, so a captured CUDA graph stays valid) (cache_v2.py:315-319)."""
        for layer in self.layers:
            layer.materialize()
        return [(l._kbuf.clone(), l._vbuf.clone(), l._reg_k.clone(), l._reg_pos.clone(), l.t,
                 list(l.region_pos), l.moved_upto) for l in self.layers], set(self.pinned)

    def restore(self, snap):
        """cache_v2.py:321-328"""
        layers, pinned = snap
        for l, (kb, vb, rk, rp, t, rpos, mu) in zip(self.layers, layers):
            l._pending = None
            l._kbuf.copy_(kb), l._vbuf.copy_(vb), l._reg_k.copy_(rk), l._reg_pos.copy_(rp)
            l.t, l.region_pos, l.moved_upto = t, list(rpos), mu
            l._position.zero_()
            l._t_dev.fill_(t)
        self.pinned.clear()
        self.pinned.update(pinned)
