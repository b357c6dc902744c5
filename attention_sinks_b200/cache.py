"""Attention-sink (StreamingLLM) KV cache for the Transformers 5 per-layer cache API, with
every cache operation in the sm_100a CUDA library.

Each layer keeps the first `n_sink` tokens forever plus a rolling window of the `window`
most recent tokens.  Transformers places a new token at position `get_seq_length()`, so
the kept keys must sit at contiguous positions 0..capacity-1: when `drop` tokens leave the
front of the window, every surviving window key is rotated by -drop (RoPE angles add).
Eviction is deferred to the next `update` so that this step's attention still sees the
keys at the positions its query was rotated for (src/sinkcache/cache.py:1-41).

Storage is the reference layout: [B, Hkv, n_sink + window + 1, D] buffers, keys in
float32 by default (one rounding per re-rotation in bf16 would drift), values in the model
dtype (src/sinkcache/cache.py:97-104).

Two ways to run a one-token decode step:
  * unfused (any attention backend): `update` evicts + re-rotates in place
    (sink_evict_rerotate), appends (sink_append) and returns the cache views;
  * fused (the model uses the attention backend of `decode_attention.register`): `update`
    records the step and returns the float32 key view; the backend then runs
    sink_fused_decode_step, which evicts, re-rotates, appends and attends in one pass over
    the cache, reading each window row once and writing it once.
"""

import weakref

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _lib
from .rope import rope_cos_sin

# K-buffer data_ptr -> layer, so the attention backend can find the layer whose deferred
# step produced the key view it was handed.
_BY_BUFFER: "weakref.WeakValueDictionary[int, SinkLayer]" = weakref.WeakValueDictionary()


def pending_layer(key: torch.Tensor) -> "SinkLayer | None":
    """The layer with a deferred one-token step whose key view is `key`, if any."""
    layer = _BY_BUFFER.get(key.data_ptr())
    if layer is None or layer._pending is None or layer._kbuf is None:
        return None
    if layer._kbuf.data_ptr() != key.data_ptr():
        return None
    return layer


class KeyCopy:
    """Device buffer for the model-dtype key copy a multi-token (or unfused) step hands to
    attention, grown on demand and reused.  A cache's layers share one: each layer's copy is
    consumed by its attention before the next layer's update overwrites it."""

    def __init__(self):
        self.buf = None

    def view(self, b: int, h: int, rows: int, d: int, dtype: torch.dtype, device) -> torch.Tensor:
        n = b * h * rows * d
        if self.buf is None or self.buf.numel() < n or self.buf.dtype != dtype or self.buf.device != device:
            self.buf = torch.empty(n, dtype=dtype, device=device)
        return self.buf[:n].view(b, h, rows, d)


class SinkLayer(CacheLayerMixin):
    """One layer's cache: `n_sink` sink tokens + a rolling window of `window` tokens
    (src/sinkcache/cache.py:54-198)."""

    is_sliding = False    # masks treat it as a full-attention layer over what it returns
    is_croppable = False  # evicted tokens are gone

    def __init__(self, n_sink: int, window: int, inv_freq: torch.Tensor, rerotate_keys: bool = True,
                 use_triton: bool | None = None, key_dtype: torch.dtype | None = None,
                 fused: bool = False, workspace: "_lib.Workspace | None" = None,
                 key_copy: "KeyCopy | None" = None):
        super().__init__()
        if n_sink < 0 or window < 1:
            raise ValueError(f"need n_sink >= 0 and window >= 1, got {n_sink}, {window}")
        self.n_sink = n_sink
        self.window = window
        self.capacity = n_sink + window
        self.inv_freq = inv_freq
        self.rerotate_keys = rerotate_keys
        self.length = 0             # valid rows in the buffer, including a pending eviction
        self.tokens_seen = 0
        self.tokens_evicted = 0
        # Accepted for signature compatibility with the reference; the CUDA kernels always run.
        self.use_triton = use_triton
        self.key_dtype = key_dtype
        self.fused = fused
        self._rot: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        self._kbuf = self._vbuf = None
        self._kstore = self._vstore = None  # row storage the buffers view (see _alloc)
        self._pending = None        # (drop, k, v, append_row) of a deferred one-token step
        self._ws = workspace if workspace is not None else _lib.Workspace()
        self._key_copy = key_copy if key_copy is not None else KeyCopy()

    # ------------------------------------------------------------------ storage

    def lazy_initialization(self, key_states, value_states):
        self.dtype, self.device = key_states.dtype, key_states.device
        _lib.check_device(self.device)
        _lib.prepare_device(self.device)  # before any graph capture of this layer's steps
        self.key_dtype = self.key_dtype or self.dtype
        self.inv_freq = self.inv_freq.to(self.device)
        if self.rerotate_keys and 2 * self.inv_freq.numel() != key_states.shape[-1]:
            raise NotImplementedError("sinkcache_b200 re-rotates full-rotary heads only "
                                      f"(rot_dim {2 * self.inv_freq.numel()} != head_dim {key_states.shape[-1]})")
        self._alloc(key_states, self.capacity + 1)
        self._rotation(1)  # the steady-state shift; built now so a graph capture never builds it
        self._size_workspace(key_states)
        if self.key_dtype != self.dtype:  # the steady step's key copy, before any capture
            b, h, _, d = key_states.shape
            self._key_copy.view(b, h, self.capacity + 1, d, self.dtype, self.device)
        self.is_initialized = True

    def _alloc(self, like, slots):
        """Make the K/V buffers `slots` rows long, keeping their first `length` rows (the
        reference reallocates on every grow and shrink, cache.py:97-104, 142-143).  The
        buffers are views of a row storage that is only replaced when a chunk needs more
        rows than it has (rows copied once, then later chunks of that size fit) or when a
        shrink back to capacity + 1 would leave more than twice the rows idle: the usual
        chunk step grows and shrinks without copying the cache, and the buffer pointers of
        a captured steady step stay valid."""
        b, h, _, d = like.shape
        store = self._kstore.shape[-2] if self._kstore is not None else 0
        small = slots == self.capacity + 1
        if slots <= store and not (small and store > 2 * slots):
            self._kbuf, self._vbuf = self._kstore[:, :, :slots], self._vstore[:, :, :slots]
            return
        k = torch.empty(b, h, slots, d, dtype=self.key_dtype, device=self.device)
        v = torch.empty(b, h, slots, d, dtype=self.dtype, device=self.device)
        if self.length:
            k[:, :, :self.length] = self._kbuf[:, :, :self.length]
            v[:, :, :self.length] = self._vbuf[:, :, :self.length]
        self._kstore, self._vstore = k, v
        self._kbuf, self._vbuf = k, v
        _BY_BUFFER[k.data_ptr()] = self

    def _size_workspace(self, like):
        """Size the shared workspace for every steady-state launch before any graph capture."""
        b, h, _, d = like.shape
        sms = _lib.sm_count(self.device)
        rows = self.capacity + 1
        hq = h * 8  # largest supported GQA group
        need = max(
            _lib.workspace_bytes(_lib.OP_EVICT, b, h, h, d, self.key_dtype, self.dtype, 0,
                                 self.n_sink, self.window, 1, sms),
            _lib.workspace_bytes(_lib.OP_FUSED_STEP, b, h, hq, d, self.key_dtype, self.dtype, rows,
                                 self.n_sink, self.window, 1, sms),
            _lib.workspace_bytes(_lib.OP_ATTEND, b, h, hq, d, self.key_dtype, self.dtype, rows,
                                 0, 1, 0, sms),
        )
        self._ws.get(need, self.device)

    # ------------------------------------------------------------------ rotation

    def _rotation(self, delta: int) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 (cos, sin) [head_dim] tables for a rotation by -delta (cache.py:108-114).
        Built once per shift with the host's libm, so the angles' cos/sin are bit-identical
        to the reference's CPU path, then copied to the device."""
        if delta not in self._rot:
            cos, sin = rope_cos_sin(torch.tensor(-delta), self.inv_freq.cpu())
            self._rot[delta] = (cos.to(self.device), sin.to(self.device))
        return self._rot[delta]

    def _evict(self, kbuf, vbuf, drop, key_copy=None):
        cos, sin = self._rotation(drop) if self.rerotate_keys else (None, None)
        if key_copy is None:
            _lib.evict_rerotate(kbuf, vbuf, self.n_sink, self.window, drop, cos, sin, self._ws)
        else:
            _lib.evict_rerotate_keycopy(kbuf, vbuf, self.n_sink, self.window, drop, cos, sin, key_copy, self._ws)

    def _evict_pending(self, key_copy=None):
        """Shift the window left by the pending `drop` rows, re-rotating keys by -drop, in
        place (cache.py:129-147).  With `key_copy`, the same pass writes the window rows'
        keys in the model dtype into it."""
        drop = self.length - self.capacity
        if drop <= 0:
            return
        self._evict(self._kbuf, self._vbuf, drop, key_copy)
        self.length = self.capacity
        self.tokens_evicted += drop
        if self._kbuf.shape[-2] > self.capacity + 1:  # a long chunk grew the buffer: shrink back
            self._alloc(self._kbuf, self.capacity + 1)

    # ------------------------------------------------------------------ cache API

    def update(self, key_states, value_states, *args, **kwargs):
        """Evict what is pending, append the new rows, return this step's K/V
        (cache.py:151-165).  In fused mode a one-token step is deferred to the attention
        backend (see the module docstring)."""
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.materialize()
        q = key_states.shape[-2]
        if self.fused and q == 1 and self._kbuf.shape[-2] == self.capacity + 1:
            drop = max(self.length - self.capacity, 0)
            row = self.length - drop
            self._pending = (drop, key_states, value_states, row)
            self.length = row + 1
            self.tokens_seen += 1
            self.tokens_evicted += drop
            self.keys, self.values = self._kbuf[:, :, :self.length], self._vbuf[:, :, :self.length]
            return self.keys, self.values
        copy_keys = self.key_dtype != self.dtype
        # The keys attention gets are the model-dtype copy of the buffer (cache.py:163).  Its
        # window rows come out of the eviction kernel's pass (no separate read of the float32
        # keys); the sink rows and the new rows are copied here.
        b, h, _, d = key_states.shape
        end = min(self.length, self.capacity) + q
        kc = self._key_copy.view(b, h, end, d, self.dtype, self.device) if copy_keys else None
        evicting = self.length > self.capacity
        self._evict_pending(kc)
        if copy_keys and not evicting and self.length > self.n_sink:  # nothing moved: convert
            _lib.evict_rerotate_keycopy(self._kbuf, self._vbuf, self.n_sink, self.length - self.n_sink, 0, None,
                                        None, kc, self._ws)
        start = self.length
        end = start + q
        if end > self._kbuf.shape[-2]:
            self._alloc(key_states, end)
        _lib.append(self._kbuf, self._vbuf, key_states, value_states, start)
        self.length = end
        self.tokens_seen += q
        if copy_keys:
            s = min(self.n_sink, start)
            if s:
                kc[:, :, :s].copy_(self._kbuf[:, :, :s])
            kc[:, :, start:end].copy_(key_states)
            keys = kc
        else:
            keys = self._kbuf[:, :, :end]
        # the layer keeps views of its own buffers; the copy is valid until the next layer's update
        self.keys, self.values = self._kbuf[:, :, :end], self._vbuf[:, :, :end]
        return keys, self.values

    def run_pending(self, query: torch.Tensor, scale: float, mask: torch.Tensor | None = None) -> torch.Tensor:
        """Run the deferred step fused with its attention; returns [B, 1, Hq, D].  `mask`:
        optional boolean [B, 1, 1, rows] (rows left out of the attention where False)."""
        drop, k, v, row = self._pending
        self._pending = None
        cos, sin = self._rotation(drop) if (drop > 0 and self.rerotate_keys) else (None, None)
        b, hq, _, d = query.shape
        out = torch.empty(b, 1, hq, d, dtype=query.dtype, device=query.device)
        return _lib.fused_decode_step(self._kbuf, self._vbuf, k, v, query, self.n_sink, self.window,
                                      drop, row, cos, sin, scale, out, self._ws, mask)

    def materialize(self) -> None:
        """Apply a deferred step (eviction + append) without its attention."""
        if self._pending is None:
            return
        drop, k, v, row = self._pending
        self._pending = None
        if drop > 0:
            self._evict(self._kbuf, self._vbuf, drop)
        _lib.append(self._kbuf, self._vbuf, k, v, row)

    def get_seq_length(self) -> int:
        """Logical length: what remains after pending evictions; the next token's position."""
        return min(self.length, self.capacity)

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.get_seq_length() + query_length, 0

    def get_max_length(self) -> int:
        return self.capacity

    def get_max_cache_shape(self) -> int:
        return self.capacity

    def kept(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The logical cache (pending eviction applied) without mutating the layer
        (cache.py:177-186): the eviction kernel runs on copies."""
        self.materialize()
        n, cap = self.length, self.capacity
        k, v = self._kbuf[:, :, :n], self._vbuf[:, :, :n]
        if n - cap <= 0:
            return k, v
        k, v = k.clone(), v.clone()
        self._evict(k, v, n - cap)
        return k[:, :, :cap], v[:, :, :cap]

    def reset(self) -> None:
        self.length = self.tokens_seen = self.tokens_evicted = 0
        self.keys = self.values = None
        self._kbuf = self._vbuf = None
        self._kstore = self._vstore = None
        self._pending = None
        self.is_initialized = False

    def crop(self, tokens_to_remove: int) -> None:
        raise NotImplementedError("SinkLayer evicts tokens permanently and cannot be cropped")

    def reorder_cache(self, beam_idx):
        raise NotImplementedError("beam search is not supported")


def find_inv_freq(model) -> torch.Tensor:
    """The RoPE inverse frequencies the model actually uses, after any rope scaling such as
    llama3 (cache.py:201-206)."""
    for module in model.modules():
        if hasattr(module, "inv_freq") and hasattr(module, "attention_scaling"):
            return module.inv_freq.detach().clone()
    raise ValueError("no rotary embedding module with `inv_freq` found in model")


def uses_sink_attention(model) -> bool:
    """True when the model dispatches attention to a backend registered by
    `decode_attention.register` (then one-token steps run fused)."""
    from .decode_attention import REGISTERED
    impl = getattr(model.config, "_attn_implementation", None)
    return impl in REGISTERED


class SinkCache(Cache):
    """StreamingLLM cache: `n_sink` attention sinks + a window of the `window` most recent
    tokens (cache.py:209-256).

        cache = SinkCache.from_model(model, n_sink=4, window=1020)
        out = model(input_ids, past_key_values=cache, use_cache=True)

    `n_sink=0` gives a plain sliding window; `rerotate_keys=False` keeps stale rotations
    (the position bug, for ablation); `key_dtype` is the key storage type (float32 by
    default, None for the model dtype).  `fused` (default: whether the model uses the
    registered attention backend) runs one-token steps as one fused kernel pass.
    """

    def __init__(self, n_sink: int, window: int, inv_freq: torch.Tensor, num_layers: int,
                 rerotate_keys: bool = True, use_triton: bool | None = None,
                 key_dtype: torch.dtype | None = torch.float32, fused: bool = False):
        # one workspace and one key copy for all layers: they run one after another on one stream
        self.workspace = _lib.Workspace()
        self.key_copy = KeyCopy()
        layers = [SinkLayer(n_sink, window, inv_freq, rerotate_keys, use_triton, key_dtype,
                            fused=fused, workspace=self.workspace, key_copy=self.key_copy)
                  for _ in range(num_layers)]
        super().__init__(layers=layers)
        self.n_sink, self.window = n_sink, window

    @classmethod
    def from_model(cls, model, n_sink: int = 4, window: int = 1020, **kwargs) -> "SinkCache":
        config = model.config.get_text_config(decoder=True)
        layer_types = getattr(config, "layer_types", None) or ["full_attention"] * config.num_hidden_layers
        if any(t != "full_attention" for t in layer_types):
            raise ValueError(f"SinkCache supports full-attention models only, got layer types {set(layer_types)}")
        kwargs.setdefault("fused", uses_sink_attention(model))
        return cls(n_sink, window, find_inv_freq(model), config.num_hidden_layers, **kwargs)

    @property
    def capacity(self) -> int:
        return self.n_sink + self.window

    @property
    def is_steady(self) -> bool:
        """Full, with exactly one pending eviction and a minimal buffer: every further
        one-token step is identical in shape and position (safe to capture in a CUDA graph)."""
        layer = self.layers[0]
        return (layer.is_initialized and layer.tokens_evicted > 0
                and layer.length == self.capacity + 1 == layer._kbuf.shape[-2])

    @property
    def tokens_seen(self) -> int:
        return self.layers[0].tokens_seen

    def check_status(self) -> None:
        """Raise RuntimeError if one of this cache's kernels reported a failure (a bounded wait
        for a bulk copy that ran out) since the last check; synchronises the stream."""
        self.workspace.check()

    # What a captured steady step depends on, and what a replay cannot advance (used by
    # StreamRunner).  Positions are in-cache here: a steady step always sits at `capacity`.
    absolute_positions = False

    def graph_signature(self):
        """The buffers and workspace the step's kernels were captured with."""
        ws = self.workspace.buf
        return (tuple((l._kbuf.data_ptr(), l._vbuf.data_ptr()) for l in self.layers),
                None if ws is None else ws.data_ptr())

    def note_replayed_step(self) -> None:
        """Counters of one replayed steady step: one token seen, one evicted, per layer."""
        for layer in self.layers:
            layer.tokens_seen += 1
            layer.tokens_evicted += 1

    @property
    def tokens_evicted(self) -> int:
        return self.layers[0].tokens_evicted
