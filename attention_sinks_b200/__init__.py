"""attention_sinks_b200: the sink-cache decode path of sinkcache (buttaRahul/Attention_sinks)
on hand-written sm_100a CUDA kernels.

Public API (src/sinkcache/__init__.py:1-7 of the reference):
    SinkCache, SinkLayer, find_inv_freq     -- the cache (Transformers CacheLayerMixin)
    SinkCacheV2, SinkLayerV2                -- ring-buffer cache (sinks moved, window untouched)
    StreamRunner                            -- CUDA-graph streaming runner (both caches)
    flash_decode, register                  -- decode attention + Transformers backend
    apply_rope, rerotate                    -- RoPE helpers
"""

from .cache import SinkCache, SinkLayer, find_inv_freq
from .cache_v2 import SinkCacheV2, SinkLayerV2
from .decode_attention import decode_attention_forward, flash_decode, register
from .graphs import StreamRunner
from .rope import apply_rope, rerotate

__all__ = ["SinkCache", "SinkLayer", "SinkCacheV2", "SinkLayerV2", "StreamRunner", "find_inv_freq",
           "flash_decode", "register", "decode_attention_forward", "apply_rope", "rerotate"]
