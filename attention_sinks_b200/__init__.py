"""attention_sinks_b200: the sink-cache decode path of sinkcache (buttaRahul/Attention_sinks)
on hand-written sm_100a CUDA kernels.

Public API (src/sinkcache/__init__.py:1-7 of the reference, v1 cache):
    SinkCache, SinkLayer, find_inv_freq     -- the cache (Transformers CacheLayerMixin)
    StreamRunner                            -- CUDA-graph streaming runner
    flash_decode, register                  -- decode attention + Transformers backend
    apply_rope, rerotate                    -- RoPE helpers
"""

from .cache import SinkCache, SinkLayer, find_inv_freq
from .decode_attention import decode_attention_forward, flash_decode, register
from .graphs import StreamRunner
from .rope import apply_rope, rerotate

__all__ = ["SinkCache", "SinkLayer", "StreamRunner", "find_inv_freq", "flash_decode", "register",
           "decode_attention_forward", "apply_rope", "rerotate"]
