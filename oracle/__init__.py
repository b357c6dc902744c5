"""CPU oracle of the sink-cache decode path -- test infrastructure only.

Restates the reference's own SinkCache algorithm (buttaRahul/Attention_sinks,
src/sinkcache/cache.py, rope.py, decode_attention.py) on the CPU.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may import it, as the checker.
The product package (attention_sinks_b200) never imports it.
"""

from .sink_oracle import (OracleSinkLayer, apply_rope, decode_attention, decode_step, reference_cpu_attention, reference_cpu_step,
                          make_prefilled_cache, rerotate, rerotate_fast, rope_cos_sin,
                          rotation_table)

from .sink_oracle_v2 import OracleSinkLayerV2, make_prefilled_cache_v2, reference_cpu_step_v2, region_rotation

__all__ = ["OracleSinkLayerV2", "make_prefilled_cache_v2", "reference_cpu_step_v2", "region_rotation",
           "OracleSinkLayer", "apply_rope", "decode_attention", "decode_step", "make_prefilled_cache", "reference_cpu_attention", "reference_cpu_step",
           "rerotate", "rerotate_fast", "rope_cos_sin", "rotation_table"]
