"""Split-K GQA decode attention for one query token, and the Transformers attention backend
that drives the fused sink-cache decode step.

`flash_decode` (src/sinkcache/decode_attention.py:102-130) runs the sm_100a kernels: each
CTA streams one split of one (batch, kv-head) pair's rows through a bulk-copy (TMA)
shared-memory pipeline, keeps an fp32 online softmax for the whole GQA group, and a second
kernel merges the splits.  Keys may be float32 (the sink cache's storage, read directly:
no bf16 copy of the cache per step) or the model dtype.

`register(name)` (decode_attention.py:149-156) installs `decode_attention_forward` as a
Transformers attention backend: one-token steps run on the kernels -- fused with the cache
update when the key view comes from a deferred SinkLayer step -- with no mask or a boolean
one; multi-token chunks (prefill) and other masks fall back to SDPA, as in the reference.
"""

import torch

from . import _lib
from .cache import pending_layer

REGISTERED: set[str] = set()
calls = {"decode_kernel": 0, "fused_step": 0, "sdpa_fallback": 0}


def flash_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                 mask: torch.Tensor | None = None) -> torch.Tensor:
    """q [B, Hq, 1, D]; k, v [B, Hkv, L, D] with contiguous rows (views of a larger cache
    buffer are fine).  Returns the attention output as [B, 1, Hq, D] in q's dtype.
    `mask`: optional boolean [B or 1, 1, 1, L], True = attend."""
    bsz, hq, q_len, dim = q.shape
    if q_len != 1 or hq % k.shape[1]:
        raise ValueError(f"flash_decode needs one query token and Hq % Hkv == 0, got q {tuple(q.shape)}, "
                         f"k {tuple(k.shape)}")
    if k.shape[-2] > 1 and k.stride(-2) != dim:  # rows must be contiguous for the bulk copies
        k = k.contiguous()
    if v.shape[-2] > 1 and v.stride(-2) != dim:
        v = v.contiguous()
    out = torch.empty(bsz, 1, hq, dim, device=q.device, dtype=q.dtype)
    return _lib.decode_attention(q, k, v, k.shape[2], scale, out, _workspace_for(q.device), mask)


# Workspaces of flash_decode, one per (device, stream): calls on one stream run in order, so
# they can share one; a call on another stream gets its own.
_WORKSPACES: dict[tuple[int, int], _lib.Workspace] = {}


def _workspace_for(device: torch.device) -> _lib.Workspace:
    """The workspace of this device's current stream, grown on demand and reused across
    calls (no allocation or memset per call).  Inside a CUDA-graph capture a fresh one is
    allocated from the graph's memory pool instead, as the reference allocates its
    partials per call: a cached buffer grown during a capture would belong to that pool."""
    if device.type != "cuda" or torch.cuda.is_current_stream_capturing():
        return _lib.Workspace()
    stream = torch.cuda.current_stream(device)
    key = (stream.device_index, stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = _WORKSPACES[key] = _lib.Workspace()
    return ws


def _on_kernel_device(query: torch.Tensor) -> bool:
    return query.is_cuda


def _kernel_mask_ok(mask, query: torch.Tensor, key: torch.Tensor) -> bool:
    """The kernels take no mask or a boolean [B or 1, 1, 1, L] one.  Transformers skips the
    mask of an unpadded one-token step, except while a CUDA graph is being captured, when it
    passes the all-True boolean mask instead; padded batches pass a boolean mask too."""
    if mask is None:
        return True
    return (mask.dtype == torch.bool and mask.dim() == 4 and mask.shape[1] == 1 and mask.shape[2] == 1
            and mask.shape[3] == key.shape[-2] and mask.shape[0] in (1, query.shape[0]))


def decode_attention_forward(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    """Transformers attention function (decode_attention.py:136-146): the sm_100a kernels
    for one query token, SDPA otherwise."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    layer = pending_layer(key)
    if (query.shape[2] == 1 and _on_kernel_device(query) and not module.training
            and _kernel_mask_ok(attention_mask, query, key)):
        scale = scaling if scaling is not None else query.shape[-1] ** -0.5
        if layer is not None:
            calls["fused_step"] += 1
            return layer.run_pending(query, scale, attention_mask), None
        calls["decode_kernel"] += 1
        return flash_decode(query, key, value, scale, attention_mask), None
    if layer is not None:
        layer.materialize()
    calls["sdpa_fallback"] += 1
    if key.dtype != query.dtype:  # float32 key storage
        key = key.to(query.dtype)
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                  scaling=scaling, **kwargs)


def register(name: str = "sdpa_decode") -> str:
    """Register the backend; then load the model with attn_implementation=name
    (decode_attention.py:149-156)."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask

    AttentionInterface.register(name, decode_attention_forward)
    AttentionMaskInterface.register(name, sdpa_mask)
    REGISTERED.add(name)
    return name
