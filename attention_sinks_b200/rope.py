"""RoPE helpers in the Transformers (Llama / Qwen) half-split convention.

Dimension i of a head of size d pairs with i + d/2 and the pair is rotated by
pos * inv_freq[i]:  rope(x, p) = x * cos(p * theta) + rotate_half(x) * sin(p * theta).
Rotations compose by adding angles, so a key rotated at position p and then by -delta is
the key rotated at p - delta: that is what lets the sink cache move kept keys to new
positions after an eviction (src/sinkcache/rope.py:1-14).

These are the host-side helpers of the package: `rope_cos_sin` builds the fp32 cos/sin
tables the eviction kernel consumes (one [head_dim] table per shift), exactly as
src/sinkcache/rope.py:24-28 does; `apply_rope` / `rerotate` keep the reference's public
helpers (src/sinkcache/rope.py:43-54) for users and tests.
"""

import torch


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """(x1, x2) -> (-x2, x1) over the last dim (src/sinkcache/rope.py:19-21)."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin of shape [..., rot_dim] for integer positions, as HF computes them
    (src/sinkcache/rope.py:24-28): angles = position * inv_freq in fp32, both halves equal."""
    freqs = positions.to(torch.float32)[..., None] * inv_freq.to(torch.float32)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate the first cos.shape[-1] dims of x in fp32, round once to x.dtype
    (src/sinkcache/rope.py:31-40)."""
    rot_dim = cos.shape[-1]
    xf = x.to(torch.float32)
    x_rot, x_pass = xf[..., :rot_dim], xf[..., rot_dim:]
    out = x_rot * cos + rotate_half(x_rot) * sin
    if x_pass.shape[-1]:
        out = torch.cat((out, x_pass), dim=-1)
    return out.to(x.dtype)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    """Rotate x [batch, heads, seq, head_dim] at `positions` [seq] (src/sinkcache/rope.py:43-46)."""
    cos, sin = rope_cos_sin(positions.to(x.device), inv_freq.to(x.device))
    return _rotate(x, cos, sin)


def rerotate(keys: torch.Tensor, delta: int, inv_freq: torch.Tensor) -> torch.Tensor:
    """Shift already-rotated keys `delta` positions earlier: a rotation by -delta
    (src/sinkcache/rope.py:49-54)."""
    cos, sin = rope_cos_sin(torch.tensor(-delta, device=keys.device), inv_freq.to(keys.device))
    return _rotate(keys, cos, sin)
