"""Helpers shared by the tests."""

import hashlib

import torch


def digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (bf16 viewed as int16), the fixture's exactness check."""
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()


def ulp_tol(dtype: torch.dtype) -> float:
    """One output rounding, relative (tests/test_cache.py:149-152 of the reference)."""
    return 2 ** -7 if dtype == torch.bfloat16 else 2 ** -22


def assert_within_rounding(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype) -> None:
    got, want = got.float().cpu(), want.float().cpu()
    u = ulp_tol(dtype)
    torch.testing.assert_close(got, want, rtol=u, atol=u * want.abs().max().item())
