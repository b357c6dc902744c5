"""sink_decode_attention_noalloc: decode attention for callers that cannot allocate device
memory -- a host that binds the C ABI from a runtime without a device allocator, or a
decode loop that must not call cudaMalloc / cudaFree because they synchronise the device.
Its split partials live in the library's static 16 MiB device array instead of a
caller-provided workspace.  Its output must match sink_decode_attention's (same kernels,
same plan) on consecutive calls that reuse the shared array, and a request larger than the
array must be refused before anything is launched.

This file is collected last on purpose, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""

import pytest
import torch

from attention_sinks_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(batch, hq, hkv, d, rows, kdt, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, hq, 1, d, generator=g).bfloat16().to(DEV)
    k = (torch.randn(batch, hkv, rows + 7, d, generator=g) * 3).to(kdt).to(DEV)
    v = torch.randn(batch, hkv, rows + 7, d, generator=g).bfloat16().to(DEV)
    return q, k, v


def test_noalloc_matches_workspace_entry_point(built_lib):
    """Two different calls in a row through the C ABI, each against the workspace entry
    point on the same inputs (tolerance of the decode-attention tests)."""
    cases = [(2, 16, 8, 128, 1500, torch.float32, 1), (3, 32, 8, 64, 777, torch.bfloat16, 2),
             (2, 16, 8, 128, 1500, torch.float32, 3)]
    for batch, hq, hkv, d, rows, kdt, seed in cases:
        q, k, v = _inputs(batch, hq, hkv, d, rows, kdt, seed)
        scale = d ** -0.5
        want = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
        _lib.decode_attention(q, k, v, rows, scale, want, _lib.Workspace())
        got = torch.full_like(want, float("nan"))
        rc = _lib.decode_attention_noalloc(q, k, v, rows, scale, got)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=1e-2)


def test_noalloc_refuses_requests_beyond_its_scratch(built_lib):
    # 16 streams x 8 kv heads with groups of 8 query heads at head_dim 256 need more split
    # partials than the static array holds
    batch, hkv, hq, d, rows = 16, 8, 64, 256, 4097
    need = _lib.workspace_bytes(_lib.OP_ATTEND, batch, hkv, hq, d, torch.float32, torch.bfloat16, rows, 0, 1, 0,
                                _lib.sm_count(torch.device(DEV)))
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    k = torch.zeros(batch, hkv, rows, d, dtype=torch.float32, device=DEV)
    v = torch.zeros(batch, hkv, rows, d, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(batch, hq, 1, d, dtype=torch.bfloat16, device=DEV)
    out = torch.full((batch, 1, hq, d), 7.0, dtype=torch.bfloat16, device=DEV)
    rc = _lib.decode_attention_noalloc(q, k, v, rows, 0.0625, out)
    assert rc == _lib.ESCRATCH
    assert "16 MiB" in _lib.strerror(rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing was launched
