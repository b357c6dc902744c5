"""sink_decode_attention_noalloc: decode attention for callers that cannot allocate device
memory -- a host that binds the C ABI from a runtime without a device allocator, or a
decode loop that must not call cudaMalloc / cudaFree because they synchronise the device.
Its split partials live in the library's static 16 MiB device array instead of a
caller-provided workspace.  Same plan and kernels as sink_decode_attention, so its output
must equal that entry point's bit for bit, on consecutive calls that reuse the shared
array; a bad request must get the same error code, and a request larger than the array
must be refused before anything is launched.

This file is collected last on purpose, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process."""

import ctypes

import pytest
import torch

import oracle
from attention_sinks_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(batch, hq, hkv, d, rows, kdt, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, hq, 1, d, generator=g).bfloat16().to(DEV)
    k = (torch.randn(batch, hkv, rows + 7, d, generator=g) * 3).to(kdt).to(DEV)
    v = torch.randn(batch, hkv, rows + 7, d, generator=g).bfloat16().to(DEV)
    return q, k, v


# (batch, hq, hkv, d, rows, key dtype, seed, masked): the stream kernel over fp32 keys and
# over bf16 keys at head_dim 64, the tensor-core kernel (bf16 keys, head_dim 128) with
# several splits, and a boolean mask
CASES = [(2, 16, 8, 128, 1500, torch.float32, 1, False),
         (3, 32, 8, 64, 777, torch.bfloat16, 2, False),
         (2, 16, 8, 128, 9000, torch.bfloat16, 3, False),
         (3, 16, 8, 128, 2100, torch.float32, 4, True),
         (2, 16, 8, 128, 1500, torch.float32, 1, False)]


def _mask(batch, rows, seed):
    g = torch.Generator().manual_seed(seed)
    m = torch.rand(batch, 1, 1, rows, generator=g) > 0.3
    m[..., 0] = True
    return m.to(DEV)


def test_noalloc_equals_workspace_entry_point(built_lib):
    """Calls in a row through the C ABI, each bit-identical to the workspace entry point on
    the same inputs, and within the decode-attention tolerance of fp32 attention."""
    dev = torch.device(DEV)
    sms = _lib.sm_count(dev)
    saw_tc_split = False
    for batch, hq, hkv, d, rows, kdt, seed, masked in CASES:
        q, k, v = _inputs(batch, hq, hkv, d, rows, kdt, seed)
        plan = _lib.plan(_lib.OP_ATTEND, batch, hkv, hq, d, kdt, torch.bfloat16, rows, 0, 1, 0, sms)
        saw_tc_split |= kdt == torch.bfloat16 and d == 128 and plan["splits"] > 1
        mask = _mask(batch, rows, seed) if masked else None
        scale = d ** -0.5
        want = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
        _lib.decode_attention(q, k, v, rows, scale, want, _lib.Workspace(), mask)
        got = torch.full_like(want, float("nan"))
        rc = _lib.decode_attention_noalloc(q, k, v, rows, scale, got, mask)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, want, rtol=0, atol=0)
        qc, kc, vc = q.cpu(), k[:, :, :rows].cpu(), v[:, :, :rows].cpu()
        if masked:
            ref = torch.cat([oracle.decode_attention(qc[b:b + 1], kc[b:b + 1, :, mask[b, 0, 0].cpu()],
                                                     vc[b:b + 1, :, mask[b, 0, 0].cpu()], scale)
                             for b in range(batch)])
        else:
            ref = oracle.decode_attention(qc, kc, vc, scale)
        torch.testing.assert_close(got.float().cpu(), ref, rtol=2e-2, atol=1e-2)
    assert saw_tc_split


def test_noalloc_allocates_nothing(built_lib):
    """After the first call, further calls leave the device's free memory unchanged."""
    batch, hq, hkv, d, rows = 2, 16, 8, 128, 9000
    q, k, v = _inputs(batch, hq, hkv, d, rows, torch.bfloat16, 9)
    out = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    assert _lib.decode_attention_noalloc(q, k, v, rows, d ** -0.5, out) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        assert _lib.decode_attention_noalloc(q, k, v, rows, d ** -0.5, out) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def _raw_codes(q, k, v, rows, out):
    """Return codes of both entry points for the same (possibly bad) request."""
    kv = _lib.kv_desc(k, v)
    qd = _lib.rows_desc(q)
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=DEV)
    st = _lib.stream_handle(k.device)
    a = _lib.lib().sink_decode_attention(ctypes.byref(qd), ctypes.byref(kv), rows, 0.1, None, 0, out.data_ptr(),
                                         out.stride(0), out.stride(2), ws.data_ptr(), ws.numel(), st)
    b = _lib.lib().sink_decode_attention_noalloc(ctypes.byref(qd), ctypes.byref(kv), rows, 0.1, None, 0,
                                                 out.data_ptr(), out.stride(0), out.stride(2), st)
    return a, b


def test_noalloc_bad_requests_get_the_same_codes(built_lib):
    q, k, v = _inputs(1, 16, 8, 128, 100, torch.float32, 5)
    out = torch.full((1, 1, 16, 128), 3.0, dtype=torch.bfloat16, device=DEV)
    a, b = _raw_codes(q, k, v, k.shape[2] + 1, out)  # more rows than the buffers hold
    assert a == b == _lib.EINVAL
    a, b = _raw_codes(q.half(), k, v, 100, out)  # query dtype != value dtype
    assert a == b == _lib.EDTYPE
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())


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
