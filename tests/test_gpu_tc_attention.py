"""Decode attention on the tensor-core kernel (sink_attend_tc_kernel: tcgen05 MMAs, TMA tiles,
TMEM accumulators), taken for 16-bit K = V dtype with head_dim 128: against the fp32 oracle
over GQA groups 1-8, bf16 and fp16, row counts around the 128-row chunk, one and many
splits, strided views and boolean masks."""

import pytest
import torch

import oracle
from attention_sinks_b200 import _lib
from tests.test_gpu_kernels import _masked_oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(q, k, v, rows, scale, mask=None):
    b, hq, _, d = q.shape
    out = torch.empty(b, 1, hq, d, dtype=q.dtype, device=DEV)
    ws = _lib.Workspace()
    _lib.decode_attention(q.to(DEV), k, v, rows, scale, out, ws, mask)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    return out.float().cpu()


def test_plan_takes_the_tensor_core_kernel():
    bf = torch.bfloat16
    p = _lib.plan(_lib.OP_ATTEND, 64, 8, 16, 128, bf, bf, 32769, 0, 1, 0, 148)
    assert p["chunk_rows"] == 128 and p["stages"] == 3 and p["smem_bytes"] <= 227 * 1024
    assert p["rows_per_split"] % 128 == 0
    # fp32 keys, head_dim 64 or mixed types stay on the CUDA-core stream kernel
    assert _lib.plan(_lib.OP_ATTEND, 1, 8, 16, 128, torch.float32, bf, 1025, 0, 1, 0, 148)["chunk_rows"] == 32
    assert _lib.plan(_lib.OP_ATTEND, 1, 8, 16, 64, bf, bf, 1025, 0, 1, 0, 148)["chunk_rows"] == 64


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 8), (14, 2), (64, 8)])
@pytest.mark.parametrize("rows", [1, 100, 128, 129, 1000, 4097, 32769])
@pytest.mark.parametrize("batch", [1, 5])
def test_tensor_core_attention_matches_oracle(dtype, hq, hkv, rows, batch):
    if batch * hkv * rows > 5 * 8 * 4097 and rows > 4097 and batch > 1:
        pytest.skip("large case covered at batch 1")
    g = torch.Generator().manual_seed(rows * 7 + hq + batch)
    d = 128
    q = torch.randn(batch, hq, 1, d, generator=g).to(dtype)
    k = (torch.randn(batch, hkv, rows + 3, d, generator=g) * 3).to(dtype)
    v = torch.randn(batch, hkv, rows + 3, d, generator=g).to(dtype)
    got = _run(q, k.to(DEV), v.to(DEV), rows, d ** -0.5)
    want = oracle.decode_attention(q, k[:, :, :rows], v[:, :, :rows], d ** -0.5)
    torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-2)


def test_tensor_core_attention_strided_heads():
    """A slot-prefix view of a larger buffer: per-head stride larger than rows * D."""
    g = torch.Generator().manual_seed(5)
    buf_k = (torch.randn(3, 8, 2000, 128, generator=g) * 3).bfloat16().to(DEV)
    buf_v = torch.randn(3, 8, 2000, 128, generator=g).bfloat16().to(DEV)
    q = torch.randn(3, 16, 1, 128, generator=g).bfloat16()
    got = _run(q, buf_k[:, :, :1500], buf_v[:, :, :1500], 1500, 0.07)
    want = oracle.decode_attention(q, buf_k[:, :, :1500].cpu(), buf_v[:, :, :1500].cpu(), 0.07)
    torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("mask_batch", [1, 3])
def test_tensor_core_attention_boolean_mask(mask_batch):
    g = torch.Generator().manual_seed(22)
    b, hq, hkv, d, rows = 3, 16, 8, 128, 2100
    q = torch.randn(b, hq, 1, d, generator=g).bfloat16()
    k = (torch.randn(b, hkv, rows, d, generator=g) * 3).bfloat16()
    v = torch.randn(b, hkv, rows, d, generator=g).bfloat16()
    mask = torch.rand(mask_batch, 1, 1, rows, generator=g) > 0.3
    mask[..., 0] = True
    got = _run(q, k.to(DEV), v.to(DEV), rows, d ** -0.5, mask.to(DEV))
    want = _masked_oracle(q, k, v, mask, d ** -0.5)
    torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-2)
    ones = torch.ones(1, 1, 1, rows, dtype=torch.bool, device=DEV)
    torch.testing.assert_close(_run(q, k.to(DEV), v.to(DEV), rows, d ** -0.5, ones),
                               _run(q, k.to(DEV), v.to(DEV), rows, d ** -0.5), rtol=0, atol=0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
def test_tensor_core_attention_running_max_jumps(dtype):
    """Scores that grow by far more than 2^8 (log2 units) from chunk to chunk within a split:
    the output accumulator is rescaled in TMEM each time the reference max moves."""
    g = torch.Generator().manual_seed(31)
    b, hq, hkv, d, rows = 2, 16, 8, 128, 5000
    q = torch.randn(b, hq, 1, d, generator=g).to(dtype)
    k = torch.randn(b, hkv, rows, d, generator=g) * 0.5
    for i, row in enumerate((700, 1500, 2600, 3900, 4999)):  # aligned keys, growing scores
        k[:, :, row] = (i + 1) * 1.5 * q.float().view(b, hkv, hq // hkv, d).mean(2)
    k = k.to(dtype)
    v = torch.randn(b, hkv, rows, d, generator=g).to(dtype)
    got = _run(q, k.to(DEV), v.to(DEV), rows, d ** -0.5)
    want = oracle.decode_attention(q, k, v, d ** -0.5)
    torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-2)
