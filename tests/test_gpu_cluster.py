"""The clustered stream-kernel launch (small states: every split of a (batch, kv-head) pair in
one thread-block cluster, halo rows staged in shared memory behind a cluster barrier, split
partials merged through distributed shared memory) against the oracle: fused steps over
3-16 splits for head_dim 64/128/256 and GQA groups 1-8, shifts of 1-4 rows (clustered) and
5 rows (halo pre-pass), attention alone over fp32 keys, boolean masks, and a stream of
steps.  Each case first checks that the plan takes the regime it is meant to cover."""

import pytest
import torch

import oracle
from attention_sinks_b200 import _lib
from tests.golden import cases
from tests.test_gpu_kernels import _masked_oracle, _status_clean
from tests.util import assert_within_rounding, digest

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cluster(op, batch, hkv, hq, d, kdt, vdt, rows, n_sink, window, drop):
    p = _lib.plan(op, batch, hkv, hq, d, kdt, vdt, rows, n_sink, window, drop,
                  _lib.sm_count(torch.device(DEV)))
    return p["cluster_ctas"], p["splits"]


@pytest.mark.parametrize("batch,hq,hkv,d,slots,n_sink,vdt", [
    (1, 16, 8, 128, 64, 4, torch.bfloat16),
    (1, 16, 8, 128, 256, 4, torch.bfloat16),
    (1, 16, 8, 128, 1024, 4, torch.bfloat16),
    (2, 16, 8, 128, 2047, 4, torch.bfloat16),
    (8, 16, 8, 128, 1024, 4, torch.bfloat16),
    (2, 32, 8, 64, 700, 4, torch.bfloat16),
    (3, 24, 3, 256, 200, 2, torch.float16),
    (2, 8, 8, 128, 333, 0, torch.bfloat16),
    (1, 64, 8, 128, 2047, 4, torch.bfloat16),  # GQA group 8: one CTA per SM, a 16-CTA cluster
])
def test_clustered_fused_step(batch, hq, hkv, d, slots, n_sink, vdt, built_lib):
    """One steady decode step on a clustered launch: cache bit for bit, output within 2e-2."""
    ctas, ns = _cluster(_lib.OP_FUSED_STEP, batch, hkv, hq, d, torch.float32, vdt, slots + 1, n_sink,
                        slots - n_sink, 1)
    assert ctas == ns > 1
    st = cases.step_inputs(batch, hq, hkv, d, slots, n_sink, seed=slots + d)
    k0, v0, k1, v1, q = (st[n].to(vdt) for n in ("k0", "v0", "k1", "v1", "q"))
    want = oracle.OracleSinkLayer(n_sink, slots - n_sink, st["inv"])
    want.update(k0, v0)
    want_out = oracle.decode_step(want, q, k1, v1, d ** -0.5)
    kbuf, vbuf = k0.float().to(DEV), v0.to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), st["inv"])]
    out = torch.empty(batch, 1, hq, d, dtype=vdt, device=DEV)
    ws = _lib.Workspace()
    _lib.fused_decode_step(kbuf, vbuf, k1.to(DEV), v1.to(DEV), q.to(DEV), n_sink, slots - n_sink, 1, slots,
                           cos, sin, d ** -0.5, out, ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    torch.testing.assert_close(vbuf.cpu(), want.vbuf, rtol=0, atol=0)
    assert digest(kbuf.cpu()) == digest(want.kbuf)
    torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("drop", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("window", [100, 1000])
def test_clustered_eviction_by_drop(drop, window, built_lib):
    """Shifts of up to 4 rows stage their halo rows in shared memory (clustered); 5 rows
    take the halo pre-pass.  V bit-exact, K within one rounding of the oracle."""
    batch, heads, n_sink, d = 2, 8, 4, 128
    ctas, ns = _cluster(_lib.OP_EVICT, batch, heads, heads, d, torch.float32, torch.bfloat16, 0, n_sink,
                        window, drop)
    assert ns > 1 and (ctas == ns) == (drop <= 4)
    g = torch.Generator().manual_seed(window + drop)
    inv = cases.inv_freq(d, 1e6)
    rows = n_sink + window + drop
    k = torch.randn(batch, heads, rows + 2, d, generator=g) * 10
    v = torch.randn(batch, heads, rows + 2, d, generator=g).bfloat16()
    want = oracle.OracleSinkLayer(n_sink, window, inv)
    want.dtype = torch.bfloat16
    want.kbuf, want.vbuf, want.length = k.clone(), v.clone(), rows
    want.evict_pending()
    cos, sin = oracle.rope_cos_sin(torch.tensor(-drop), inv)
    kbuf, vbuf = k.to(DEV), v.to(DEV)
    ws = _lib.Workspace()
    _lib.evict_rerotate(kbuf, vbuf, n_sink, window, drop, cos.to(DEV), sin.to(DEV), ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    cap = n_sink + window
    torch.testing.assert_close(vbuf[:, :, :cap].cpu(), want.vbuf[:, :, :cap], rtol=0, atol=0)
    assert_within_rounding(kbuf[:, :, :cap].cpu(), want.kbuf[:, :, :cap], torch.float32)
    torch.testing.assert_close(kbuf[:, :, cap:].cpu(), k[:, :, cap:], rtol=0, atol=0)


@pytest.mark.parametrize("batch,hq,hkv,d,rows", [(1, 16, 8, 128, 300), (1, 8, 8, 64, 2000),
                                                (4, 64, 8, 128, 1000), (2, 16, 2, 256, 150)])
def test_clustered_attention_fp32_keys(batch, hq, hkv, d, rows, built_lib):
    """Attention alone over fp32 keys (drop 0): partials merged across the cluster."""
    ctas, ns = _cluster(_lib.OP_ATTEND, batch, hkv, hq, d, torch.float32, torch.bfloat16, rows, 0, 1, 0)
    assert ctas == ns > 1
    g = torch.Generator().manual_seed(rows + hq)
    q = torch.randn(batch, hq, 1, d, generator=g).bfloat16()
    k = torch.randn(batch, hkv, rows + 5, d, generator=g) * 3
    v = torch.randn(batch, hkv, rows + 5, d, generator=g).bfloat16()
    out = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    ws = _lib.Workspace()
    _lib.decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), rows, d ** -0.5, out, ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    want = oracle.decode_attention(q, k[:, :, :rows], v[:, :, :rows], d ** -0.5)
    torch.testing.assert_close(out.float().cpu(), want, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("mask_batch", [1, 2])
def test_clustered_fused_step_with_mask(mask_batch, built_lib):
    """Masked rows on a clustered launch, including a split whose rows are all masked."""
    spec = dict(batch=2, hq=16, hkv=8, d=128, slots=1024, n_sink=4)
    n_sink, slots = spec["n_sink"], spec["slots"]
    ctas, ns = _cluster(_lib.OP_FUSED_STEP, 2, 8, 16, 128, torch.float32, torch.bfloat16, slots + 1, n_sink,
                        slots - n_sink, 1)
    assert ctas == ns > 2
    st = cases.step_inputs(**spec)
    want = oracle.OracleSinkLayer(n_sink, slots - n_sink, st["inv"])
    want.update(st["k0"], st["v0"])
    keys, values = want.update(st["k1"], st["v1"])
    g = torch.Generator().manual_seed(9)
    mask = torch.rand(mask_batch, 1, 1, slots + 1, generator=g) > 0.4
    mask[..., 200:500] = False  # the whole second split, and parts of its neighbours
    mask[..., -1] = True
    want_out = _masked_oracle(st["q"], keys, values, mask, spec["d"] ** -0.5)
    kbuf, vbuf = st["k0"].float().to(DEV), st["v0"].to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), st["inv"])]
    out = torch.empty(2, 1, 16, 128, dtype=torch.bfloat16, device=DEV)
    ws = _lib.Workspace()
    _lib.fused_decode_step(kbuf, vbuf, st["k1"].to(DEV), st["v1"].to(DEV), st["q"].to(DEV), n_sink,
                           slots - n_sink, 1, slots, cos, sin, spec["d"] ** -0.5, out, ws, mask.to(DEV))
    torch.cuda.synchronize()
    _status_clean(ws)
    assert digest(kbuf.cpu()) == digest(want.kbuf)
    torch.testing.assert_close(vbuf.cpu(), want.vbuf, rtol=0, atol=0)
    torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)


def test_clustered_stream_of_steps(built_lib):
    """Fill then evict every step on a clustered plan, the cache bit-exact throughout; the
    plan moves from unclustered (few rows: one split) to clustered as the cache fills."""
    batch, hq, hkv, d, n_sink, window = 2, 16, 8, 128, 4, 508
    g = torch.Generator().manual_seed(21)
    inv = cases.inv_freq(d, 1e6)
    cap = n_sink + window
    assert _cluster(_lib.OP_FUSED_STEP, batch, hkv, hq, d, torch.float32, torch.bfloat16, cap + 1, n_sink,
                    window, 1)[0] > 1
    want = oracle.OracleSinkLayer(n_sink, window, inv)
    kbuf = torch.zeros(batch, hkv, cap + 1, d, device=DEV)
    vbuf = torch.zeros(batch, hkv, cap + 1, d, dtype=torch.bfloat16, device=DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), inv)]
    ws = _lib.Workspace()
    out = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    length = 0
    for step in range(cap + 40):
        k1 = (torch.randn(batch, hkv, 1, d, generator=g) * 2).bfloat16()
        v1 = torch.randn(batch, hkv, 1, d, generator=g).bfloat16()
        q = torch.randn(batch, hq, 1, d, generator=g).bfloat16()
        want_out = oracle.decode_step(want, q, k1, v1, d ** -0.5)
        drop = max(length - cap, 0)
        row = length - drop
        _lib.fused_decode_step(kbuf, vbuf, k1.to(DEV), v1.to(DEV), q.to(DEV), n_sink, window, drop, row,
                               cos if drop else None, sin if drop else None, d ** -0.5, out, ws)
        length = row + 1
        if step % 37 == 0 or step >= cap + 30:
            torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)
            torch.testing.assert_close(vbuf[:, :, :length].cpu(), want.vbuf[:, :, :length], rtol=0, atol=0)
            assert digest(kbuf[:, :, :length].cpu()) == digest(want.kbuf[:, :, :length])
    _status_clean(ws)
