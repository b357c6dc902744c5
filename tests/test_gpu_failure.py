"""Failure detection on the device, without faulting it: a bounded mbarrier wait that a test
makes run out.  The library's test hook (sink_debug_fail_next_wait) makes the next
stream-kernel launch leave one row chunk of every split unissued -- no copy, no arrival --
with every wait of that launch bounded to a few thousand polls.  The wait for that chunk
runs out, the CTAs wait for the copies they did issue, store nothing further and set
SINK_STATUS_WAIT_TIMEOUT; the host reads the status word (read_status) or raises
(Workspace.check / SinkCache.check_status).  The context stays usable: the next normal
launch on the same (restored) buffers matches the oracle bit for bit.

The reference has no device-side failure detection (it records out-of-memory failures
only, experiments/ppl.py:76-78)."""

import pytest
import torch

import oracle
from attention_sinks_b200 import SinkLayer, _lib, flash_decode
from attention_sinks_b200.decode_attention import _workspace_for
from tests.golden import cases
from tests.util import digest

pytestmark = pytest.mark.gpu
DEV = "cuda"
POLLS = 4096


@pytest.mark.parametrize("slots,streams,clustered", [(4096, 8, False), (1024, 1, True)],
                         ids=["split_launch", "clustered_launch"])
def test_fused_step_wait_runs_out_and_is_reported(slots, streams, clustered, built_lib):
    spec = dict(batch=streams, hq=16, hkv=8, d=128, slots=slots, n_sink=4)
    plan = _lib.plan(_lib.OP_FUSED_STEP, streams, 8, 16, 128, torch.float32, torch.bfloat16, slots + 1, 4,
                     slots - 4, 1, _lib.sm_count(torch.device(DEV)))
    assert (plan["cluster_ctas"] > 1) == clustered
    assert plan["rows_per_split"] // plan["chunk_rows"] >= 2  # chunk 1 exists in every split but the last
    st = cases.step_inputs(**spec)
    k0, v0 = st["k0"].float().to(DEV), st["v0"].to(DEV)
    k1, v1, q = st["k1"].to(DEV), st["v1"].to(DEV), st["q"].to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), st["inv"])]
    out = torch.empty(streams, 1, 16, 128, dtype=torch.bfloat16, device=DEV)
    ws = _lib.Workspace()

    def step(kbuf, vbuf):
        _lib.fused_decode_step(kbuf, vbuf, k1, v1, q, 4, slots - 4, 1, slots, cos, sin, 128 ** -0.5, out, ws)

    kbuf, vbuf = k0.clone(), v0.clone()
    _lib.fail_next_wait(1, POLLS)
    step(kbuf, vbuf)
    torch.cuda.synchronize()
    assert ws.read_status() == _lib.STATUS_WAIT_TIMEOUT
    assert ws.read_status() == 0  # read_status clears the word

    kbuf, vbuf = k0.clone(), v0.clone()
    _lib.fail_next_wait(1, POLLS)
    step(kbuf, vbuf)
    with pytest.raises(RuntimeError, match="bounded wait"):
        ws.check()

    # the context is usable: a normal step on restored buffers matches the oracle
    want = oracle.OracleSinkLayer(4, slots - 4, st["inv"])
    want.update(st["k0"], st["v0"])
    want_out = oracle.decode_step(want, st["q"], st["k1"], st["v1"], 128 ** -0.5)
    kbuf, vbuf = k0.clone(), v0.clone()
    step(kbuf, vbuf)
    ws.check()
    torch.testing.assert_close(vbuf.cpu(), want.vbuf, rtol=0, atol=0)
    assert digest(kbuf.cpu()) == digest(want.kbuf)
    torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)


def test_attention_wait_runs_out_and_leaves_the_cache_untouched(built_lib):
    """Attention only (fp32 keys, the stream kernel): a failed launch reads, never writes, so
    the next normal call on the same buffers is exact."""
    g = torch.Generator().manual_seed(31)
    b, hq, hkv, d, rows = 4, 16, 8, 128, 6000
    q = torch.randn(b, hq, 1, d, generator=g).bfloat16()
    k = torch.randn(b, hkv, rows, d, generator=g) * 3
    v = torch.randn(b, hkv, rows, d, generator=g).bfloat16()
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    _lib.fail_next_wait(2, POLLS)
    flash_decode(qd, kd, vd, d ** -0.5)
    with pytest.raises(RuntimeError, match="bounded wait"):
        _workspace_for(qd.device).check()
    assert torch.equal(kd.cpu(), k) and torch.equal(vd.cpu(), v)
    got = flash_decode(qd, kd, vd, d ** -0.5)
    _workspace_for(qd.device).check()
    torch.testing.assert_close(got.float().cpu(), oracle.decode_attention(q, k, v, d ** -0.5), rtol=2e-2, atol=1e-2)


def test_cache_check_status_raises_after_a_failed_step(built_lib):
    """The cache-level check: a SinkLayer's fused step whose wait ran out makes
    SinkCache-style status checks raise (the layer's workspace is the cache's)."""
    ws = _lib.Workspace()
    layer = SinkLayer(4, 2044, cases.inv_freq(128, 1e6), key_dtype=torch.float32, fused=True, workspace=ws)
    g = torch.Generator(device=DEV).manual_seed(3)
    layer.update(torch.randn(2, 8, 2049, 128, device=DEV, generator=g).bfloat16(),
                 torch.randn(2, 8, 2049, 128, device=DEV, generator=g).bfloat16())
    k = torch.randn(2, 8, 1, 128, device=DEV, generator=g).bfloat16()
    q = torch.randn(2, 16, 1, 128, device=DEV, generator=g).bfloat16()
    layer.update(k, k)
    _lib.fail_next_wait(1, POLLS)
    layer.run_pending(q, 128 ** -0.5)
    with pytest.raises(RuntimeError, match="void"):
        ws.check()
    ws.check()  # the word was cleared by the check that raised
