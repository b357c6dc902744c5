"""The sm_100a kernels against the CPU oracle and the reference's golden outputs.

Tolerances are the reference tests': eviction V bit-exact and K within one rounding
(tests/test_cache.py:130-152); decode attention rtol 2e-2 / atol 1e-2 against an fp32
reference (tests/test_decode_attention.py:23-41).  The re-rotation reproduces the
reference CPU path's arithmetic (fp32 mul, then a fused multiply-add), so K is also
checked bit for bit against the reference's recorded output."""

import pytest
import torch

import oracle
from attention_sinks_b200 import _lib, flash_decode
from tests.golden import cases
from tests.util import assert_within_rounding, digest

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _status_clean(ws):
    assert ws.read_status() == 0, "a kernel's bounded wait ran out"


@pytest.mark.parametrize("case", cases.EVICT_CASES, ids=lambda c: cases.evict_name(*c))
def test_eviction_matches_reference(case, golden, built_lib):
    """Fused in-place shift + re-rotation == the reference PyTorch path, including drops
    larger than a chunk and windows smaller than one (test_cache.py:130-152)."""
    dtype_name, n_sink, window, drop = case
    k, v, inv = cases.evict_inputs(*case)
    want = oracle.OracleSinkLayer(n_sink, window, inv, key_dtype=None)
    want.update(k, v)
    want.evict_pending()
    cap = n_sink + window
    kbuf, vbuf = k.to(DEV), v.to(DEV)
    cos, sin = oracle.rope_cos_sin(torch.tensor(-drop), inv)
    ws = _lib.Workspace()
    _lib.evict_rerotate(kbuf, vbuf, n_sink, window, drop, cos.to(DEV), sin.to(DEV), ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    kf, vf = kbuf[:, :, :cap].cpu(), vbuf[:, :, :cap].cpu()
    torch.testing.assert_close(vf, want.vbuf[:, :, :cap], rtol=0, atol=0)
    assert_within_rounding(kf, want.kbuf[:, :, :cap], k.dtype)
    gold = golden["evict"][cases.evict_name(*case)]
    if digest(k) == gold["in_k"]:
        assert digest(kf) == gold["k"], "re-rotated keys differ from the reference's bits"
        assert digest(vf) == gold["v"]
    # rows past the window are untouched
    torch.testing.assert_close(kbuf[:, :, cap:].cpu(), k[:, :, cap:], rtol=0, atol=0)


@pytest.mark.parametrize("batch,heads,n_sink,window,drop,kdt,vdt", [
    (3, 8, 4, 1020, 1, torch.float32, torch.bfloat16),
    (2, 8, 4, 4092, 1, torch.float32, torch.bfloat16),
    (1, 8, 4, 32764, 1, torch.float32, torch.bfloat16),
    (4, 2, 0, 300, 33, torch.float32, torch.float16),
    (2, 4, 4, 100, 250, torch.float32, torch.float32),
    (2, 8, 3, 513, 7, torch.bfloat16, torch.bfloat16),
])
def test_eviction_shapes(batch, heads, n_sink, window, drop, kdt, vdt, built_lib):
    """Multi-split shifts (halo rows across split boundaries), batch/head strides, dtypes."""
    d = 128 if vdt != torch.float32 else 64
    g = torch.Generator().manual_seed(batch * 1000 + drop)
    inv = cases.inv_freq(d, 1e6)
    rows = n_sink + window + drop
    k = (torch.randn(batch, heads, rows + 3, d, generator=g) * 10).to(kdt)
    v = torch.randn(batch, heads, rows + 3, d, generator=g).to(vdt)
    want = oracle.OracleSinkLayer(n_sink, window, inv, key_dtype=kdt)
    want.dtype = vdt
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
    assert_within_rounding(kbuf[:, :, :cap].cpu(), want.kbuf[:, :, :cap], kdt)
    torch.testing.assert_close(kbuf.cpu()[:, :, cap:], k[:, :, cap:], rtol=0, atol=0)


def test_eviction_without_rotation(built_lib):
    """rerotate_keys=False: the window shifts, keys keep their stale rotation."""
    k = torch.randn(2, 8, 70, 128)
    v = torch.randn(2, 8, 70, 128).bfloat16()
    kbuf, vbuf = k.to(DEV), v.to(DEV)
    _lib.evict_rerotate(kbuf, vbuf, 4, 60, 5, None, None, _lib.Workspace())
    torch.testing.assert_close(kbuf[:, :, 4:64].cpu(), k[:, :, 9:69], rtol=0, atol=0)
    torch.testing.assert_close(vbuf[:, :, 4:64].cpu(), v[:, :, 9:69], rtol=0, atol=0)
    torch.testing.assert_close(kbuf[:, :, :4].cpu(), k[:, :, :4], rtol=0, atol=0)


@pytest.mark.parametrize("shape", cases.ATTN_SHAPES, ids=lambda s: "_".join(map(str, s)))
@pytest.mark.parametrize("seq_len", cases.ATTN_LENS)
def test_flash_decode_matches_reference(shape, seq_len, golden_arrays, built_lib):
    """bf16 K/V, the shapes of test_decode_attention.py:23-31, against the fp32 oracle and
    the reference's recorded CPU output."""
    hq, hkv, d = shape
    q, k, v = cases.attn_inputs(hq, hkv, d, seq_len)
    got = flash_decode(q.to(DEV), k.to(DEV), v.to(DEV), d ** -0.5).float().cpu()
    torch.testing.assert_close(got, oracle.decode_attention(q, k, v, d ** -0.5), rtol=2e-2, atol=1e-2)
    ref = torch.from_numpy(golden_arrays[f"attn_{hq}_{hkv}_{d}_{seq_len}"])
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=1e-2)


def test_flash_decode_strided_view(built_lib):
    """A view into a larger buffer, non-contiguous over heads (test_decode_attention.py:34-41)."""
    g = torch.Generator().manual_seed(3)
    buf_k = torch.randn(2, 8, 1100, 128, generator=g).bfloat16()
    buf_v = torch.randn(2, 8, 1100, 128, generator=g).bfloat16()
    q = torch.randn(2, 16, 1, 128, generator=g).bfloat16()
    k, v = buf_k[:, :, :1025], buf_v[:, :, :1025]
    got = flash_decode(q.to(DEV), buf_k.to(DEV)[:, :, :1025], buf_v.to(DEV)[:, :, :1025], 0.088)
    torch.testing.assert_close(got.float().cpu(), oracle.decode_attention(q, k, v, 0.088), rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("batch,hq,hkv,d,rows", [(1, 16, 8, 128, 1025), (8, 16, 8, 128, 4097),
                                                (3, 32, 8, 64, 777), (2, 64, 8, 128, 300)])
def test_decode_attention_fp32_keys(batch, hq, hkv, d, rows, built_lib):
    """float32 key storage read directly (no bf16 copy of the cache)."""
    g = torch.Generator().manual_seed(rows)
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


@pytest.mark.parametrize("spec", cases.STEP_CASES, ids=lambda s: cases.step_name(**s))
def test_fused_step_matches_reference(spec, golden, golden_arrays, built_lib):
    """One fused decode step (evict + re-rotate + append + attend) == SinkLayer.update then
    attention on the reference's CPU path: cache contents bit for bit, output within 2e-2."""
    name = cases.step_name(**spec)
    st = cases.step_inputs(**spec)
    n_sink, slots = spec["n_sink"], spec["slots"]
    want = oracle.OracleSinkLayer(n_sink, slots - n_sink, st["inv"])
    want.update(st["k0"], st["v0"])
    want_out = oracle.decode_step(want, st["q"], st["k1"], st["v1"], spec["d"] ** -0.5)

    kbuf = st["k0"].float().to(DEV)
    vbuf = st["v0"].to(DEV)
    cos, sin = oracle.rope_cos_sin(torch.tensor(-1), st["inv"])
    out = torch.empty(spec["batch"], 1, spec["hq"], spec["d"], dtype=torch.bfloat16, device=DEV)
    ws = _lib.Workspace()
    _lib.fused_decode_step(kbuf, vbuf, st["k1"].to(DEV), st["v1"].to(DEV), st["q"].to(DEV), n_sink,
                           slots - n_sink, 1, slots, cos.to(DEV), sin.to(DEV), spec["d"] ** -0.5, out, ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    torch.testing.assert_close(vbuf.cpu(), want.vbuf, rtol=0, atol=0)
    assert_within_rounding(kbuf.cpu(), want.kbuf, torch.float32)
    assert digest(kbuf.cpu()) == golden["step"][name]["k"]
    torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(golden_arrays[name + "/out"]),
                               rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("batch,hq,hkv,d,n_sink,window,steps", [
    (2, 16, 8, 128, 4, 60, 90), (1, 32, 8, 64, 4, 1020, 40), (3, 16, 8, 128, 0, 33, 50),
    (1, 16, 8, 128, 4, 1020, 12),
])
def test_fused_stream_matches_oracle(batch, hq, hkv, d, n_sink, window, steps, built_lib):
    """Many fused steps in a row, filling the cache and then evicting every step, against
    the oracle fed the same tokens: cache bit-exact at every step, outputs within 2e-2.
    One stream at 1,024 slots runs clustered plans of every size while it fills."""
    g = torch.Generator().manual_seed(11)
    inv = cases.inv_freq(d, 1e6)
    cap = n_sink + window
    want = oracle.OracleSinkLayer(n_sink, window, inv)
    prefill = 8
    k0 = (torch.randn(batch, hkv, prefill, d, generator=g) * 2).bfloat16()
    v0 = torch.randn(batch, hkv, prefill, d, generator=g).bfloat16()
    want.update(k0, v0)
    kbuf = torch.zeros(batch, hkv, cap + 1, d, device=DEV)
    vbuf = torch.zeros(batch, hkv, cap + 1, d, dtype=torch.bfloat16, device=DEV)
    kbuf[:, :, :prefill] = k0.float().to(DEV)
    vbuf[:, :, :prefill] = v0.to(DEV)
    length = prefill
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), inv)]
    ws = _lib.Workspace()
    out = torch.empty(batch, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    for step in range(steps + cap):
        k1 = (torch.randn(batch, hkv, 1, d, generator=g) * 2).bfloat16()
        v1 = torch.randn(batch, hkv, 1, d, generator=g).bfloat16()
        q = torch.randn(batch, hq, 1, d, generator=g).bfloat16()
        want_out = oracle.decode_step(want, q, k1, v1, d ** -0.5)
        drop = max(length - cap, 0)
        row = length - drop
        _lib.fused_decode_step(kbuf, vbuf, k1.to(DEV), v1.to(DEV), q.to(DEV), n_sink, window, drop, row,
                               cos if drop else None, sin if drop else None, d ** -0.5, out, ws)
        length = row + 1
        if step % 7 == 0 or step >= steps + cap - 2:
            torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)
            torch.testing.assert_close(vbuf[:, :, :length].cpu(), want.vbuf[:, :, :length], rtol=0, atol=0)
            assert digest(kbuf[:, :, :length].cpu()) == digest(want.kbuf[:, :, :length])
    assert length == cap + 1 and want.tokens_evicted == prefill + steps + cap - (cap + 1)
    _status_clean(ws)


@pytest.mark.parametrize("b,window,launch", [(4, 2044, _lib.LAUNCH_SPLIT), (1, 1020, _lib.LAUNCH_CLUSTER),
                                              (8, 252, _lib.LAUNCH_CLUSTER)])
def test_fused_equals_unfused(b, window, launch, built_lib):
    """The fused step leaves the cache bit-identical to evict + append, and its output equals
    decode attention over the updated cache -- bit for bit, with both on the split launch
    (halo pre-pass, combine) and with both as one clustered launch (merge in the cluster)."""
    g = torch.Generator().manual_seed(5)
    hkv, hq, d, n_sink = 8, 16, 128, 4
    sms = _lib.sm_count(torch.device(DEV))
    for op, rows, drop in ((_lib.OP_FUSED_STEP, n_sink + window + 1, 1), (_lib.OP_ATTEND, n_sink + window + 1, 0)):
        p = _lib.plan(op, b, hkv, hq, d, torch.float32, torch.bfloat16, rows, n_sink, window, drop, sms)
        assert p["launch"] == launch
    inv = cases.inv_freq(d, 1e6)
    k = (torch.randn(b, hkv, n_sink + window + 1, d, generator=g) * 5).to(DEV)
    v = torch.randn(b, hkv, n_sink + window + 1, d, generator=g).bfloat16().to(DEV)
    k1 = torch.randn(b, hkv, 1, d, generator=g).bfloat16().to(DEV)
    v1 = torch.randn(b, hkv, 1, d, generator=g).bfloat16().to(DEV)
    q = torch.randn(b, hq, 1, d, generator=g).bfloat16().to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), inv)]
    ws = _lib.Workspace()
    ka, va = k.clone(), v.clone()
    oa = torch.empty(b, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    _lib.fused_decode_step(ka, va, k1, v1, q, n_sink, window, 1, n_sink + window, cos, sin, d ** -0.5, oa, ws)
    kb, vb = k.clone(), v.clone()
    _lib.evict_rerotate(kb, vb, n_sink, window, 1, cos, sin, ws)
    _lib.append(kb, vb, k1, v1, n_sink + window)
    ob = torch.empty_like(oa)
    _lib.decode_attention(q, kb, vb, n_sink + window + 1, d ** -0.5, ob, ws)
    torch.cuda.synchronize()
    torch.testing.assert_close(ka, kb, rtol=0, atol=0)
    torch.testing.assert_close(va, vb, rtol=0, atol=0)
    torch.testing.assert_close(oa, ob, rtol=0, atol=0)


@pytest.mark.parametrize("op,drop,launches", [("fused", 1, 3), ("fused", 3, 3), ("evict", 2, 2), ("attend", 0, 2)])
def test_cluster_fallback_runs_the_plan_split(op, drop, launches, built_lib):
    """A clustered plan (one stream, 1,024 slots: clusters of 11 or 16 CTAs) on a device that
    cannot place the cluster runs the same splits as a split launch -- halo pre-pass (when
    the window shifts), stream kernel, combine (when it attends) -- with the cache left bit
    for bit as the clustered launch leaves it and outputs equal within 1e-2."""
    g = torch.Generator().manual_seed(11 + drop)
    b, hkv, hq, d, n_sink, window = 1, 8, 16, 128, 4, 1020
    inv = cases.inv_freq(d, 1e6)
    k = (torch.randn(b, hkv, n_sink + window + 4, d, generator=g) * 5).to(DEV)
    v = torch.randn(b, hkv, n_sink + window + 4, d, generator=g).bfloat16().to(DEV)
    k1 = torch.randn(b, hkv, 1, d, generator=g).bfloat16().to(DEV)
    v1 = torch.randn(b, hkv, 1, d, generator=g).bfloat16().to(DEV)
    q = torch.randn(b, hq, 1, d, generator=g).bfloat16().to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-drop), inv)]
    f32, bf = torch.float32, torch.bfloat16
    plans = {"fused": (_lib.OP_FUSED_STEP, hq, n_sink + window + 1), "evict": (_lib.OP_EVICT, hkv, 0),
             "attend": (_lib.OP_ATTEND, hq, n_sink + window)}
    code, heads_q, rows = plans[op]
    p = _lib.plan(code, b, hkv, heads_q, d, f32, bf, rows, n_sink, window, drop, _lib.sm_count(torch.device(DEV)))
    assert p["cluster_ctas"] > 1

    def run(capacity):
        kk, vv = k.clone(), v.clone()
        out = torch.zeros(b, 1, hq, d, dtype=bf, device=DEV)
        ws = _lib.Workspace()
        _lib.force_cluster_capacity(capacity)
        try:
            torch.cuda.synchronize()
            n0 = _lib.launch_count()
            if op == "fused":
                _lib.fused_decode_step(kk, vv, k1, v1, q, n_sink, window, drop, n_sink + window, cos, sin,
                                       d ** -0.5, out, ws)
            elif op == "evict":
                _lib.evict_rerotate(kk, vv, n_sink, window, drop, cos, sin, ws)
            else:
                _lib.decode_attention(q, kk, vv, rows, d ** -0.5, out, ws)
            n = _lib.launch_count() - n0
            torch.cuda.synchronize()
        finally:
            _lib.force_cluster_capacity(-1)
        _status_clean(ws)
        return kk, vv, out, n

    ka, va, oa, na = run(-1)
    kb, vb, ob, nb = run(0)
    assert (na, nb) == (1, launches)
    torch.testing.assert_close(ka, kb, rtol=0, atol=0)
    torch.testing.assert_close(va, vb, rtol=0, atol=0)
    torch.testing.assert_close(oa.float(), ob.float(), rtol=0, atol=1e-2)


@pytest.mark.parametrize("batch,slots,launches", [(1, 256, 1), (8, 256, 1), (1, 1024, 1), (8, 1024, 1),
                                                 (7, 4096, 1), (2, 2047, 3)])
def test_planned_clusters_launch_as_one_wave(batch, slots, launches, built_lib):
    """The small fused steps the planner clusters (clusters of 3 to 16 CTAs, one per (batch,
    head) pair) stay a single launch where the B200 holds all their clusters at once by its
    own count; 16 clusters of 16 CTAs (2,048 slots x 2 streams) do not fit one wave there
    (a cluster must fit one GPC), so that step runs split: halo pre-pass, stream kernel,
    combine."""
    f32, bf = torch.float32, torch.bfloat16
    hkv, hq, d, n_sink, window = 8, 16, 128, 4, slots - 4
    p = _lib.plan(_lib.OP_FUSED_STEP, batch, hkv, hq, d, f32, bf, slots + 1, n_sink, window, 1,
                  _lib.sm_count(torch.device(DEV)))
    assert p["cluster_ctas"] > 1
    g = torch.Generator().manual_seed(slots + batch)
    k = torch.randn(batch, hkv, slots + 1, d, generator=g).to(DEV)
    v = torch.randn(batch, hkv, slots + 1, d, generator=g).bfloat16().to(DEV)
    k1, v1 = [torch.randn(batch, hkv, 1, d, generator=g).bfloat16().to(DEV) for _ in range(2)]
    q = torch.randn(batch, hq, 1, d, generator=g).bfloat16().to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), cases.inv_freq(d, 1e6))]
    out = torch.empty(batch, 1, hq, d, dtype=bf, device=DEV)
    ws = _lib.Workspace()
    n0 = _lib.launch_count()
    _lib.fused_decode_step(k, v, k1, v1, q, n_sink, window, 1, slots, cos, sin, d ** -0.5, out, ws)
    assert _lib.launch_count() - n0 == launches
    _status_clean(ws)


def _masked_oracle(q, k, v, mask, scale):
    """Attention per stream over the rows its boolean mask keeps."""
    outs = []
    for b in range(q.shape[0]):
        keep = mask[min(b, mask.shape[0] - 1), 0, 0]
        outs.append(oracle.decode_attention(q[b:b + 1], k[b:b + 1, :, keep], v[b:b + 1, :, keep], scale))
    return torch.cat(outs, 0)


@pytest.mark.parametrize("mask_batch", [1, 3])
def test_decode_attention_with_boolean_mask(mask_batch, built_lib):
    """A padded batch's boolean [B, 1, 1, L] mask: masked rows get no weight."""
    g = torch.Generator().manual_seed(21)
    b, hq, hkv, d, rows = 3, 16, 8, 128, 2100
    q = torch.randn(b, hq, 1, d, generator=g).bfloat16()
    k = torch.randn(b, hkv, rows, d, generator=g) * 3
    v = torch.randn(b, hkv, rows, d, generator=g).bfloat16()
    mask = torch.rand(mask_batch, 1, 1, rows, generator=g) > 0.3
    mask[..., 0] = True
    out = torch.empty(b, 1, hq, d, dtype=torch.bfloat16, device=DEV)
    _lib.decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), rows, d ** -0.5, out, _lib.Workspace(), mask.to(DEV))
    want = _masked_oracle(q, k, v, mask, d ** -0.5)
    torch.testing.assert_close(out.float().cpu(), want, rtol=2e-2, atol=1e-2)
    # an all-True mask gives exactly the unmasked result (what graph capture passes)
    ones = torch.ones(1, 1, 1, rows, dtype=torch.bool, device=DEV)
    o1, o2 = torch.empty_like(out), torch.empty_like(out)
    _lib.decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), rows, d ** -0.5, o1, _lib.Workspace(), ones)
    _lib.decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), rows, d ** -0.5, o2, _lib.Workspace())
    torch.testing.assert_close(o1, o2, rtol=0, atol=0)


def test_fused_step_with_boolean_mask(built_lib):
    """Masked rows are still evicted and re-rotated; they only leave the attention."""
    spec = dict(batch=2, hq=16, hkv=8, d=128, slots=300, n_sink=4)
    st = cases.step_inputs(**spec)
    n_sink, slots = spec["n_sink"], spec["slots"]
    want = oracle.OracleSinkLayer(n_sink, slots - n_sink, st["inv"])
    want.update(st["k0"], st["v0"])
    keys, values = want.update(st["k1"], st["v1"])
    g = torch.Generator().manual_seed(2)
    mask = torch.rand(2, 1, 1, slots + 1, generator=g) > 0.5
    mask[..., -1] = True
    want_out = _masked_oracle(st["q"], keys, values, mask, spec["d"] ** -0.5)
    kbuf, vbuf = st["k0"].float().to(DEV), st["v0"].to(DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-1), st["inv"])]
    out = torch.empty(2, 1, 16, 128, dtype=torch.bfloat16, device=DEV)
    _lib.fused_decode_step(kbuf, vbuf, st["k1"].to(DEV), st["v1"].to(DEV), st["q"].to(DEV), n_sink,
                           slots - n_sink, 1, slots, cos, sin, spec["d"] ** -0.5, out, _lib.Workspace(),
                           mask.to(DEV))
    assert digest(kbuf.cpu()) == digest(want.kbuf)
    torch.testing.assert_close(vbuf.cpu(), want.vbuf, rtol=0, atol=0)
    torch.testing.assert_close(out.float().cpu(), want_out, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("batch,heads,n_sink,window,drop,d", [
    (1, 8, 4, 1020, 1, 128), (2, 8, 4, 4092, 16, 128), (1, 8, 4, 32764, 16, 128),
    (3, 8, 0, 300, 37, 64), (2, 8, 4, 1020, 0, 128), (1, 8, 2, 500, 3, 256),
])
def test_eviction_key_copy_matches_reference(batch, heads, n_sink, window, drop, d, built_lib):
    """The eviction pass also writes the window rows' keys in the model dtype (what a chunk
    step hands to SDPA, cache.py:163): bit for bit the bf16 rounding of the reference's
    re-rotated fp32 keys; drop 0 converts without moving anything."""
    g = torch.Generator().manual_seed(batch * 100 + window + drop)
    inv = cases.inv_freq(d, 1e6)
    rows = n_sink + window + drop
    k = torch.randn(batch, heads, rows + 2, d, generator=g) * 10
    v = torch.randn(batch, heads, rows + 2, d, generator=g).bfloat16()
    want = oracle.OracleSinkLayer(n_sink, window, inv, key_dtype=torch.float32)
    want.dtype = torch.bfloat16
    want.kbuf, want.vbuf, want.length = k.clone(), v.clone(), rows
    want.evict_pending()
    kbuf, vbuf = k.to(DEV), v.to(DEV)
    copy = torch.full((batch, heads, rows, d), float("nan"), dtype=torch.bfloat16, device=DEV)
    cos, sin = [t.to(DEV) for t in oracle.rope_cos_sin(torch.tensor(-max(drop, 1)), inv)]
    ws = _lib.Workspace()
    _lib.evict_rerotate_keycopy(kbuf, vbuf, n_sink, window, drop, cos, sin, copy, ws)
    torch.cuda.synchronize()
    _status_clean(ws)
    cap = n_sink + window
    got = copy[:, :, n_sink:cap].cpu()
    torch.testing.assert_close(got, want.kbuf[:, :, n_sink:cap].bfloat16(), rtol=0, atol=0)
    assert torch.isnan(copy[:, :, :n_sink].float()).all()  # sink rows are the caller's
    assert digest(kbuf[:, :, :cap].cpu()) == digest(want.kbuf[:, :, :cap])
    torch.testing.assert_close(vbuf[:, :, :cap].cpu(), want.vbuf[:, :, :cap], rtol=0, atol=0)
