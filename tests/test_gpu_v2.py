"""The ring-buffer cache (SinkCacheV2 / SinkLayerV2) on the GPU.

Kernel level: sink_v2_place and sink_v2_decode_step against the oracle and against the
reference's own fixtures (region rotation with fp64 angles bit for bit, ring slots, the
device position).  Layer level: the reference's SinkLayerV2 checkpoints reproduced bit for
bit by the CUDA path.  Model level: the reference's tests/test_cache_v2.py checks on a
random-init Qwen3, in both modes -- unfused (stock SDPA over the returned views) and fused
(the registered backend running sink_v2_decode_step)."""

import pytest
import torch
from transformers import DynamicCache
from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

import oracle
from attention_sinks_b200 import SinkCache, SinkCacheV2, SinkLayerV2, StreamRunner, _lib, register
from attention_sinks_b200.decode_attention import calls
from tests.golden import cases
from tests.test_gpu_cache import PreRopeRecorder, stream
from tests.test_oracle_golden import drive_v2, v2_pinned
from tests.util import digest

pytestmark = pytest.mark.gpu
DEV = "cuda"
BACKEND = register()
MODES = [False, True]
MODE_IDS = ["unfused", "fused"]


def model_for(dtype, fused, n_tokens=401):
    model, ids = cases.tiny_qwen3(dtype, attn=BACKEND if fused else "sdpa", n_tokens=n_tokens)
    return model.to(DEV), ids.to(DEV)


# ------------------------------------------------------------------ kernels


def test_region_rotation_matches_reference_far_from_origin(golden):
    """sink_v2_place into a separate output at window starts up to 5e7: bit-identical to the
    reference's _rotate_region (fp64 angles)."""
    want = golden["v2"]["rotation"]
    reg_k, reg_pos, inv = cases.v2_rotation_inputs()
    assert digest(reg_k) == want["in_k"]
    kbuf = torch.zeros(1, 8, 61 + 6, 128, dtype=torch.bfloat16, device=DEV)
    rk, rp = reg_k.to(DEV), torch.tensor(reg_pos, device=DEV)
    inv64 = inv.to(DEV, torch.float64)
    for ws in cases.V2_ROTATION_WS:
        out = torch.empty(1, 8, 6, 128, dtype=torch.bfloat16, device=DEV)
        t = ws + 60  # window start t - window
        _lib.v2_place(kbuf, kbuf.clone(), None, None, rk, rp, 6, out, None, t, 4, 60, inv64)
        assert digest(out) == want[f"ws_{ws}"], ws


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("d,rot", [(128, 128), (64, 64), (256, 256), (128, 64)])
@pytest.mark.parametrize("t", [64 + 4, 3_000_001])
def test_place_step_matches_oracle(dtype, d, rot, t):
    """The steady place step: new row into slot (t - n_sink) mod ring, region rotated from
    its originals (bit-exact against the oracle), device position advanced by one and the
    arrival counter back at 0; nothing else in the buffers changes."""
    g = torch.Generator().manual_seed(t % 97 + d)
    b, h, n_sink, window, R = 3, 4, 4, 64, 7
    ring = window + 1
    kbuf = (torch.randn(b, h, ring + 9, d, generator=g) * 3).to(dtype)
    vbuf = torch.randn(b, h, ring + 9, d, generator=g).to(dtype)
    reg_k = (torch.randn(b, h, 9, d, generator=g) * 30).to(dtype)
    reg_pos = [0, 1, 2, 3, 17, 40, t - 70]
    k, v = torch.randn(b, h, 1, d, generator=g).to(dtype), torch.randn(b, h, 1, d, generator=g).to(dtype)
    inv = cases.inv_freq(rot, 1e6)
    want_k, want_v = kbuf.clone(), vbuf.clone()
    sl = (t - n_sink) % ring
    want_k[:, :, sl], want_v[:, :, sl] = k[:, :, 0], v[:, :, 0]
    want_k[:, :, ring:ring + R] = oracle.region_rotation(reg_k[:, :, :R], reg_pos, t - window, inv)
    gk, gv = kbuf.to(DEV), vbuf.to(DEV)
    pos = torch.tensor([t, 0], device=DEV)
    _lib.v2_place(gk, gv, k.to(DEV), v.to(DEV), reg_k.to(DEV), torch.tensor(reg_pos + [0, 0], device=DEV), R,
                  None, pos, 0, n_sink, window, inv.to(DEV, torch.float64))
    assert pos.tolist() == [t + 1, 0]
    assert digest(gv) == digest(want_v)
    assert digest(gk) == digest(want_k)


@pytest.mark.parametrize("batch,hq,hkv,d,window,R", [
    (1, 16, 8, 128, 1020, 4), (4, 32, 8, 64, 300, 0), (2, 14, 2, 128, 4095, 36), (3, 8, 8, 256, 60, 1),
    (1, 16, 8, 128, 32764, 4), (32, 16, 8, 128, 4095, 4), (8, 64, 8, 128, 1020, 4),
    (8, 16, 8, 128, 32764, 4), (18, 16, 8, 128, 2047, 4), (19, 16, 8, 128, 2047, 4),
    (64, 16, 8, 128, 252, 4), (2, 16, 8, 128, 4095, 4),
])
def test_fused_decode_step_matches_place_then_attention(batch, hq, hkv, d, window, R):
    """sink_v2_decode_step leaves the cache exactly as sink_v2_place does, and its
    attention over ring + region is within 2e-2 of fp32 attention over the same rows, in
    every way the step runs: on the tensor-core path (16-bit, head_dim 128) with the place
    work in two warps beside the pipeline (CTAs walking several items, at least 16 chunks of
    128 rows per CTA: 32 x 8 pairs at 4,096 slots, 8 x 8 at 32,768, 19 x 8 at 2,048), with
    every thread placing first (other steps over at most one pair per SM: 18 x 8 at 2,048,
    1 x 8 at 1,024 and 32,768, 2 x 8 at 4,096, GQA 8 and 7), and with the place kernel first
    (64 x 8 pairs at 256 slots); on the stream kernel after the place kernel (head_dim 64
    and 256).  The launch count tells which ran: the step
    launches what attention over the same rows launches, plus the place kernel where it is
    not fused."""
    g = torch.Generator().manual_seed(window + R)
    ring, dt = window + 1, torch.bfloat16
    t = 5 * window + 13
    kbuf = (torch.randn(batch, hkv, ring + R + 2, d, generator=g) * 3).to(dt).to(DEV)
    vbuf = torch.randn(batch, hkv, ring + R + 2, d, generator=g).to(dt).to(DEV)
    reg_k = (torch.randn(batch, hkv, max(R, 1), d, generator=g) * 3).to(dt).to(DEV)
    reg_pos = torch.tensor(list(range(R)) or [0], device=DEV)
    k, v = [torch.randn(batch, hkv, 1, d, generator=g).to(dt).to(DEV) for _ in range(2)]
    q = torch.randn(batch, hq, 1, d, generator=g).to(dt).to(DEV)
    inv = cases.inv_freq(d, 1e6).to(DEV, torch.float64)
    ref_k, ref_v, ref_pos = kbuf.clone(), vbuf.clone(), torch.tensor([t, 0], device=DEV)
    _lib.v2_place(ref_k, ref_v, k, v, reg_k, reg_pos, R, None, ref_pos, 0, 4, window, inv)
    pos = torch.tensor([t, 0], device=DEV)
    out = torch.empty(batch, 1, hq, d, dtype=dt, device=DEV)
    ws = _lib.Workspace()
    n0 = _lib.launch_count()
    _lib.v2_decode_step(kbuf, vbuf, k, v, reg_k, reg_pos, R, pos, 4, window, inv, q, d ** -0.5, out, ws)
    n_step = _lib.launch_count() - n0
    assert pos.tolist() == ref_pos.tolist() == [t + 1, 0]
    assert torch.equal(kbuf, ref_k) and torch.equal(vbuf, ref_v)
    rows = ring + R
    n0 = _lib.launch_count()
    _lib.decode_attention(q, ref_k, ref_v, rows, d ** -0.5, torch.empty_like(out), _lib.Workspace())
    n_attend = _lib.launch_count() - n0
    sms = _lib.sm_count(torch.device(DEV))
    pairs = batch * hkv
    plan = _lib.plan(_lib.OP_ATTEND, batch, hkv, hq, d, dt, dt, rows, 0, 1, 0, sms)
    items = pairs * plan["splits"]
    ctas = min(items, sms)
    fused = d == 128 and ((items > ctas and pairs * -(-rows // 128) >= 16 * ctas) or pairs <= sms)
    assert n_step == n_attend + (0 if fused else 1)
    want = oracle.decode_attention(q.cpu(), ref_k[:, :, :rows].cpu(), ref_v[:, :, :rows].cpu(), d ** -0.5)
    torch.testing.assert_close(out.float().cpu(), want, rtol=0, atol=2e-2)
    assert ws.read_status() == 0


def test_place_argument_errors():
    kb = torch.zeros(1, 2, 70, 128, dtype=torch.bfloat16, device=DEV)
    inv = torch.ones(64, dtype=torch.float64, device=DEV)
    rk, rp = torch.zeros(1, 2, 4, 128, dtype=torch.bfloat16, device=DEV), torch.zeros(4, dtype=torch.long, device=DEV)
    with pytest.raises(RuntimeError, match="out of range"):  # ring + R > slots
        _lib.v2_place(kb, kb.clone(), None, None, rk, rp, 4, None, None, 10, 4, 66, inv)
    with pytest.raises(RuntimeError, match="dtype"):  # K and V types differ
        _lib.v2_place(kb.float(), kb.clone(), None, None, rk, rp, 4, None, None, 10, 4, 60, inv)
    with pytest.raises(RuntimeError, match="out of range"):  # rotary dims beyond head_dim
        _lib.v2_place(kb, kb.clone(), None, None, rk, rp, 4, None, None, 10, 4, 60,
                      torch.ones(65, dtype=torch.float64, device=DEV))


# ------------------------------------------------------------------ layer


@pytest.mark.parametrize("spec", cases.V2_CASES, ids=lambda s: s["name"])
def test_layer_matches_reference_fixtures(spec, golden):
    """The reference's SinkLayerV2 checkpoints (kept keys/values, positions, region, pins,
    the K/V each step returned) reproduced bit for bit on the GPU."""
    want = golden["v2"][spec["name"]]
    k, v, inv = cases.v2_inputs(sum(spec["plan"]), spec["dtype"], spec.get("rot", 128))
    assert digest(k) == want["in_k"]
    layer = SinkLayerV2(spec["n_sink"], spec["window"], inv, spec.get("max_pinned", 0), v2_pinned(spec))
    for (keys, values), mark in zip(drive_v2(layer, spec, k.to(DEV), v.to(DEV)), want["marks"], strict=True):
        assert digest(keys) == mark["step_k"] and digest(values) == mark["step_v"]
        kk, vv, pos = layer.kept()
        assert layer.t == mark["t"] and pos == mark["positions"]
        assert layer.region_pos == mark["region_pos"] and layer.pins_dropped == mark["pins_dropped"]
        assert digest(vv) == mark["kept_v"]
        assert digest(kk) == mark["kept_k"]
        assert int(layer._t_dev) == layer.t and int(layer._position[1]) == 0


# ------------------------------------------------------------------ model (tests/test_cache_v2.py)


def reference_from_kept(model, rec, cache):
    """DynamicCache holding the tokens v2 keeps, each pre-RoPE key rotated once by HF at the
    position v2 says it sits at (test_cache_v2.py:15-32)."""
    layer0 = cache.layers[0]
    t = layer0.t
    ws = layer0._window_start(t)
    kept_pos = list(layer0.region_pos) + list(range(max(ws, layer0.n_sink), t))
    at = torch.tensor(layer0.kept()[2], device=DEV)[None]
    idx = torch.tensor(kept_pos, device=DEV)
    ref = DynamicCache()
    for i in range(model.config.num_hidden_layers):
        k, v = rec.get(i)
        k, v = k[:, :, idx], v[:, :, idx]
        cos, sin = model.model.rotary_emb(k, at)
        _, k = apply_rotary_pos_emb(k, k, cos, sin)
        ref.update(k, v, i)
    return ref, kept_pos


def check(model, ids, n_sink, window, prefill=16, pins=(), max_pinned=0, plan=None):
    """test_cache_v2.py:35-58"""
    rec = PreRopeRecorder(model)
    cache = SinkCacheV2.from_model(model, n_sink=n_sink, window=window, max_pinned=max_pinned)
    for a, b in pins:
        cache.pin(a, b)
    if plan is None:
        stream(model, ids[:, :-1], cache, prefill=prefill)
    else:
        t = 0
        with torch.no_grad():
            for n in plan:
                model(ids[:, t:t + n], past_key_values=cache, use_cache=True)
                t += n
        assert t == ids.shape[1] - 1
    rec.remove()
    ref, kept_pos = reference_from_kept(model, rec, cache)
    snap = [(l.kept()[0].clone(), l.kept()[1].clone(), r.keys.clone(), r.values.clone())
            for l, r in zip(cache.layers, ref.layers)]
    t = cache.tokens_seen
    pos = torch.tensor([[t]], device=DEV)
    with torch.no_grad():
        got = model(ids[:, -1:], past_key_values=cache, use_cache=True).logits.float()
        want = model(ids[:, -1:], past_key_values=ref, use_cache=True, position_ids=pos).logits.float()
    return got, want, cache, snap, kept_pos


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_no_eviction_matches_dynamic_cache_bitwise(fused):
    model, ids = model_for(torch.bfloat16, fused)
    ids = ids[:, :200]
    ref = stream(model, ids, DynamicCache())
    got = stream(model, ids, SinkCacheV2.from_model(model, n_sink=4, window=1020))
    torch.testing.assert_close(got, ref, rtol=0, atol=0)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
@pytest.mark.parametrize("n_sink", [0, 1, 4])
def test_matches_reference_fp32(n_sink, fused):
    """test_cache_v2.py:68-77: values exact, sink keys within 1e-4 of HF's fp32 angles,
    logits within 2e-3 of attention over exactly the kept tokens."""
    model, ids = model_for(torch.float32, fused)
    before = calls["fused_step"]
    got, want, cache, snap, kept = check(model, ids[:, :301], n_sink, 60)
    assert (calls["fused_step"] > before) == fused
    assert len(kept) == n_sink + 60 and cache.tokens_evicted == 301 - n_sink - 60
    assert cache.get_seq_length() == 301
    for ka, va, kb, vb in snap:
        torch.testing.assert_close(va, vb, rtol=0, atol=0)
        torch.testing.assert_close(ka, kb, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(got, want, rtol=0, atol=2e-3)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_bf16_window_keys_are_exact(fused):
    """test_cache_v2.py:80-89: window keys bit-for-bit what the model wrote after 236
    evictions; sink keys within one bf16 rounding of a direct rotation."""
    model, ids = model_for(torch.bfloat16, fused)
    got, want, cache, snap, _ = check(model, ids[:, :301], 4, 60)
    for ka, va, kb, vb in snap:
        torch.testing.assert_close(ka[:, :, 4:], kb[:, :, 4:], rtol=0, atol=0)
        torch.testing.assert_close(va, vb, rtol=0, atol=0)
        torch.testing.assert_close(ka[:, :, :4].float(), kb[:, :, :4].float(), rtol=2 ** -7,
                                   atol=2 ** -7 * kb.float().abs().max().item())
    assert (got.argmax(-1) == want.argmax(-1)).all()


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_matches_v1(fused):
    """test_cache_v2.py:92-97: same relative positions as v1 -> same logits up to rounding."""
    model, ids = model_for(torch.float32, fused)
    ids = ids[:, :400]
    v1 = stream(model, ids, SinkCache.from_model(model, 4, 60))
    v2 = stream(model, ids, SinkCacheV2.from_model(model, 4, 60))
    torch.testing.assert_close(v2, v1, rtol=0, atol=1e-3)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_chunks_and_long_prefill(fused):
    """test_cache_v2.py:100-109: chunks larger than the window and a prefill longer than the
    cache."""
    model, ids = model_for(torch.float32, fused)
    ids = ids[:, :401]
    got, want, *_ = check(model, ids, 4, 60, plan=[200, 1, 1, 37, 90, 1, 1, 69])
    torch.testing.assert_close(got, want, rtol=0, atol=2e-3)
    with torch.no_grad():
        dyn = model(ids[:, :200], past_key_values=DynamicCache(), use_cache=True).logits
        chunk = model(ids[:, :200], past_key_values=SinkCacheV2.from_model(model, 4, 60), use_cache=True).logits
    torch.testing.assert_close(chunk, dyn, rtol=0, atol=0)


def test_chunk_after_eviction_is_causal():
    """A chunk's query i does not see chunk tokens after i (the mask sizes line the chunk's
    queries up with its keys): the first 10 logits of a 30-token chunk equal those of the
    same chunk cut to 10 tokens."""
    model, ids = model_for(torch.float32, fused=False)
    outs = []
    for n in (30, 10):
        cache = SinkCacheV2.from_model(model, 4, 60)
        with torch.no_grad():
            model(ids[:, :100], past_key_values=cache, use_cache=True)
            outs.append(model(ids[:, 100:100 + n], past_key_values=cache, use_cache=True).logits)
    torch.testing.assert_close(outs[0][:, :10], outs[1], rtol=0, atol=1e-5)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_pinned_tokens_move_to_region(fused):
    """test_cache_v2.py:112-120"""
    model, ids = model_for(torch.float32, fused)
    pins = [(20, 30), (100, 105)]
    got, want, cache, _, kept = check(model, ids[:, :301], 4, 60, pins=pins, max_pinned=32,
                                      plan=[16] + [1] * 84 + [40] + [1] * 160)
    assert kept[:19] == [0, 1, 2, 3] + list(range(20, 30)) + list(range(100, 105))
    assert cache.region_size == 19
    torch.testing.assert_close(got, want, rtol=0, atol=2e-3)


def test_pin_budget_drops_oldest():
    """test_cache_v2.py:123-129"""
    model, ids = model_for(torch.bfloat16, fused=True)
    cache = SinkCacheV2.from_model(model, n_sink=4, window=60, max_pinned=8)
    cache.pin(10, 16)
    cache.pin(30, 36)
    stream(model, ids[:, :200], cache)
    layer = cache.layers[0]
    assert layer.region_pos == [0, 1, 2, 3, 14, 15, 30, 31, 32, 33, 34, 35] and layer.pins_dropped == 4


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
@pytest.mark.parametrize("pinned", [False, True])
def test_cuda_graph_replay_matches_eager(fused, pinned):
    """test_cache_v2.py:132-155: graphed steady steps (growing positions from the device
    counter), chunks in between, pin moves forcing eager steps + recapture: bitwise equal to
    all-eager."""
    model, ids = model_for(torch.bfloat16, fused)
    ids = ids[:, :400]
    plan = [16] + [1] * 120 + [30] + [1] * 80 + [45] + [1] * 100
    outs, replays = {}, {}
    for graphed in (False, True):
        cache = SinkCacheV2.from_model(model, n_sink=4, window=60, max_pinned=16 if pinned else 0)
        if pinned:
            cache.pin(140, 146)
            cache.pin(200, 203)
        runner = StreamRunner(model, cache, use_graph=graphed)
        out, t = [], 0
        with torch.no_grad():
            for n in plan:
                out.append(runner.step(ids[:, t:t + n]).float().clone())
                t += n
        outs[graphed], replays[graphed] = torch.cat(out, 1), runner.replays
        assert cache.tokens_seen == sum(plan)
        assert all(int(l._t_dev) == l.t for l in cache.layers)
        if pinned:
            assert cache.region_size == 4 + 9
    assert replays[True] > 200
    torch.testing.assert_close(outs[True], outs[False], rtol=0, atol=0)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_snapshot_restore(fused):
    """test_cache_v2.py:158-167"""
    model, ids = model_for(torch.bfloat16, fused)
    ids = ids[:, :300]
    cache = SinkCacheV2.from_model(model, 4, 60)
    stream(model, ids[:, :200], cache)
    snap = cache.snapshot()
    with torch.no_grad():
        a = model(ids[:, 200:260], past_key_values=cache, use_cache=True).logits
        cache.restore(snap)
        b = model(ids[:, 200:260], past_key_values=cache, use_cache=True).logits
    torch.testing.assert_close(a, b, rtol=0, atol=0)


@pytest.mark.parametrize("fused", MODES, ids=MODE_IDS)
def test_streamed_nll_matches_reference(fused, golden, golden_arrays):
    """Per-token NLL of the tiny fp32 Qwen3 streamed through SinkCacheV2(4, 60) (graphed
    steady steps) vs the reference's own CPU run: mean within 0.5%, each token within 1e-3."""
    model, ids = model_for(torch.float32, fused, n_tokens=301)
    cache = SinkCacheV2.from_model(model, n_sink=4, window=60)
    runner = StreamRunner(model, cache)
    nll, logits = cases.stream_nll(model, ids, cache, prefill=16, step=runner.step)
    want = golden["v2_stream"]
    assert runner.replays > 200
    assert abs(nll.mean().item() - want["mean_nll"]) < 5e-3 * want["mean_nll"]
    torch.testing.assert_close(nll, torch.from_numpy(golden_arrays["v2_stream/nll"]), rtol=0, atol=1e-3)
    torch.testing.assert_close(logits, torch.from_numpy(golden_arrays["v2_stream/last_logits"]), rtol=0, atol=2e-3)
    assert cache.tokens_evicted == want["tokens_evicted"] and cache.region_size == want["region_size"]
    assert cache.workspace.read_status() == 0


@pytest.mark.parametrize("window,n_sink,R,t,n,d", [
    (60, 4, 4, 200, 16, 128),      # window wraps around the ring's end
    (60, 4, 12, 64, 0, 64),        # window exactly full, no chunk
    (1020, 4, 4, 1500, 37, 128),
    (30, 0, 0, 20, 5, 256),        # no sinks, window not full yet
])
def test_gather_matches_ring_order(window, n_sink, R, t, n, d):
    """sink_v2_gather: [region values, window rows in position order, chunk] -- the rows the
    reference gathers with index_select and cat (cache_v2.py:189-193) -- bit for bit."""
    g = torch.Generator(device=DEV).manual_seed(window + t)
    b, h = 2, 4
    ring = window + 1
    kbuf = torch.randn(b, h, ring + R + 3, d, device=DEV, generator=g).bfloat16()
    vbuf = torch.randn(b, h, ring + R + 3, d, device=DEV, generator=g).bfloat16()
    lo, hi = max(max(min(t, n_sink), t - window), n_sink), t
    k = torch.randn(b, h, n, d, device=DEV, generator=g).bfloat16() if n else None
    v = torch.randn(b, h, n, d, device=DEV, generator=g).bfloat16() if n else None
    rows = R + max(0, hi - lo) + n
    ok = torch.full((b, h, rows, d), 7.0, dtype=torch.bfloat16, device=DEV)
    ov = torch.full((b, h, rows, d), 7.0, dtype=torch.bfloat16, device=DEV)
    _lib.v2_gather(kbuf, vbuf, n_sink, window, R, lo, hi, k, v, ok, ov)
    slots = torch.tensor([(p - n_sink) % ring for p in range(lo, hi)], dtype=torch.long, device=DEV)
    want_k = torch.cat([kbuf.index_select(2, slots)] + ([k] if n else []), -2)
    want_v = torch.cat([vbuf[:, :, ring:ring + R], vbuf.index_select(2, slots)] + ([v] if n else []), -2)
    torch.testing.assert_close(ok[:, :, R:], want_k, rtol=0, atol=0)
    torch.testing.assert_close(ov, want_v, rtol=0, atol=0)
    assert bool((ok[:, :, :R] == 7.0).all())  # the region's keys are the place kernel's
