"""Host-side logic of SinkLayerV2 / SinkCacheV2 on the CPU: ring slots, the general (chunk)
step's gather and stores, pins moving into the region and the pin budget, the deferred
(fused) steady step, snapshot/restore and the mask sizes.  The two v2 kernel bindings are
replaced, for these tests only, by CPU stand-ins built on the oracle's math; the layer is
then checked against the fixtures recorded from the reference's SinkLayerV2.  The CUDA path
itself is covered by tests/test_gpu_v2.py."""

import pytest
import torch

import oracle
from attention_sinks_b200 import SinkCacheV2, SinkLayerV2, _lib
from attention_sinks_b200 import decode_attention as da
from tests.golden import cases
from tests.test_oracle_golden import _inputs_match, drive_v2, v2_pinned
from tests.util import digest


def fake_place(kbuf, vbuf, k, v, reg_k, reg_pos, R, region_out, position, t, n_sink, window, inv_freq):
    if position is not None:
        t = int(position[0])
    ring = window + 1
    if k is not None:
        sl = (t - n_sink) % ring
        kbuf[:, :, sl] = k[:, :, 0]
        vbuf[:, :, sl] = v[:, :, 0]
    if R:
        ws = max(min(t, n_sink), t - window)
        rot = oracle.region_rotation(reg_k[:, :, :R], reg_pos[:R].tolist(), ws, inv_freq)
        dst = region_out if region_out is not None else kbuf[:, :, ring:ring + R]
        dst[:, :, :R] = rot
    if position is not None:
        position[0] += 1


def fake_gather(kbuf, vbuf, n_sink, window, R, lo, hi, k, v, out_k, out_v):
    ring = window + 1
    if R:
        out_v[:, :, :R] = vbuf[:, :, ring:ring + R]
    nwin = max(0, hi - lo)
    for i in range(nwin):
        slot = (lo + i - n_sink) % ring
        out_k[:, :, R + i] = kbuf[:, :, slot]
        out_v[:, :, R + i] = vbuf[:, :, slot]
    if k is not None:
        n = k.shape[-2]
        out_k[:, :, R + nwin:R + nwin + n] = k
        out_v[:, :, R + nwin:R + nwin + n] = v


def fake_decode_step(kbuf, vbuf, k, v, reg_k, reg_pos, R, position, n_sink, window, inv_freq, q, scale,
                     out, ws, mask=None):
    fake_place(kbuf, vbuf, k, v, reg_k, reg_pos, R, None, position, 0, n_sink, window, inv_freq)
    rows = window + 1 + R
    keep = mask[0, 0, 0] if mask is not None else slice(None)
    out.copy_(oracle.decode_attention(q, kbuf[:, :, :rows][:, :, keep], vbuf[:, :, :rows][:, :, keep], scale))
    return out


@pytest.fixture
def cpu_v2(monkeypatch):
    calls = {"place": 0, "fused": 0}

    def count(name, fn):
        def wrapped(*a, **k):
            calls[name] += 1
            return fn(*a, **k)
        return wrapped

    monkeypatch.setattr(_lib, "check_device", lambda device: None)
    monkeypatch.setattr(_lib, "prepare_device", lambda device: None)
    monkeypatch.setattr(_lib, "sm_count", lambda device: 148)
    monkeypatch.setattr(_lib, "v2_place", count("place", fake_place))
    monkeypatch.setattr(_lib, "v2_decode_step", count("fused", fake_decode_step))
    monkeypatch.setattr(_lib, "v2_gather", fake_gather)
    monkeypatch.setattr(da, "_on_kernel_device", lambda q: True)
    return calls


@pytest.mark.parametrize("spec", cases.V2_CASES, ids=lambda s: s["name"])
def test_layer_matches_reference_fixtures(cpu_v2, spec, golden):
    """Every checkpoint of the reference's SinkLayerV2 run: the logical cache bit for bit,
    the positions, the region, the pin bookkeeping and what each step returned."""
    want = golden["v2"][spec["name"]]
    k, v, inv = cases.v2_inputs(sum(spec["plan"]), spec["dtype"], spec.get("rot", 128))
    _inputs_match(want, in_k=k, in_v=v)
    layer = SinkLayerV2(spec["n_sink"], spec["window"], inv, spec.get("max_pinned", 0), v2_pinned(spec))
    for (keys, values), mark in zip(drive_v2(layer, spec, k, v), want["marks"], strict=True):
        assert digest(keys) == mark["step_k"] and digest(values) == mark["step_v"]
        kk, vv, pos = layer.kept()
        assert layer.t == mark["t"] and pos == mark["positions"]
        assert layer.region_pos == mark["region_pos"] and layer.pins_dropped == mark["pins_dropped"]
        assert layer.in_cache_length() == mark["in_cache"]
        assert digest(kk) == mark["kept_k"] and digest(vv) == mark["kept_v"]
        assert int(layer._t_dev) == layer.t


class _Module:
    training = False
    num_key_value_groups = 2
    is_causal = True


def test_fused_steady_step_defers_to_the_backend(cpu_v2):
    inv = cases.inv_freq(64, 1e6)
    layer = SinkLayerV2(2, 6, inv, fused=True)
    want = oracle.OracleSinkLayerV2(2, 6, inv)
    g = torch.Generator().manual_seed(3)
    k0, v0 = torch.randn(1, 2, 9, 64, generator=g), torch.randn(1, 2, 9, 64, generator=g)
    layer.update(k0, v0)
    want.update(k0, v0)
    for step in range(12):
        k, v = torch.randn(1, 2, 1, 64, generator=g), torch.randn(1, 2, 1, 64, generator=g)
        q = torch.randn(1, 4, 1, 64, generator=g)
        keys, values = layer.update(k, v)
        wk, wv = want.update(k, v)
        assert layer._pending is not None and keys.data_ptr() == layer._kbuf.data_ptr()
        mask = torch.ones(1, 1, 1, keys.shape[-2], dtype=torch.bool) if step == 5 else None
        o, _ = da.decode_attention_forward(_Module(), q, keys, values, mask, scaling=0.125)
        assert layer._pending is None
        torch.testing.assert_close(o.reshape(1, 1, 4, 64), oracle.decode_attention(q, wk, wv, 0.125),
                                   rtol=1e-5, atol=1e-5)
    assert cpu_v2["fused"] == 12
    kk, vv, pos = layer.kept()
    wk, wv, wpos = want.kept()
    assert pos == wpos
    torch.testing.assert_close(kk, wk, rtol=0, atol=0)
    torch.testing.assert_close(vv, wv, rtol=0, atol=0)


def test_step_that_moves_a_pin_is_placed_before_attention(cpu_v2):
    """The reference moves the pin inside update(), after the step's region rotation and
    before attention: the fused path must not defer that step."""
    inv = cases.inv_freq(64, 1e6)
    cache = SinkCacheV2(2, 6, inv, num_layers=1, max_pinned=4, fused=True)
    cache.pin(4, 5)
    layer = cache.layers[0]
    g = torch.Generator().manual_seed(4)
    layer.update(torch.randn(1, 2, 8, 64, generator=g), torch.randn(1, 2, 8, 64, generator=g))
    moved = []
    for _ in range(5):
        steady = cache.is_steady
        layer.update(torch.randn(1, 2, 1, 64, generator=g), torch.randn(1, 2, 1, 64, generator=g))
        moved.append((steady, layer._pending is None, list(layer.region_pos)))
        layer.materialize()
    # t = 8: position 8 - 6 = 2 (a sink) leaves; t = 10: pinned 4 leaves -> not steady, placed now
    assert moved[2] == (False, True, [0, 1, 4])
    assert all(m[1] is False for i, m in enumerate(moved) if i != 2)


def test_mask_sizes_line_chunk_queries_up_causally(cpu_v2):
    layer = SinkLayerV2(4, 60, cases.inv_freq(64, 1e6))
    layer.update(torch.randn(1, 2, 200, 64), torch.randn(1, 2, 200, 64))
    n = layer.in_cache_length()
    assert n == 64 and layer.get_seq_length() == 200
    kv_len, kv_off = layer.get_mask_sizes(30)
    assert (kv_len, kv_off) == (94, 136)
    # chunk query i (absolute position 200 + i) sees chunk key j (kv index n + j) iff j <= i
    for i, j in ((0, 0), (5, 5), (5, 6), (29, 29)):
        assert ((n + j) + kv_off <= 200 + i) == (j <= i)


def test_snapshot_restore_keeps_pointers(cpu_v2):
    inv = cases.inv_freq(64, 1e6)
    cache = SinkCacheV2(4, 20, inv, num_layers=2)
    g = torch.Generator().manual_seed(5)
    for layer in cache.layers:
        layer.update(torch.randn(1, 2, 30, 64, generator=g), torch.randn(1, 2, 30, 64, generator=g))
    ptrs = [l._kbuf.data_ptr() for l in cache.layers]
    snap = cache.snapshot()
    before = [l.kept() for l in cache.layers]
    for layer in cache.layers:
        for _ in range(7):
            layer.update(torch.randn(1, 2, 1, 64, generator=g), torch.randn(1, 2, 1, 64, generator=g))
    cache.restore(snap)
    assert [l._kbuf.data_ptr() for l in cache.layers] == ptrs
    for layer, (k, v, pos) in zip(cache.layers, before):
        kk, vv, pp = layer.kept()
        assert pp == pos and int(layer._t_dev) == layer.t == 30
        torch.testing.assert_close(kk, k, rtol=0, atol=0)
        torch.testing.assert_close(vv, v, rtol=0, atol=0)


def test_reference_argument_checks_v2():
    with pytest.raises(ValueError):
        SinkLayerV2(-1, 10, torch.ones(4))
    with pytest.raises(ValueError):
        SinkLayerV2(0, 0, torch.ones(4))
    cache = SinkCacheV2(4, 60, torch.ones(4), num_layers=1)
    with pytest.raises(ValueError):
        cache.pin(0, 3)  # max_pinned=0
    layer = cache.layers[0]
    with pytest.raises(NotImplementedError):
        layer.crop(1)
    with pytest.raises(NotImplementedError):
        layer.reorder_cache(None)


def test_v2_place_requires_a_cuda_tensor():
    k = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        _lib.v2_place(k, k, None, None, None, None, 0, None, None, 5, 4, 3, None)
    layer = SinkLayerV2(4, 60, torch.ones(32))
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.update(torch.zeros(1, 2, 1, 64, dtype=torch.bfloat16), torch.zeros(1, 2, 1, 64, dtype=torch.bfloat16))
