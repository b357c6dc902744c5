"""Host-side logic of SinkLayer / SinkCache / the attention backend on the CPU: the
deferred (fused) one-token step, materialisation, buffer growth and shrink, bookkeeping
and backend routing.  The four kernel bindings are replaced, for these tests only, by CPU
stand-ins built on the oracle's math; the CUDA path itself is covered by the gpu tests."""

import pytest
import torch

import oracle
from attention_sinks_b200 import SinkCache, SinkLayer, _lib
from attention_sinks_b200 import decode_attention as da


def _rot(x, cos, sin):
    half = x.shape[-1] // 2
    sin_signed = torch.cat((-sin[:half], sin[half:]))
    return x.float().mul(cos).addcmul_(x.float().roll(half, dims=-1), sin_signed)


def fake_evict(kbuf, vbuf, n_sink, window, drop, cos, sin, ws):
    s = n_sink
    src_k = kbuf[:, :, s + drop:s + drop + window]
    new_k = _rot(src_k, cos, sin) if cos is not None else src_k.clone()
    new_v = vbuf[:, :, s + drop:s + drop + window].clone()
    kbuf[:, :, s:s + window].copy_(new_k)
    vbuf[:, :, s:s + window].copy_(new_v)


def fake_evict_keycopy(kbuf, vbuf, n_sink, window, drop, cos, sin, k_copy, ws):
    if drop:
        fake_evict(kbuf, vbuf, n_sink, window, drop, cos, sin, ws)
    k_copy[:, :, n_sink:n_sink + window].copy_(kbuf[:, :, n_sink:n_sink + window])


def fake_append(kbuf, vbuf, k, v, row):
    kbuf[:, :, row:row + k.shape[-2]].copy_(k)
    vbuf[:, :, row:row + v.shape[-2]].copy_(v)


def fake_attention(q, kbuf, vbuf, rows, scale, out, ws, mask=None):
    if mask is not None:  # rows a boolean mask leaves out: the kernels give them no weight
        keep = mask[0, 0, 0]
        out.copy_(oracle.decode_attention(q, kbuf[:, :, :rows][:, :, keep], vbuf[:, :, :rows][:, :, keep], scale))
        return out
    out.copy_(oracle.decode_attention(q, kbuf[:, :, :rows], vbuf[:, :, :rows], scale))
    return out


def fake_fused(kbuf, vbuf, k, v, q, n_sink, window, drop, append_row, cos, sin, scale, out, ws, mask=None):
    if drop:
        fake_evict(kbuf, vbuf, n_sink, window, drop, cos, sin, ws)
    fake_append(kbuf, vbuf, k, v, append_row)
    return fake_attention(q, kbuf, vbuf, append_row + 1, scale, out, ws, mask)


@pytest.fixture
def cpu_kernels(monkeypatch):
    calls = {"evict": 0, "evict_keycopy": 0, "append": 0, "fused": 0, "attend": 0}

    def count(name, fn):
        def wrapped(*a, **k):
            calls[name] += 1
            return fn(*a, **k)
        return wrapped

    monkeypatch.setattr(_lib, "check_device", lambda device: None)
    monkeypatch.setattr(_lib, "prepare_device", lambda device: None)
    monkeypatch.setattr(_lib, "sm_count", lambda device: 148)
    monkeypatch.setattr(_lib, "evict_rerotate", count("evict", fake_evict))
    monkeypatch.setattr(_lib, "evict_rerotate_keycopy", count("evict_keycopy", fake_evict_keycopy))
    monkeypatch.setattr(_lib, "append", count("append", fake_append))
    monkeypatch.setattr(_lib, "fused_decode_step", count("fused", fake_fused))
    monkeypatch.setattr(_lib, "decode_attention", count("attend", fake_attention))
    monkeypatch.setattr(da, "_on_kernel_device", lambda q: True)
    return calls


class _Module:
    training = False
    num_key_value_groups = 2
    is_causal = True


def _feed(layer, want, plan, hkv=2, hq=4, d=64, seed=0, mask_at=(-1, -1)):
    """Feed chunks through the layer (+ the backend for one-token steps) and the oracle."""
    g = torch.Generator().manual_seed(seed)
    outs = []
    for i, n in enumerate(plan):
        k = torch.randn(1, hkv, n, d, generator=g)
        v = torch.randn(1, hkv, n, d, generator=g)
        q = torch.randn(1, hq, n, d, generator=g)
        keys, values = layer.update(k, v)
        wk, wv = want.update(k, v)
        if n == 1:
            # step 40 passes an additive float mask (SDPA fallback), step 45 the all-True
            # boolean mask Transformers builds while a CUDA graph is captured (kernel path)
            mask = None
            if i in mask_at:
                mask = (torch.zeros(1, 1, 1, keys.shape[-2]) if i == mask_at[0]
                        else torch.ones(1, 1, 1, keys.shape[-2], dtype=torch.bool))
            o, _ = da.decode_attention_forward(_Module(), q, keys, values, mask, scaling=d ** -0.5)
            outs.append((o.reshape(1, 1, hq, d), oracle.decode_attention(q, wk, wv, d ** -0.5)))
        assert layer.get_seq_length() == want.get_seq_length()
        assert (layer.tokens_seen, layer.tokens_evicted) == (want.tokens_seen, want.tokens_evicted)
    return outs


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_bookkeeping_and_contents_follow_the_reference(cpu_kernels, fused):
    inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    layer = SinkLayer(4, 20, inv, key_dtype=torch.float32, fused=fused)
    want = oracle.OracleSinkLayer(4, 20, inv, key_dtype=torch.float32)
    plan = [6] + [1] * 30 + [9] + [1] * 5 + [40] + [1] * 12
    outs = _feed(layer, want, plan, mask_at=(40, 45))
    for got, ref in outs:
        torch.testing.assert_close(got.float(), ref, rtol=1e-5, atol=1e-5)
    k, v = layer.kept()
    wk, wv = want.kept()
    torch.testing.assert_close(k, wk, rtol=0, atol=0)
    torch.testing.assert_close(v, wv, rtol=0, atol=0)
    assert layer._kbuf.shape[-2] == 25  # shrunk back after the 40-token chunk
    if fused:
        assert cpu_kernels["fused"] > 0
        assert layer._pending is None
    else:
        assert cpu_kernels["fused"] == 0 and cpu_kernels["attend"] > 0


def test_fused_defers_until_attention(cpu_kernels):
    inv = torch.ones(32)
    layer = SinkLayer(2, 6, inv, fused=True)
    g = torch.Generator().manual_seed(1)
    layer.update(torch.randn(1, 2, 9, 64, generator=g), torch.randn(1, 2, 9, 64, generator=g))
    keys, values = layer.update(torch.randn(1, 2, 1, 64, generator=g), torch.randn(1, 2, 1, 64, generator=g))
    assert layer._pending is not None and layer._pending[0] == 1  # drop 1, not yet run
    assert layer.length == 9 and layer.tokens_evicted == 1
    assert keys.dtype == torch.float32 and keys.data_ptr() == layer._kbuf.data_ptr()
    from attention_sinks_b200.cache import pending_layer
    assert pending_layer(keys) is layer
    n = cpu_kernels["evict"] + cpu_kernels["fused"]
    layer.kept()  # materialises the deferred step without attention
    # one eviction applies the deferred step, one more evicts the copies kept() returns
    assert layer._pending is None and cpu_kernels["evict"] + cpu_kernels["fused"] == n + 2
    assert pending_layer(keys) is None


def test_unfused_returns_model_dtype_keys(cpu_kernels):
    layer = SinkLayer(2, 6, torch.ones(32), key_dtype=torch.float32)
    keys, _ = layer.update(torch.randn(1, 2, 3, 64).bfloat16(), torch.randn(1, 2, 3, 64).bfloat16())
    assert keys.dtype == torch.bfloat16  # what stock SDPA expects (cache.py:163)
    assert layer._kbuf.dtype == torch.float32


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_model_dtype_keys_come_from_the_eviction_pass(cpu_kernels, fused):
    """fp32 key storage, bf16 model: every multi-token (and unfused) step returns the bf16
    copy of the cache (cache.py:163) -- window rows written by the eviction pass itself (or
    converted when nothing is evicted), sink and new rows copied -- bit for bit what the
    reference returns; the layer keeps views of its own fp32 buffers."""
    inv = 1.0 / (1e6 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    layer = SinkLayer(4, 20, inv, key_dtype=torch.float32, fused=fused)
    want = oracle.OracleSinkLayer(4, 20, inv, key_dtype=torch.float32)
    g = torch.Generator().manual_seed(9)
    for n in [6, 9, 1, 1, 14, 3, 40, 2, 1, 30]:
        k = torch.randn(1, 2, n, 64, generator=g).bfloat16()
        v = torch.randn(1, 2, n, 64, generator=g).bfloat16()
        keys, values = layer.update(k, v)
        wk, wv = want.update(k, v)
        if layer._pending is not None:  # a fused one-token step, deferred: the fp32 view
            assert fused and n == 1 and keys.dtype == torch.float32
            layer.materialize()
            continue
        assert keys.dtype == torch.bfloat16 and layer.keys.dtype == torch.float32
        torch.testing.assert_close(keys, wk, rtol=0, atol=0)
        torch.testing.assert_close(values, wv, rtol=0, atol=0)
    assert cpu_kernels["evict_keycopy"] > 0


def test_reference_argument_checks():
    with pytest.raises(ValueError):
        SinkLayer(-1, 10, torch.ones(4))
    with pytest.raises(ValueError):
        SinkLayer(0, 0, torch.ones(4))
    layer = SinkLayer(1, 3, torch.ones(4))
    with pytest.raises(NotImplementedError):
        layer.crop(1)
    with pytest.raises(NotImplementedError):
        layer.reorder_cache(None)


def test_from_model_rejects_sliding_layers():
    from transformers import Qwen3Config

    class _M:
        def __init__(self, cfg):
            self.config = cfg

        def modules(self):
            return []

    cfg = Qwen3Config(num_hidden_layers=2, layer_types=["full_attention", "sliding_attention"],
                      use_sliding_window=True, sliding_window=16)
    with pytest.raises(ValueError):
        SinkCache.from_model(_M(cfg), 4, 60)


def test_from_model_picks_fused_mode_from_the_backend():
    from tests.golden import cases
    name = da.register()
    m = cases.build_model(cases.tiny_qwen3_config(), torch.float32, attn=name)
    assert all(l.fused for l in SinkCache.from_model(m, 4, 60).layers)
    m = cases.build_model(cases.tiny_qwen3_config(), torch.float32, attn="sdpa")
    assert not any(l.fused for l in SinkCache.from_model(m, 4, 60).layers)
