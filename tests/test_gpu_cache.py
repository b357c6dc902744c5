"""SinkCache / SinkLayer through a Transformers model on the GPU: the reference's
tests/test_cache.py checks, on a random-init Qwen3 (no weights available) with seeded
uniform tokens, in both modes -- unfused (stock SDPA backend) and fused (the registered
`sdpa_decode` backend running sink_fused_decode_step)."""

import numpy as np
import pytest
import torch
from transformers import DynamicCache
from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

from attention_sinks_b200 import SinkCache, StreamRunner, register
from attention_sinks_b200.decode_attention import calls
from tests.golden import cases

pytestmark = pytest.mark.gpu
DEV = "cuda"
BACKEND = register()


def model_for(dtype, fused):
    model, ids = cases.tiny_qwen3(dtype, attn=BACKEND if fused else "sdpa")
    return model.to(DEV), ids.to(DEV)


class PreRopeRecorder:
    """Each layer's keys before RoPE (after k_norm) and values, for every token fed."""

    def __init__(self, model):
        self.keys = {i: [] for i in range(model.config.num_hidden_layers)}
        self.values = {i: [] for i in range(model.config.num_hidden_layers)}
        self.handles = []
        for i, layer in enumerate(model.model.layers):
            attn = layer.self_attn
            self.handles.append(attn.k_norm.register_forward_hook(self._hook(self.keys[i], attn.head_dim)))
            self.handles.append(attn.v_proj.register_forward_hook(self._hook(self.values[i], attn.head_dim)))

    @staticmethod
    def _hook(store, hd):
        def fn(_mod, _inp, out):
            b, q = out.shape[:2]
            store.append(out.reshape(b, q, -1, hd).transpose(1, 2).detach())
        return fn

    def get(self, layer):
        return torch.cat(self.keys[layer], -2), torch.cat(self.values[layer], -2)

    def remove(self):
        for h in self.handles:
            h.remove()


@torch.no_grad()
def stream(model, ids, cache, prefill=16):
    out = [model(ids[:, :prefill], past_key_values=cache, use_cache=True).logits]
    for t in range(prefill, ids.shape[1]):
        out.append(model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits)
    return torch.cat(out, 1).float()


@torch.no_grad()
def kept_tokens_reference(model, rec, n_tokens, n_sink, window):
    """DynamicCache of exactly the kept tokens, rotated once by HF at positions 0..cap-1."""
    kept = list(range(n_sink)) + list(range(n_tokens - window, n_tokens))
    idx = torch.tensor(kept, device=DEV)
    pos = torch.arange(len(kept), device=DEV)[None]
    ref = DynamicCache()
    for layer in range(model.config.num_hidden_layers):
        k, v = rec.get(layer)
        k, v = k[:, :, idx], v[:, :, idx]
        cos, sin = model.model.rotary_emb(k, pos)
        _, k = apply_rotary_pos_emb(k, k, cos, sin)
        ref.update(k, v, layer)
    return ref


def eviction_check(model, ids, n_sink, window, rerotate_keys=True, prefill=16, key_dtype=torch.float32):
    rec = PreRopeRecorder(model)
    cache = SinkCache.from_model(model, n_sink=n_sink, window=window, rerotate_keys=rerotate_keys,
                                 key_dtype=key_dtype)
    stream(model, ids[:, :-1], cache, prefill=prefill)
    rec.remove()
    ref = kept_tokens_reference(model, rec, ids.shape[1] - 1, n_sink, window)
    snap = [(*[t.clone() for t in a.kept()], b.keys.clone(), b.values.clone())
            for a, b in zip(cache.layers, ref.layers)]
    with torch.no_grad():
        got = model(ids[:, -1:], past_key_values=cache, use_cache=True).logits.float()
        want = model(ids[:, -1:], past_key_values=ref, use_cache=True).logits.float()
    return got, want, cache, snap


def test_no_eviction_matches_dynamic_cache_bitwise():
    model, ids = model_for(torch.bfloat16, fused=False)
    ids = ids[:, :200]
    ref = stream(model, ids, DynamicCache())
    sink = stream(model, ids, SinkCache.from_model(model, n_sink=4, window=1020))
    torch.testing.assert_close(sink, ref, rtol=0, atol=0)


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_cache_size_is_bounded(fused, golden):
    model, ids = model_for(torch.bfloat16, fused)
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    assert all(l.fused == fused for l in cache.layers)
    stream(model, ids[:, :300], cache)
    want = golden["stream"]
    assert cache.get_seq_length() == want["seq_length"] == 64
    assert cache.is_steady
    assert cache.tokens_seen == 300 and cache.tokens_evicted == 235
    for layer in cache.layers:
        k, v = layer.kept()
        assert k.shape[-2] == v.shape[-2] == 64
        assert layer._kbuf.shape[-2] == want["buffer_slots"] == 65
    assert cache.workspace.read_status() == 0


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
@pytest.mark.parametrize("n_sink", [0, 4])
def test_eviction_equals_attention_over_kept_tokens_fp32(n_sink, fused):
    """After 230+ evictions the cache is the kept tokens at contiguous positions
    (test_cache.py:189-202): key rel err < 1e-5, values exact, logits within 2e-3."""
    model, ids = model_for(torch.float32, fused)
    calls_before = calls["fused_step"]
    got, want, cache, snap = eviction_check(model, ids[:, :301], n_sink, 60)
    assert cache.tokens_evicted > 200
    assert (calls["fused_step"] > calls_before) == fused
    kerr = max(((ka - kb).norm() / kb.norm()).item() for ka, _, kb, _ in snap)
    for ka, va, kb, vb in snap:
        torch.testing.assert_close(va, vb, rtol=0, atol=0)
    assert kerr < 1e-5, kerr
    torch.testing.assert_close(got, want, rtol=0, atol=2e-3)


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
@pytest.mark.parametrize("n_sink", [0, 4])
def test_eviction_equals_attention_over_kept_tokens_bf16(n_sink, fused):
    """bf16 model and bf16 key storage (test_cache.py:205-216)."""
    model, ids = model_for(torch.bfloat16, fused)
    got, want, cache, snap = eviction_check(model, ids[:, :301], n_sink, 60, key_dtype=None)
    err = (got - want).abs().max().item()
    kerr = max(((ka.float() - kb.float()).norm() / kb.float().norm()).item() for ka, _, kb, _ in snap)
    assert kerr < 2e-2
    assert err < 0.5


def test_fp32_key_storage_removes_drift():
    """test_cache.py:219-228"""
    model, ids = model_for(torch.bfloat16, fused=True)
    _, _, _, snap16 = eviction_check(model, ids[:, :301], 4, 60, key_dtype=None)
    _, _, _, snap32 = eviction_check(model, ids[:, :301], 4, 60, key_dtype=torch.float32)
    rel = lambda snap: max(((ka.float() - kb.float()).norm() / kb.float().norm()).item() for ka, _, kb, _ in snap)
    e16, e32 = rel(snap16), rel(snap32)
    assert e32 < e16 / 3 and e32 < 5e-3, (e16, e32)


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_stale_rotation_is_caught(fused):
    """Negative control (test_cache.py:231-234): without re-rotation the check fails.
    A random-init model's logits are small, so the bar is relative to the logit scale."""
    model, ids = model_for(torch.float32, fused)
    got, want, _, _ = eviction_check(model, ids[:, :301], 4, 60, rerotate_keys=False)
    good, want2, _, _ = eviction_check(model, ids[:, :301], 4, 60)
    assert (got - want).abs().max().item() > 100 * max((good - want2).abs().max().item(), 1e-6)


def test_prefill_longer_than_cache():
    """A chunk longer than the cache gets full causal attention within itself; the cache is
    then trimmed (test_cache.py:237-249)."""
    model, ids = model_for(torch.float32, fused=True)
    ids = ids[:, :201]
    with torch.no_grad():
        dyn = model(ids[:, :200], past_key_values=DynamicCache(), use_cache=True).logits
    got, want, cache, _ = eviction_check(model, ids, 4, 60, prefill=200)
    assert cache.get_seq_length() == 64
    torch.testing.assert_close(got, want, rtol=0, atol=2e-3)
    with torch.no_grad():
        chunk = model(ids[:, :200], past_key_values=SinkCache.from_model(model, 4, 60), use_cache=True).logits
    torch.testing.assert_close(chunk, dyn, rtol=0, atol=0)


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_cuda_graph_replay_matches_eager(fused):
    """The graphed steady-state step runs the same kernels on the same buffers: bitwise
    (test_cache.py:252-265)."""
    model, ids = model_for(torch.bfloat16, fused)
    ids = ids[:, :260]
    eager = stream(model, ids, SinkCache.from_model(model, n_sink=4, window=60))
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    runner = StreamRunner(model, cache, use_graph=True)
    with torch.no_grad():
        out = [model(ids[:, :16], past_key_values=cache, use_cache=True).logits.float()]
        for t in range(16, ids.shape[1]):
            out.append(runner.step(ids[:, t:t + 1]).float().clone())
    assert runner.graph is not None and runner.replays > 100
    assert cache.tokens_seen == 260 and cache.tokens_evicted == 260 - 65
    torch.testing.assert_close(torch.cat(out, 1), eager, rtol=0, atol=0)


def test_cuda_graph_survives_chunks():
    """Chunks reallocate buffers between graphed steps; the runner recaptures
    (test_cache.py:268-284)."""
    model, ids = model_for(torch.bfloat16, fused=True)
    ids = ids[:, :301]
    plan = [16] + [1] * 120 + [30] + [1] * 80 + [45] + [1] * 10
    outs = {}
    for graphed in (False, True):
        cache = SinkCache.from_model(model, n_sink=4, window=60)
        runner = StreamRunner(model, cache, use_graph=graphed)
        out, t = [], 0
        with torch.no_grad():
            for n in plan:
                out.append(runner.step(ids[:, t:t + n]).float().clone())
                t += n
        outs[graphed] = torch.cat(out, 1)
    torch.testing.assert_close(outs[True], outs[False], rtol=0, atol=0)


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_streamed_nll_matches_reference(fused, golden, golden_arrays):
    """Per-token NLL of the tiny fp32 Qwen3 streamed through SinkCache(4, 60) vs the
    reference's own CPU run (fixture): mean within 0.5%, every token within 1e-3."""
    model, ids = model_for(torch.float32, fused)
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    runner = StreamRunner(model, cache)
    nll, logits = cases.stream_nll(model, ids, cache, prefill=16, step=runner.step)
    want = torch.from_numpy(golden_arrays["stream/nll"])
    assert abs(nll.mean().item() - golden["stream"]["mean_nll"]) < 5e-3 * golden["stream"]["mean_nll"]
    torch.testing.assert_close(nll, want, rtol=0, atol=1e-3)
    torch.testing.assert_close(logits, torch.from_numpy(golden_arrays["stream/last_logits"]), rtol=0, atol=2e-3)
    assert cache.tokens_evicted == golden["stream"]["tokens_evicted"]


def test_backend_in_model():
    """Qwen3 with the registered backend: decode runs the fused kernels, prefill SDPA; its
    logits are no further from an fp32 model than stock bf16 SDPA's (test_decode_attention.py:44-67)."""
    ids = cases.tiny_qwen3(torch.float32)[1].to(DEV)
    m32 = cases.tiny_qwen3(torch.float32, attn="sdpa")[0].to(DEV)
    m16 = cases.tiny_qwen3(torch.bfloat16, attn="sdpa")[0].to(DEV)
    mk = cases.tiny_qwen3(torch.bfloat16, attn=BACKEND)[0].to(DEV)
    before = dict(calls)

    def run(m, sink):
        cache = SinkCache.from_model(m, 4, 124) if sink else DynamicCache()
        with torch.no_grad():
            out = [m(ids[:, :200], past_key_values=cache, use_cache=True).logits[:, -1:]]
            for t in range(200, 264):
                out.append(m(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits)
        return torch.cat(out, 1).float()

    for sink in (False, True):
        ref, sdpa, kern = run(m32, sink), run(m16, sink), run(mk, sink)
        e_sdpa, e_kern = (sdpa - ref).abs().mean().item(), (kern - ref).abs().mean().item()
        assert e_kern <= 1.25 * e_sdpa, (sink, e_kern, e_sdpa)
    assert calls["fused_step"] > before["fused_step"]
    assert calls["decode_kernel"] > before["decode_kernel"]  # DynamicCache decode steps
    assert calls["sdpa_fallback"] > before["sdpa_fallback"]
