"""The CPU oracle against the golden fixtures recorded from the reference itself
(tests/golden/make_golden.py).  Bit-exact where the reference's CPU arithmetic is
reproduced op for op; otherwise within the reference tests' tolerances."""

import numpy as np
import pytest
import torch

import oracle
from tests.golden import cases
from tests.util import digest


def _inputs_match(want: dict, **tensors) -> None:
    for key, t in tensors.items():
        if digest(t) != want[key]:
            pytest.skip(f"seeded input {key} differs from the fixture's (torch RNG changed)")


@pytest.mark.parametrize("case", cases.EVICT_CASES, ids=lambda c: cases.evict_name(*c))
def test_oracle_eviction_matches_reference(case, golden, golden_arrays):
    """cache.py:129-147 (PyTorch branch) restated: K and V identical to the reference's."""
    dtype_name, n_sink, window, drop = case
    name = cases.evict_name(*case)
    want = golden["evict"][name]
    k, v, inv = cases.evict_inputs(*case)
    _inputs_match(want, in_k=k, in_v=v)
    layer = oracle.OracleSinkLayer(n_sink, window, inv, key_dtype=None)
    layer.update(k, v)
    layer.evict_pending()
    cap = n_sink + window
    kk, vv = layer.kbuf[:, :, :cap], layer.vbuf[:, :, :cap]
    assert layer.length == want["length"] and layer.tokens_evicted == want["tokens_evicted"]
    assert digest(vv) == want["v"]  # values only move
    if digest(kk) != want["k"]:  # a CPU whose vector unit rounds the fused add differently
        np.testing.assert_allclose(kk.double().sum(-1).numpy(), golden_arrays[name + "/k_rowsum"],
                                   rtol=1e-5, atol=1e-3)


def test_oracle_rerotate_matches_reference(golden):
    """cache.py:116-127 and rope.py:49-54 restated."""
    want = golden["rerotate"]
    torch.manual_seed(0)
    inv = cases.inv_freq(128, 1e6)
    k = torch.randn(1, 8, 60, 128, dtype=torch.bfloat16)
    _inputs_match(want, fast_input=k)
    for d in (1, 5, 300):
        assert digest(oracle.rerotate_fast(k, d, inv)) == want[f"fast_{d}"]
        assert digest(oracle.rerotate(k, d, inv)) == want[f"slow_{d}"]
        # the two reference formulations agree once rounded to bf16 (test_cache.py:155-165),
        # to within one rounding where the CPU fuses the product-add of the fast path
        fast, slow = oracle.rerotate_fast(k, d, inv).to(k.dtype), oracle.rerotate(k, d, inv)
        assert (fast != slow).float().mean().item() < 1e-3
        torch.testing.assert_close(fast.float(), slow.float(), rtol=2 ** -7, atol=2 ** -7 * slow.abs().max().item())


@pytest.mark.parametrize("p", [5, 1024, 40_000])
@pytest.mark.parametrize("delta", [1, 7, 1000])
def test_oracle_rerotation_identity(p, delta, golden):
    """rope(k, p) rotated by -delta == rope(k, p - delta) (tests/test_rope.py:30-41)."""
    want = golden["rerotate"][f"identity_{p}_{delta}"]
    inv = cases.inv_freq(128, 1e6)
    torch.manual_seed(p + delta)
    k = torch.randn(1, 8, 16, 128)
    pos = torch.arange(p, p + 16) + delta
    shifted = oracle.rerotate(oracle.apply_rope(k, pos, inv), delta, inv)
    direct = oracle.apply_rope(k, pos - delta, inv)
    assert digest(shifted) == want["shifted"] and digest(direct) == want["direct"]
    torch.testing.assert_close(shifted, direct, rtol=0, atol=4e-7 * (p + delta + 16) + 1e-6)


@pytest.mark.parametrize("shape", cases.ATTN_SHAPES, ids=lambda s: "_".join(map(str, s)))
@pytest.mark.parametrize("seq_len", cases.ATTN_LENS)
def test_oracle_attention_matches_reference(shape, seq_len, golden, golden_arrays):
    """decode attention: the reference's CPU path (SDPA fallback over bf16 K/V) vs the
    oracle's fp32 softmax; tolerance of tests/test_decode_attention.py:23-31."""
    hq, hkv, d = shape
    name = f"attn_{hq}_{hkv}_{d}_{seq_len}"
    q, k, v = cases.attn_inputs(hq, hkv, d, seq_len)
    _inputs_match(golden["attention"][name], in_q=q, in_k=k, in_v=v)
    got = oracle.decode_attention(q, k, v, d ** -0.5)
    torch.testing.assert_close(got, torch.from_numpy(golden_arrays[name]), rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("spec", cases.STEP_CASES, ids=lambda s: cases.step_name(**s))
def test_oracle_decode_step_matches_reference(spec, golden, golden_arrays):
    """SinkLayer.update (evict + append) + attention, one decode step."""
    name = cases.step_name(**spec)
    want = golden["step"][name]
    st = cases.step_inputs(**spec)
    _inputs_match(want, in_k0=st["k0"])
    layer = oracle.OracleSinkLayer(spec["n_sink"], spec["slots"] - spec["n_sink"], st["inv"])
    layer.update(st["k0"], st["v0"])
    out = oracle.decode_step(layer, st["q"], st["k1"], st["v1"], spec["d"] ** -0.5)
    assert (layer.length, layer.tokens_seen, layer.tokens_evicted) == (
        want["length"], want["tokens_seen"], want["tokens_evicted"])
    assert digest(layer.vbuf) == want["v"]
    if digest(layer.kbuf) != want["k"]:
        np.testing.assert_allclose(layer.kbuf.double().sum(-1).numpy(), golden_arrays[name + "/k_rowsum"],
                                   rtol=1e-5, atol=1e-3)
    torch.testing.assert_close(out, torch.from_numpy(golden_arrays[name + "/out"]), rtol=2e-2, atol=1e-2)


def test_oracle_bookkeeping_known_answers(golden):
    """tests/test_cache.py:117-127 of the reference: 300 tokens through (4, 60), prefill 16.
    The fixture holds what the reference reported on a random-init Qwen3; the oracle layer
    fed the same update sequence reports the same counters."""
    want = golden["stream"]
    assert want["seq_length"] == 64 and want["is_steady"]
    assert want["tokens_seen"] == 300 and want["tokens_evicted"] == 235
    assert want["kept_rows"] == [64, 64] and want["buffer_slots"] == 65
    layer = oracle.OracleSinkLayer(4, 60, cases.inv_freq(128, 1e6))
    g = torch.Generator().manual_seed(0)
    plan = [16] + [1] * 284
    for n in plan:
        layer.update(torch.randn(1, 2, n, 128, generator=g).bfloat16(),
                     torch.randn(1, 2, n, 128, generator=g).bfloat16())
    assert layer.get_seq_length() == want["seq_length"]
    assert layer.tokens_seen == want["tokens_seen"] and layer.tokens_evicted == want["tokens_evicted"]
    assert layer.kbuf.shape[-2] == want["buffer_slots"]
    assert layer.kept()[0].shape[-2] == want["kept_rows"][0]


def test_find_inv_freq_llama3_scaling(golden_arrays):
    """find_inv_freq returns the post-scaling (llama3) inverse frequencies (cache.py:201-206)."""
    from attention_sinks_b200 import find_inv_freq
    model = cases.tiny_llama3()
    got = find_inv_freq(model).numpy()
    np.testing.assert_array_equal(got, golden_arrays["llama3_inv_freq"])
    plain = cases.inv_freq(64, 5e5).numpy()
    assert not np.array_equal(got, plain)  # the scaling changed the low frequencies


# ------------------------------------------------------------------ ring-buffer (v2) layer


def drive_v2(layer, spec, k, v):
    """Feed the plan's chunks; after each run of equal steps, yield (keys, values) of the
    last step (the segments make_golden.py records)."""
    t, segments = 0, []
    for n in spec["plan"]:
        if segments and n == 1 and segments[-1][1] == 1:
            segments[-1][2] += 1
        else:
            segments.append([t, n, 1])
        t += n
    t = 0
    for _start, n, reps in segments:
        for _ in range(reps):
            keys, values = layer.update(k[:, :, t:t + n], v[:, :, t:t + n])
            t += n
        yield keys, values


def v2_pinned(spec):
    pinned = set()
    for a, b in spec.get("pins", []):
        pinned.update(range(a, b))
    return pinned


@pytest.mark.parametrize("spec", cases.V2_CASES, ids=lambda s: s["name"])
def test_oracle_v2_layer_matches_reference(spec, golden):
    """cache_v2.py:59-248 restated: ring slots, region rotation with fp64 angles, pins moving
    into the region and the pin budget -- every checkpoint bit-identical to the reference."""
    want = golden["v2"][spec["name"]]
    k, v, inv = cases.v2_inputs(sum(spec["plan"]), spec["dtype"], spec.get("rot", 128))
    _inputs_match(want, in_k=k, in_v=v)
    layer = oracle.OracleSinkLayerV2(spec["n_sink"], spec["window"], inv, spec.get("max_pinned", 0),
                                     v2_pinned(spec))
    for (keys, values), mark in zip(drive_v2(layer, spec, k, v), want["marks"], strict=True):
        kk, vv, pos = layer.kept()
        assert layer.t == mark["t"] and pos == mark["positions"]
        assert layer.region_pos == mark["region_pos"] and layer.pins_dropped == mark["pins_dropped"]
        assert layer.moved_upto == mark["moved_upto"] and layer.in_cache_length() == mark["in_cache"]
        assert keys.shape[-2] == mark["step_rows"]
        assert digest(vv) == mark["kept_v"] and digest(values) == mark["step_v"]
        assert digest(kk) == mark["kept_k"] and digest(keys) == mark["step_k"]


def test_oracle_v2_region_rotation_far_positions(golden):
    """_rotate_region at window starts up to 5e7 (fp64 angles): bit-identical."""
    want = golden["v2"]["rotation"]
    reg_k, reg_pos, inv = cases.v2_rotation_inputs()
    _inputs_match(want, in_k=reg_k)
    for ws in cases.V2_ROTATION_WS:
        assert digest(oracle.region_rotation(reg_k, reg_pos, ws, inv)) == want[f"ws_{ws}"]
