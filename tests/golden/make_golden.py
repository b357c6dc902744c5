"""Generate the golden fixtures by running the reference itself (buttaRahul/Attention_sinks,
imported from its source tree) on the CPU.

    SINKCACHE_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py [--config1 N]
    python tests/golden/make_golden.py --reference <reference checkout>/src [--config1 N]

Writes tests/golden/golden.json (known answers, digests) and tests/golden/arrays.npz
(small output arrays).  The reference is pure Python; its PyTorch eviction path and the
SDPA attention fallback are what run on the CPU.  Installed transformers 5.5.0 declares
`get_max_cache_shape` abstract where the reference implements `get_max_length`; the shim
below aliases it (harness only, the reference source is not modified).

Inputs are regenerated from seeds by the tests (torch's CPU generator is deterministic);
their digests are recorded so a test can tell an RNG difference from a real mismatch.
"""

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases  # noqa: E402


def digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()


def load_reference(path: str):
    sys.path.insert(0, path)
    import sinkcache.cache as rc  # noqa: F401
    from sinkcache.cache import SinkLayer
    from sinkcache.cache_v2 import SinkLayerV2
    for cls in (SinkLayer, SinkLayerV2):
        cls.get_max_cache_shape = cls.get_max_length
        cls.__abstractmethods__ = frozenset()
    import sinkcache
    return sinkcache


def v2_causal_chunk_mask(layer_cls):
    """Harness shim for the v2 layer under the installed transformers 5.5.0, which places a
    chunk's queries at get_seq_length() (the absolute position, for a v2 layer) when it builds
    the causal mask: returning kv_offset = t - in_cache_length makes chunk query i see chunk
    keys 0..i and every cached key -- the causal mask the reference gets under the
    transformers it pins (its SinkCacheV2.get_query_offset).  Decode steps are unaffected."""
    def get_mask_sizes(self, query_length):
        n = self.in_cache_length()
        return n + query_length, self.t - n
    layer_cls.get_mask_sizes = get_mask_sizes


def evict_cases(ref, out, arrays):
    from sinkcache.cache import SinkLayer
    res = {}
    for dtype_name, n_sink, window, drop in cases.EVICT_CASES:
        k, v, inv = cases.evict_inputs(dtype_name, n_sink, window, drop)
        layer = SinkLayer(n_sink, window, inv, use_triton=False)  # key_dtype None: model dtype
        layer.update(k, v)
        layer._evict_pending()
        assert not layer.use_triton
        cap = n_sink + window
        kk, vv = layer._kbuf[:, :, :cap], layer._vbuf[:, :, :cap]
        name = cases.evict_name(dtype_name, n_sink, window, drop)
        res[name] = {"in_k": digest(k), "in_v": digest(v), "k": digest(kk), "v": digest(vv),
                     "length": layer.length, "tokens_evicted": layer.tokens_evicted}
        arrays[name + "/k_rowsum"] = kk.double().sum(-1).numpy()
    out["evict"] = res


def rerotate_cases(ref, out, arrays):
    from sinkcache.cache import SinkLayer
    from sinkcache.rope import apply_rope, rerotate
    res = {}
    # cache.py fast path == rope.rerotate (tests/test_cache.py:155-165 of the reference)
    torch.manual_seed(0)
    inv = cases.inv_freq(128, 1e6)
    layer = SinkLayer(4, 60, inv)
    layer.device = "cpu"
    layer.inv_freq = inv
    k = torch.randn(1, 8, 60, 128, dtype=torch.bfloat16)
    res["fast_input"] = digest(k)
    for d in (1, 5, 300):
        fast = layer._rerotate(k, d)
        res[f"fast_{d}"] = digest(fast)
        res[f"slow_{d}"] = digest(rerotate(k, d, inv))
    # rerotation identity (tests/test_rope.py:30-41 of the reference)
    for p in (5, 1024, 40_000):
        for delta in (1, 7, 1000):
            torch.manual_seed(p + delta)
            kk = torch.randn(1, 8, 16, 128)
            pos = torch.arange(p, p + 16) + delta
            shifted = rerotate(apply_rope(kk, pos, inv), delta, inv)
            direct = apply_rope(kk, pos - delta, inv)
            res[f"identity_{p}_{delta}"] = {"shifted": digest(shifted), "direct": digest(direct),
                                            "max_abs_diff": float((shifted - direct).abs().max())}
    out["rerotate"] = res


class _Module:
    """Stand-in for an HF attention module: what sdpa_attention_forward reads."""

    def __init__(self, groups):
        self.num_key_value_groups = groups
        self.is_causal = True
        self.training = False


def attention_cases(ref, out, arrays):
    from sinkcache.decode_attention import decode_attention_forward
    res = {}
    for hq, hkv, d in cases.ATTN_SHAPES:
        for seq_len in cases.ATTN_LENS:
            q, k, v = cases.attn_inputs(hq, hkv, d, seq_len)
            o, _ = decode_attention_forward(_Module(hq // hkv), q, k, v, None, scaling=d ** -0.5)
            name = f"attn_{hq}_{hkv}_{d}_{seq_len}"
            res[name] = {"in_q": digest(q), "in_k": digest(k), "in_v": digest(v)}
            arrays[name] = o.float().numpy()
    out["attention"] = res


def step_cases(ref, out, arrays):
    """A SinkLayer decode step on the CPU path: update (evict pending + append) then the
    attention fallback, for a few small op-bench shapes."""
    from sinkcache.cache import SinkLayer
    from sinkcache.decode_attention import decode_attention_forward
    res = {}
    for spec in cases.STEP_CASES:
        st = cases.step_inputs(**spec)
        layer = SinkLayer(spec["n_sink"], spec["slots"] - spec["n_sink"], st["inv"], key_dtype=torch.float32)
        layer.update(st["k0"], st["v0"])  # prefill slots + 1 rows: one pending eviction
        keys, values = layer.update(st["k1"], st["v1"])
        o, _ = decode_attention_forward(_Module(spec["hq"] // spec["hkv"]), st["q"], keys, values, None,
                                        scaling=spec["d"] ** -0.5)
        name = cases.step_name(**spec)
        kk, vv = layer._kbuf, layer._vbuf
        res[name] = {"in_k0": digest(st["k0"]), "k": digest(kk), "v": digest(vv), "length": layer.length,
                     "tokens_seen": layer.tokens_seen, "tokens_evicted": layer.tokens_evicted}
        arrays[name + "/out"] = o.float().numpy()
        arrays[name + "/k_rowsum"] = kk.double().sum(-1).numpy()
    out["step"] = res


def stream_case(ref, out, arrays):
    """Tiny random-init Qwen3 streamed through the reference SinkCache (4, 60): the
    bookkeeping known answers of tests/test_cache.py:117-127 and the per-token NLL."""
    from sinkcache import SinkCache
    model, ids = cases.tiny_qwen3(torch.float32)
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    nll, logits = cases.stream_nll(model, ids, cache, prefill=16)
    layer = cache.layers[0]
    kept = [l.kept() for l in cache.layers]
    out["stream"] = {
        "seq_length": cache.get_seq_length(), "is_steady": bool(cache.is_steady),
        "tokens_seen": cache.tokens_seen, "tokens_evicted": cache.tokens_evicted,
        "kept_rows": [int(k.shape[-2]) for k, _ in kept], "buffer_slots": int(layer._kbuf.shape[-2]),
        "mean_nll": float(nll.mean()), "ids": digest(ids),
    }
    arrays["stream/nll"] = nll.numpy()
    arrays["stream/last_logits"] = logits.numpy()
    arrays["stream/kept_k_rowsum"] = np.stack([k.double().sum(-1).numpy() for k, _ in kept])


def llama_stream_case(ref, out, arrays):
    """Tiny Llama-3.2-shaped model (llama3 rope scaling, GQA 4, head_dim 64), batch 2,
    streamed through the reference SinkCache (4, 60): per-token NLL of both streams."""
    from sinkcache import SinkCache
    model, ids = cases.tiny_llama3_stream(torch.float32)
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    nll = []
    import torch.nn.functional as F
    with torch.no_grad():
        logits = model(ids[:, :16], past_key_values=cache, use_cache=True).logits[:, -1]
        nll.append(F.cross_entropy(logits.float(), ids[:, 16], reduction="none"))
        for t in range(16, ids.shape[1] - 1):
            logits = model(ids[:, t:t + 1], past_key_values=cache, use_cache=True).logits[:, -1]
            nll.append(F.cross_entropy(logits.float(), ids[:, t + 1], reduction="none"))
    nll = torch.stack(nll, 1)
    out["llama_stream"] = {"mean_nll": float(nll.mean()), "tokens_evicted": cache.tokens_evicted,
                           "ids": digest(ids)}
    arrays["llama_stream/nll"] = nll.numpy()
    arrays["llama_stream/last_logits"] = logits.float().numpy()


def v2_layer_cases(ref, out, arrays):
    """The reference SinkLayerV2 driven directly with seeded K/V chunks (cache_v2.py:159-208):
    after every segment of the plan, the logical cache (kept(): keys, values, positions) and
    the bookkeeping; the K/V the last step returned."""
    from sinkcache.cache_v2 import SinkLayerV2
    res = {}
    for spec in cases.V2_CASES:
        rot = spec.get("rot", 128)
        total = sum(spec["plan"])
        k, v, inv = cases.v2_inputs(total, spec["dtype"], rot)
        pinned = set()
        for a, b in spec.get("pins", []):
            pinned.update(range(a, b))
        layer = SinkLayerV2(spec["n_sink"], spec["window"], inv, spec.get("max_pinned", 0), pinned)
        t, marks = 0, []
        segments = []  # (start, n) runs of equal-size steps
        for n in spec["plan"]:
            if segments and n == 1 and segments[-1][1] == 1:
                segments[-1][2] += 1
            else:
                segments.append([t, n, 1])
            t += n
        t = 0
        for start, n, reps in segments:
            for _ in range(reps):
                keys, values = layer.update(k[:, :, t:t + n], v[:, :, t:t + n])
                t += n
            kk, vv, pos = layer.kept()
            marks.append({"t": layer.t, "kept_k": digest(kk), "kept_v": digest(vv), "positions": pos,
                          "region_pos": list(layer.region_pos), "moved_upto": layer.moved_upto,
                          "pins_dropped": layer.pins_dropped, "in_cache": layer.in_cache_length(),
                          "step_k": digest(keys), "step_v": digest(values),
                          "step_rows": int(keys.shape[-2])})
        res[spec["name"]] = {"in_k": digest(k), "in_v": digest(v), "marks": marks}
        arrays[spec["name"] + "/kept_k_rowsum"] = kk.double().sum(-1).numpy()
    # the region rotation alone, far from the origin (fp64 angles): _rotate_region(ws)
    reg_k, reg_pos, inv = cases.v2_rotation_inputs()
    layer = SinkLayerV2(4, 60, inv, max_pinned=2)
    layer.lazy_initialization(reg_k[:, :, :1], reg_k[:, :, :1])
    layer._reg_k[:, :, :6] = reg_k
    layer._reg_pos[:6] = torch.tensor(reg_pos)
    layer.region_pos = list(reg_pos)
    rot = {"in_k": digest(reg_k)}
    for ws in cases.V2_ROTATION_WS:
        rot[f"ws_{ws}"] = digest(layer._rotate_region(ws))
    res["rotation"] = rot
    out["v2"] = res


def v2_stream_case(ref, out, arrays):
    """Tiny random-init Qwen3 (fp32) streamed through the reference SinkCacheV2(4, 60): prefill
    16, then one token at a time; per-token NLL and bookkeeping."""
    from sinkcache.cache_v2 import SinkCacheV2, SinkLayerV2
    v2_causal_chunk_mask(SinkLayerV2)
    model, ids = cases.tiny_qwen3(torch.float32)
    cache = SinkCacheV2.from_model(model, n_sink=4, window=60)
    nll, logits = cases.stream_nll(model, ids, cache, prefill=16)
    out["v2_stream"] = {"tokens_seen": cache.tokens_seen, "tokens_evicted": cache.tokens_evicted,
                        "region_size": cache.region_size, "mean_nll": float(nll.mean()), "ids": digest(ids)}
    arrays["v2_stream/nll"] = nll.numpy()
    arrays["v2_stream/last_logits"] = logits.numpy()


def inv_freq_case(ref, out, arrays):
    """find_inv_freq on a Llama-3.2-1B-shaped config with llama3 rope scaling."""
    from sinkcache.cache import find_inv_freq
    model = cases.tiny_llama3()
    arrays["llama3_inv_freq"] = find_inv_freq(model).numpy()
    out["llama3_inv_freq"] = {"n": int(arrays["llama3_inv_freq"].shape[0])}


def config1_case(ref, out, arrays, steps):
    """Random-init Qwen3-0.6B, SinkCache(4, 1020), batch 1, uniform tokens, streamed one token
    at a time on the reference CPU path: per-step NLL series."""
    from sinkcache import SinkCache
    model, ids = cases.qwen3_0_6b(steps)
    cache = SinkCache.from_model(model, n_sink=4, window=1020)
    t0 = time.time()
    nll, _ = cases.stream_nll(model, ids, cache, prefill=1)
    out["config1"] = {"steps": steps, "mean_nll": float(nll.mean()), "seconds": time.time() - t0,
                      "threads": torch.get_num_threads(), "ids": digest(ids),
                      "tokens_evicted": cache.tokens_evicted}
    arrays["config1/nll"] = nll.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SINKCACHE_REFERENCE_SRC"),
                    help="the reference's src/ directory (default: $SINKCACHE_REFERENCE_SRC)")
    ap.add_argument("--config1", type=int, default=0, help="also stream N steps of random-init Qwen3-0.6B")
    ap.add_argument("--only", default="", help="comma-separated case functions to regenerate (default: all)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference's src/ directory with --reference or SINKCACHE_REFERENCE_SRC")
    ref = load_reference(args.reference)
    json_path = os.path.join(HERE, "golden.json")
    npz_path = os.path.join(HERE, "arrays.npz")
    out = json.load(open(json_path)) if os.path.exists(json_path) else {}
    arrays = dict(np.load(npz_path)) if os.path.exists(npz_path) else {}
    out["meta"] = {"torch": torch.__version__, "reference": "buttaRahul/Attention_sinks src/sinkcache",
                   "transformers": __import__("transformers").__version__}
    ap_only = args.only.split(",") if args.only else None
    for fn in (evict_cases, rerotate_cases, attention_cases, step_cases, stream_case, llama_stream_case,
               inv_freq_case, v2_layer_cases, v2_stream_case):
        if ap_only and fn.__name__ not in ap_only:
            continue
        t0 = time.time()
        fn(ref, out, arrays)
        print(f"{fn.__name__}: {time.time() - t0:.1f}s", flush=True)
    if args.config1:
        config1_case(ref, out, arrays, args.config1)
    with open(json_path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    np.savez_compressed(npz_path, **arrays)
    print("wrote", json_path, npz_path)


if __name__ == "__main__":
    main()
