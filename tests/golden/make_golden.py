"""Generate the golden fixtures by running the reference itself (buttaRahul/Attention_sinks,
imported from its source tree) on the CPU.

    python tests/golden/make_golden.py [--reference /root/reference/src] [--config1]

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
    SinkLayer.get_max_cache_shape = SinkLayer.get_max_length
    SinkLayer.__abstractmethods__ = frozenset()
    import sinkcache
    return sinkcache


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
    ap.add_argument("--reference", default="/root/reference/src")
    ap.add_argument("--config1", type=int, default=0, help="also stream N steps of random-init Qwen3-0.6B")
    args = ap.parse_args()
    ref = load_reference(args.reference)
    json_path = os.path.join(HERE, "golden.json")
    npz_path = os.path.join(HERE, "arrays.npz")
    out = json.load(open(json_path)) if os.path.exists(json_path) else {}
    arrays = dict(np.load(npz_path)) if os.path.exists(npz_path) else {}
    out["meta"] = {"torch": torch.__version__, "reference": "buttaRahul/Attention_sinks src/sinkcache",
                   "transformers": __import__("transformers").__version__}
    for fn in (evict_cases, rerotate_cases, attention_cases, step_cases, stream_case, llama_stream_case,
               inv_freq_case):
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
