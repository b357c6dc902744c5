"""Case definitions and seeded input generators shared by the golden-fixture generator and
the tests.  Shapes and value distributions follow the reference's own tests
(tests/test_cache.py:130-152, tests/test_decode_attention.py:23-41, tests/test_rope.py) and
the op-bench / model configurations of the decode path; models are random-init (no
weights are available), tokens uniform from a seed."""

import torch

EVICT_GRID = [(4, 60, 1), (0, 60, 1), (4, 1020, 1), (4, 100, 37), (2, 7, 200)]
EVICT_CASES = [(dt, s, w, d) for dt in ("bf16", "fp32") for (s, w, d) in EVICT_GRID]
ATTN_SHAPES = [(16, 8, 128), (32, 8, 64), (8, 8, 128), (14, 2, 64)]
ATTN_LENS = [1, 63, 64, 1025, 4097, 32768]
STEP_CASES = [
    dict(batch=2, hq=16, hkv=8, d=128, slots=64, n_sink=4),
    dict(batch=3, hq=32, hkv=8, d=64, slots=100, n_sink=4),
    dict(batch=1, hq=16, hkv=8, d=128, slots=1024, n_sink=4),
    dict(batch=2, hq=14, hkv=2, d=64, slots=40, n_sink=0),
    dict(batch=1, hq=16, hkv=8, d=256, slots=48, n_sink=2),
]
DTYPES = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}


def inv_freq(dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))


def evict_name(dtype_name, n_sink, window, drop):
    return f"evict_{dtype_name}_{n_sink}_{window}_{drop}"


def evict_inputs(dtype_name, n_sink, window, drop):
    """[1, 8, n_sink + window + drop, 128] keys ~ 30 N(0,1), values N(0,1), seed = drop."""
    dtype = DTYPES[dtype_name]
    torch.manual_seed(drop)
    k = torch.randn(1, 8, n_sink + window + drop, 128, dtype=dtype) * 30
    v = torch.randn_like(k)
    return k, v, inv_freq(128, 1e6)


def attn_inputs(hq, hkv, d, seq_len):
    """q N(0,1), k 3 N(0,1), v N(0,1) in bf16, seed = seq_len."""
    torch.manual_seed(seq_len)
    q = torch.randn(1, hq, 1, d, dtype=torch.bfloat16)
    k = torch.randn(1, hkv, seq_len, d, dtype=torch.bfloat16) * 3
    v = torch.randn_like(k)
    return q, k, v


def step_name(batch, hq, hkv, d, slots, n_sink):
    return f"step_b{batch}_q{hq}_kv{hkv}_d{d}_s{slots}_n{n_sink}"


def rotated_keys(raw: torch.Tensor, positions: torch.Tensor, inv: torch.Tensor) -> torch.Tensor:
    """HF-convention RoPE of raw [B, H, T, D] at positions [T], fp32 math."""
    freqs = positions.float()[:, None] * inv
    emb = torch.cat((freqs, freqs), -1)
    x1, x2 = raw.float().chunk(2, -1)
    return raw.float() * emb.cos() + torch.cat((-x2, x1), -1) * emb.sin()


def step_inputs(batch, hq, hkv, d, slots, n_sink, seed=7):
    """A cache prefilled with slots + 1 rows (keys rotated at their positions, so one row is
    pending eviction) and one decode step's q, k, v -- all bf16."""
    g = torch.Generator().manual_seed(seed)
    inv = inv_freq(d, 1e6)
    k0 = rotated_keys(torch.randn(batch, hkv, slots + 1, d, generator=g), torch.arange(slots + 1), inv)
    v0 = torch.randn(batch, hkv, slots + 1, d, generator=g)
    k1 = rotated_keys(torch.randn(batch, hkv, 1, d, generator=g), torch.tensor([slots]), inv)
    v1 = torch.randn(batch, hkv, 1, d, generator=g)
    q = rotated_keys(torch.randn(batch, hq, 1, d, generator=g), torch.tensor([slots]), inv)
    bf = torch.bfloat16
    return dict(inv=inv, k0=k0.to(bf), v0=v0.to(bf), k1=k1.to(bf), v1=v1.to(bf), q=q.to(bf))


def tiny_qwen3_config():
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=128, rope_theta=1e6,
                       max_position_embeddings=4096, tie_word_embeddings=True, rms_norm_eps=1e-6)


def build_model(config, dtype, attn="sdpa", seed=0):
    from transformers import AutoModelForCausalLM
    torch.manual_seed(seed)
    model = AutoModelForCausalLM.from_config(config, attn_implementation=attn)
    return model.to(dtype).eval()


def tiny_qwen3(dtype, attn="sdpa", n_tokens=301):
    model = build_model(tiny_qwen3_config(), dtype, attn)
    ids = torch.randint(0, 512, (1, n_tokens), generator=torch.Generator().manual_seed(1))
    return model, ids


def qwen3_0_6b_config():
    from transformers import Qwen3Config
    return Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                       max_position_embeddings=40960, tie_word_embeddings=True, rms_norm_eps=1e-6,
                       initializer_range=0.02)


def qwen3_0_6b(steps, attn="sdpa", batch=1, seed=1):
    model = build_model(qwen3_0_6b_config(), torch.bfloat16, attn)
    ids = torch.randint(0, 151936, (batch, steps + 1), generator=torch.Generator().manual_seed(seed))
    return model, ids


def tiny_llama3_stream_config():
    """Llama-3.2 geometry (32 q / 8 kv heads, head_dim 64, theta 5e5, llama3 scaling), 2 layers."""
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=32, num_key_value_heads=8, head_dim=64, rope_theta=5e5,
                       rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                       max_position_embeddings=131072, tie_word_embeddings=True, rms_norm_eps=1e-5)


def tiny_llama3_stream(dtype, attn="sdpa", n_tokens=301, batch=2):
    model = build_model(tiny_llama3_stream_config(), dtype, attn)
    ids = torch.randint(0, 512, (batch, n_tokens), generator=torch.Generator().manual_seed(2))
    return model, ids


def tiny_llama3():
    from transformers import LlamaConfig
    cfg = LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=1,
                      num_attention_heads=4, num_key_value_heads=1, head_dim=64, rope_theta=5e5,
                      rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                      max_position_embeddings=131072)
    return build_model(cfg, torch.float32)


@torch.no_grad()
def stream_nll(model, ids, cache, prefill=16, step=None):
    """Prefill `prefill` tokens, then one token at a time; the NLL of every next token
    (the shape of experiments/ppl.py:70-84).  Returns (nll [n - prefill] fp32, last logits)."""
    import torch.nn.functional as F
    step = step or (lambda x: model(x, past_key_values=cache, use_cache=True).logits)
    logits = model(ids[:, :prefill], past_key_values=cache, use_cache=True).logits[:, -1]
    nll = [F.cross_entropy(logits.float(), ids[:, prefill])]
    for t in range(prefill, ids.shape[1] - 1):
        logits = step(ids[:, t:t + 1])[:, -1]
        nll.append(F.cross_entropy(logits.float(), ids[:, t + 1]))
    return torch.stack(nll).float().cpu(), logits[0].float().cpu()


# ------------------------------------------------------------------ ring-buffer (v2) layer

V2_CASES = [
    dict(name="v2_s4_w60_bf16", n_sink=4, window=60, dtype="bf16", plan=[16] + [1] * 150),
    dict(name="v2_s0_w60_bf16", n_sink=0, window=60, dtype="bf16", plan=[16] + [1] * 100),
    dict(name="v2_s1_w60_fp32", n_sink=1, window=60, dtype="fp32", plan=[16] + [1] * 100),
    dict(name="v2_pins", n_sink=4, window=60, dtype="bf16", pins=[(20, 30), (100, 105)], max_pinned=32,
         plan=[16] + [1] * 84 + [40] + [1] * 160),
    dict(name="v2_pin_budget", n_sink=4, window=60, dtype="bf16", pins=[(10, 16), (30, 36)], max_pinned=8,
         plan=[16] + [1] * 183),
    dict(name="v2_chunks", n_sink=4, window=60, dtype="bf16", plan=[200, 1, 1, 37, 90, 1, 1, 69]),
    dict(name="v2_partial_rot", n_sink=4, window=30, dtype="bf16", rot=64, plan=[8] + [1] * 60),
]
V2_ROTATION_WS = [64, 2_000_000, 50_000_000]


def v2_inputs(n_tokens, dtype_name, rot=128, batch=2, heads=2, d=128, seed=11):
    """Keys as a model writes them (rotated at their absolute positions, first `rot` dims),
    values N(0,1); [batch, heads, n_tokens, d] in the case dtype."""
    g = torch.Generator().manual_seed(seed)
    dtype = DTYPES[dtype_name]
    inv = inv_freq(rot, 1e6)
    raw = torch.randn(batch, heads, n_tokens, d, generator=g) * 3
    k = torch.cat((rotated_keys(raw[..., :rot], torch.arange(n_tokens), inv), raw[..., rot:]), -1)
    v = torch.randn(batch, heads, n_tokens, d, generator=g)
    return k.to(dtype), v.to(dtype), inv


def v2_rotation_inputs(seed=12):
    """Region keys at their original rotations and far-apart original positions."""
    g = torch.Generator().manual_seed(seed)
    reg_k = (torch.randn(1, 8, 6, 128, generator=g) * 30).to(torch.bfloat16)
    return reg_k, [0, 1, 2, 3, 500_000, 1_200_000], inv_freq(128, 1e6)
