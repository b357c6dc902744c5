"""Streamed-NLL parity at model level against the reference's own CPU runs (fixtures):
random-init Qwen3-0.6B with SinkCache(4, 1020) over 4,096 one-token steps (so
eviction and re-rotation fire from step 1,025 on) and a Llama-3.2-shaped model (llama3
rope scaling, head_dim 64, GQA 4, batch 2).  Both run the fused kernels under the
CUDA-graph StreamRunner.  Target: mean NLL within 0.5 % of the reference's."""

import pytest
import torch
import torch.nn.functional as F

from attention_sinks_b200 import SinkCache, StreamRunner, register
from attention_sinks_b200.decode_attention import calls
from tests.golden import cases
from tests.util import digest

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_qwen3_streamed_nll_matches_reference(golden, golden_arrays):
    want_meta = golden["config1"]
    steps = want_meta["steps"]
    name = register()
    model, ids = cases.qwen3_0_6b(steps, attn=name)
    assert digest(ids) == want_meta["ids"]
    model, ids = model.to(DEV), ids.to(DEV)
    cache = SinkCache.from_model(model, n_sink=4, window=1020)
    runner = StreamRunner(model, cache)
    before = calls["fused_step"]
    nll, _ = cases.stream_nll(model, ids, cache, prefill=1, step=runner.step)
    want = torch.from_numpy(golden_arrays["config1/nll"])
    assert nll.shape == want.shape
    rel = abs(nll.mean().item() - want.mean().item()) / want.mean().item()
    rel_evicting = abs(nll[1024:].mean().item() - want[1024:].mean().item()) / want[1024:].mean().item()
    diff = (nll - want).abs()
    print(f"qwen3-0.6b 4+1020: mean NLL {nll.mean():.5f} vs reference {want.mean():.5f} (rel {rel:.2e}; "
          f"evicting steps rel {rel_evicting:.2e}); per-token |d| mean {diff.mean():.4f} max {diff.max():.4f}")
    assert rel < 5e-3 and rel_evicting < 5e-3
    assert cache.tokens_evicted == want_meta["tokens_evicted"]
    assert runner.replays > steps - 1100 and calls["fused_step"] > before
    assert cache.workspace.read_status() == 0


@pytest.mark.parametrize("fused", [False, True], ids=["unfused", "fused"])
def test_llama3_stream_matches_reference(fused, golden, golden_arrays):
    model, ids = cases.tiny_llama3_stream(torch.float32, attn=register() if fused else "sdpa")
    assert digest(ids) == golden["llama_stream"]["ids"]
    model, ids = model.to(DEV), ids.to(DEV)
    cache = SinkCache.from_model(model, n_sink=4, window=60)
    runner = StreamRunner(model, cache)
    nll = []
    with torch.no_grad():
        logits = model(ids[:, :16], past_key_values=cache, use_cache=True).logits[:, -1]
        nll.append(F.cross_entropy(logits.float(), ids[:, 16], reduction="none"))
        for t in range(16, ids.shape[1] - 1):
            logits = runner.step(ids[:, t:t + 1])[:, -1]
            nll.append(F.cross_entropy(logits.float(), ids[:, t + 1], reduction="none"))
    nll = torch.stack(nll, 1).cpu()
    want = torch.from_numpy(golden_arrays["llama_stream/nll"])
    torch.testing.assert_close(nll, want, rtol=0, atol=1e-3)
    assert abs(nll.mean().item() - want.mean().item()) < 5e-3 * want.mean().item()
    torch.testing.assert_close(logits.float().cpu(), torch.from_numpy(golden_arrays["llama_stream/last_logits"]),
                               rtol=0, atol=2e-3)
    assert cache.tokens_evicted == golden["llama_stream"]["tokens_evicted"]
