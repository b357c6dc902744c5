"""A CUDA graph captured before any eager launch of the library in the process: a v2 cache
is steady right after its fill, so StreamRunner's very first one-token step is a capture.
The library's one-time device set-up (kernel shared-memory opt-ins, the tensor-map encoder
lookup) must already have run -- the caches do it at lazy initialisation.  Runs in a fresh
process so that no earlier test has prepared the device."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r'''
import torch
from attention_sinks_b200 import SinkCacheV2, StreamRunner, register
from tests.golden import cases
name = register()
model, ids = cases.tiny_qwen3(torch.bfloat16, attn=name, n_tokens=120)
model, ids = model.cuda(), ids.cuda()
outs = {}
for graphed in (True, False):
    cache = SinkCacheV2.from_model(model, n_sink=4, window=60)
    runner = StreamRunner(model, cache, use_graph=graphed)
    with torch.no_grad():
        model(ids[:, :64], past_key_values=cache, use_cache=True)   # fills the cache: steady
        assert cache.is_steady
        outs[graphed] = torch.cat([runner.step(ids[:, t:t + 1]).float().clone() for t in range(64, 120)], 1)
    if graphed:
        assert runner.replays == 55, runner.replays
torch.testing.assert_close(outs[True], outs[False], rtol=0, atol=0)
print("ok")
'''


def test_first_step_is_a_capture():
    r = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
