"""The fused decode step in the exact regime of the headline op-bench line: 32,768 slots,
one Qwen3-0.6B attention layer (16 query heads, 8 KV heads, head_dim 128), fp32 K / bf16 V,
n_sink 4.  At 8 and 64 streams (and with a 37-row shift) the plan is unclustered and
multi-split, so the step is the halo pre-pass, the stream kernel and the split combine --
the three launches whose time the bench reports.

Checks, per the reference's tolerances (src/sinkcache/cache.py:129-165 for the step,
tests/test_cache.py:130-152 and tests/test_decode_attention.py:23-41 for the tolerances):
  * three streams spread over the batch against the CPU oracle of SinkLayer.update: V bit
    for bit, K bit for bit (sha256 of the fp32 rows), the output within 2e-2 abs of the
    reference's attention over its bf16 key copy and of fp32 attention over the updated
    cache;
  * every stream of the batch (size-independent properties): V equals the shifted input
    bit for bit, K equals a GPU re-rotation of the shifted input within one fp32 rounding,
    rows past the written range are untouched, and the kernels' status word is clean.
"""

import pytest
import torch

import oracle
from attention_sinks_b200 import _lib
from tests.golden import cases
from tests.util import digest

pytestmark = pytest.mark.gpu
DEV = "cuda"
HQ, HKV, D, N_SINK, SLOTS = 16, 8, 128, 4, 32768


def _state(streams: int, drop: int):
    """K (fp32, rotated at positions 0..rows-1), V, and one step's q / k / v, every stream
    from its own seed."""
    rows = SLOTS + drop
    inv = cases.inv_freq(D, 1e6)
    k = torch.empty(streams, HKV, rows, D, device=DEV)
    v = torch.empty(streams, HKV, rows, D, dtype=torch.bfloat16, device=DEV)
    pos = torch.arange(rows, device=DEV)
    for s in range(streams):
        g = torch.Generator(device=DEV).manual_seed(100 + s)
        k[s] = cases.rotated_keys(torch.randn(1, HKV, rows, D, device=DEV, generator=g), pos, inv.to(DEV))[0]
        v[s] = torch.randn(HKV, rows, D, device=DEV, generator=g).bfloat16()
    g = torch.Generator(device=DEV).manual_seed(7)
    q = torch.randn(streams, HQ, 1, D, device=DEV, generator=g).bfloat16()
    k1 = torch.randn(streams, HKV, 1, D, device=DEV, generator=g).bfloat16()
    v1 = torch.randn(streams, HKV, 1, D, device=DEV, generator=g).bfloat16()
    return inv, k, v, q, k1, v1


@pytest.mark.parametrize("streams,drop,probe", [
    (8, 1, (0, 3, 7)),
    (64, 1, (0, 31, 63)),
    (8, 37, (0, 5, 7)),
], ids=["s32768_b8_drop1", "s32768_b64_drop1", "s32768_b8_drop37"])
def test_headline_fused_step_matches_oracle(streams, drop, probe, built_lib):
    window = SLOTS - N_SINK
    sms = _lib.sm_count(torch.device(DEV))
    plan = _lib.plan(_lib.OP_FUSED_STEP, streams, HKV, HQ, D, torch.float32, torch.bfloat16, SLOTS + 1,
                     N_SINK, window, drop, sms)
    # the bench's regime: several splits per pair, no cluster -> halo pre-pass + combine launch
    assert plan["splits"] > 1 and plan["cluster_ctas"] == 1
    if drop > 1:
        assert drop > 4  # more than a cluster stages: the workspace halo path

    inv, k, v, q, k1, v1 = _state(streams, drop)
    k_in = {s: k[s:s + 1].cpu() for s in probe}
    v_in = {s: v[s:s + 1].cpu() for s in probe}
    cos, sin = oracle.rope_cos_sin(torch.tensor(-drop), inv)
    out = torch.empty(streams, 1, HQ, D, dtype=torch.bfloat16, device=DEV)
    ws = _lib.Workspace()
    _lib.fused_decode_step(k, v, k1, v1, q, N_SINK, window, drop, SLOTS, cos.to(DEV), sin.to(DEV),
                           D ** -0.5, out, ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0

    # --- the oracle on a few streams: bit-exact cache, output within 2e-2 abs
    for s in probe:
        want = oracle.OracleSinkLayer(N_SINK, window, inv)
        want.dtype = torch.bfloat16
        want.kbuf, want.vbuf, want.length = k_in[s].clone(), v_in[s].clone(), SLOTS + drop
        keys, values = want.update(k1[s:s + 1].cpu(), v1[s:s + 1].cpu())
        want_out = oracle.decode_attention(q[s:s + 1].cpu(), keys, values, D ** -0.5)
        got_k, got_v = k[s:s + 1, :, :SLOTS + 1].cpu(), v[s:s + 1, :, :SLOTS + 1].cpu()
        assert want.length == SLOTS + 1 and want.tokens_evicted == drop
        torch.testing.assert_close(got_v, want.vbuf[:, :, :SLOTS + 1], rtol=0, atol=0)
        assert digest(got_k) == digest(want.kbuf[:, :, :SLOTS + 1]), f"stream {s}: K differs from the oracle"
        got = out[s:s + 1].float().cpu()
        torch.testing.assert_close(got, want_out, rtol=0, atol=2e-2)
        fp32 = oracle.decode_attention(q[s:s + 1].cpu(), want.kbuf[:, :, :SLOTS + 1], want.vbuf[:, :, :SLOTS + 1],
                                       D ** -0.5)
        torch.testing.assert_close(got, fp32, rtol=0, atol=2e-2)

    # --- every stream: the shift and rotation as size-independent properties, on the GPU
    cos_d, sin_d = cos.to(DEV), sin.to(DEV)
    half = D // 2
    sin_signed = torch.cat((-sin_d[:half], sin_d[half:]))
    _, k0, v0, _, _, _ = _state(streams, drop)  # the same seeds: the inputs again
    for s in range(streams):
        src_k = k0[s, :, N_SINK + drop:SLOTS + drop]
        rolled = torch.cat((src_k[..., half:], src_k[..., :half]), -1)
        want_k = torch.addcmul(src_k * cos_d, rolled, sin_signed)
        torch.testing.assert_close(v[s, :, N_SINK:SLOTS], v0[s, :, N_SINK + drop:SLOTS + drop], rtol=0, atol=0)
        torch.testing.assert_close(v[s, :, :N_SINK], v0[s, :, :N_SINK], rtol=0, atol=0)
        torch.testing.assert_close(v[s, :, SLOTS], v1[s, :, 0], rtol=0, atol=0)
        torch.testing.assert_close(k[s, :, :N_SINK], k0[s, :, :N_SINK], rtol=0, atol=0)
        torch.testing.assert_close(k[s, :, SLOTS], k1[s, :, 0].float(), rtol=0, atol=0)
        tol = 2 ** -22 * float(want_k.abs().max())
        torch.testing.assert_close(k[s, :, N_SINK:SLOTS], want_k, rtol=2 ** -22, atol=tol)
        if drop > 1:  # rows past the step's written range keep their contents
            torch.testing.assert_close(k[s, :, SLOTS + 1:], k0[s, :, SLOTS + 1:], rtol=0, atol=0)
            torch.testing.assert_close(v[s, :, SLOTS + 1:], v0[s, :, SLOTS + 1:], rtol=0, atol=0)
    assert torch.isfinite(out.float()).all()
