"""Properties of the split planner (`sink_plan` / `sink_workspace_bytes`, host arithmetic
through the C ABI, no GPU) over random shapes: the splits tile each (batch, head) pair's
rows exactly; a clustered single-launch plan respects the limits its kernel relies on (at
most 16 CTAs, every CTA in one wave, a shift of at most 4 rows, clusters above 8 CTAs only
for splits of at most 4 chunks, never for the tensor-core attention); and the workspace
holds what the split launch of the plan uses, clustered or not (a device that cannot place
the cluster runs the same plan split)."""

import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from attention_sinks_b200 import _lib

SMEM_PER_SM, SMEM_RESERVED = 233472, 1024


@st.composite
def shapes(draw):
    op = draw(st.sampled_from([_lib.OP_FUSED_STEP, _lib.OP_EVICT, _lib.OP_ATTEND]))
    kdt = draw(st.sampled_from([torch.float32, torch.bfloat16]))
    d = draw(st.sampled_from([64, 128, 256]))
    hkv = draw(st.sampled_from([1, 2, 4, 8]))
    group = draw(st.sampled_from([1, 2, 3, 4, 8]))
    batch = draw(st.integers(1, 128))
    n_sink = draw(st.integers(0, 8))
    window = draw(st.integers(1, 40000))
    sms = draw(st.sampled_from([148, 132, 16]))
    if op == _lib.OP_ATTEND:
        rows, drop, n_sink, window = draw(st.integers(1, 40000)), 0, 0, 1
    elif op == _lib.OP_EVICT:
        rows, drop = 0, draw(st.integers(1, 6))
    else:
        rows, drop = n_sink + window + 1, draw(st.integers(0, 6))
    return op, batch, hkv, hkv * group, d, kdt, torch.bfloat16, rows, n_sink, window, drop, sms


@settings(max_examples=400, deadline=None)
@given(shapes())
def test_plan_invariants(built_lib, args):
    op, batch, hkv, hq, d, kdt, vdt, rows, n_sink, window, drop, sms = args
    p = _lib.plan(*args)
    ns, rps, t, ctas = p["splits"], p["rows_per_split"], p["chunk_rows"], p["cluster_ctas"]
    total = window if op == _lib.OP_EVICT else rows
    # the splits tile the rows: no gap, no empty split, items of at most 32 chunks -- longer
    # only for a shift, whose splits stay 3 to 6 shifts long
    assert ns >= 1 and rps % t == 0 and rps <= max(32 * t, 6 * drop + 2 * t)
    if drop > 0 and ns > 1 and op != _lib.OP_ATTEND:
        assert rps >= 3 * drop
    assert (ns - 1) * rps < total <= ns * rps
    pairs = batch * hkv
    tensor_cores = t == 128 and p["stages"] == 3
    assert ctas in (1, ns)
    if ctas > 1:
        slots = sms * (SMEM_PER_SM // (p["smem_bytes"] + SMEM_RESERVED))
        assert not tensor_cores
        assert ns <= 16 and pairs * ns <= slots and drop <= 4
        if ns > 8:
            assert rps // t <= 4
    # the launch mode agrees with the plan: clusters of ns CTAs, or the tensor-core kernel's
    # persistent grid (one CTA per SM at most), or one CTA per split
    if ctas > 1:
        assert p["launch"] == _lib.LAUNCH_CLUSTER and p["ctas"] == pairs * ns
    elif tensor_cores:
        assert p["launch"] == _lib.LAUNCH_TENSOR and p["ctas"] == min(pairs * ns, sms)
    else:
        assert p["launch"] == _lib.LAUNCH_SPLIT and p["ctas"] == pairs * ns
    ws = _lib.workspace_bytes(*args)
    attends = op != _lib.OP_EVICT
    if ns == 1:
        assert ws == 256  # the status word alone: no partials, no halo rows
    else:
        need = 256
        if attends:
            need += pairs * ns * (hq // hkv) * d * 4  # the split partials of O
        assert ws >= need


@pytest.mark.parametrize("sms", [148, 16])
def test_cluster_regime_depends_on_the_sm_count(built_lib, sms):
    """The same small step fits one wave of a 148-SM part as one cluster per pair; on a part
    with few SMs its CTAs no longer fit one wave, and it keeps the split launch."""
    f32, bf16 = torch.float32, torch.bfloat16
    p = _lib.plan(_lib.OP_FUSED_STEP, 8, 8, 16, 128, f32, bf16, 1025, 4, 1020, 1, sms)
    assert (p["cluster_ctas"] > 1) == (sms == 148)
