"""The C ABI library: it loads, exports every entry point include/*.h declares, and its
host-only functions (planning, workspace sizing, argument checks) behave -- no GPU needed."""

import ctypes
import glob
import os
import re

import pytest
import torch

from attention_sinks_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(sink_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(built_lib):
    names = declared_functions()
    assert len(names) >= 9, names
    for name in names:
        assert hasattr(built_lib, name), f"{name} declared in include/ but not exported"
    assert set(_lib.EXPORTED_SYMBOLS) <= set(names)


def test_abi_version_and_errors(built_lib):
    assert built_lib.sink_abi_version() == 1
    for code in (0, -1, -2, -3, -4, -5, -6, -7):
        assert _lib.strerror(code)
    assert "sinkcache_b200" in _lib.strerror(-6)


def test_workspace_and_plan_are_host_arithmetic(built_lib):
    f32, bf16 = torch.float32, torch.bfloat16
    # op bench at 32,768 slots: 8 streams take ~16 waves of 14-chunk items; 1 stream takes
    # one wave (37 splits of each of its 8 heads over 296 CTA slots)
    p = _lib.plan(_lib.OP_FUSED_STEP, 8, 8, 16, 128, f32, bf16, 32769, 4, 32764, 1, 148)
    assert p["chunk_rows"] == 32 and p["stages"] == 4
    assert (p["smem_bytes"] + 1024) * 2 <= 233472  # two CTAs per SM
    assert p["splits"] == 74 and p["rows_per_split"] == 14 * 32
    p = _lib.plan(_lib.OP_FUSED_STEP, 1, 8, 16, 128, f32, bf16, 32769, 4, 32764, 1, 148)
    assert p["splits"] * 8 == 296 and p["rows_per_split"] == 28 * 32
    assert p["launch"] == _lib.LAUNCH_SPLIT and p["ctas"] == 296
    ws = _lib.workspace_bytes(_lib.OP_FUSED_STEP, 8, 8, 16, 128, f32, bf16, 32769, 4, 32764, 1, 148)
    assert ws >= 256
    # unsupported shapes are rejected with 0 bytes / an error code
    assert built_lib.sink_workspace_bytes(_lib.OP_ATTEND, 1, 8, 16, 96, 0, 1, 10, 0, 1, 0, 148) == 0
    assert built_lib.sink_workspace_bytes(_lib.OP_ATTEND, 1, 8, 12, 128, 0, 1, 10, 0, 1, 0, 148) == 0
    assert built_lib.sink_workspace_bytes(_lib.OP_ATTEND, 1, 1, 16, 128, 0, 1, 10, 0, 1, 0, 148) == 0
    # sizes whose pair count would overflow the kernels' int indexing are refused, not planned
    assert built_lib.sink_workspace_bytes(_lib.OP_ATTEND, 1 << 23, 8, 8, 64, 0, 1, 1, 0, 1, 0, 148) == 0
    assert built_lib.sink_workspace_bytes(_lib.OP_ATTEND, 1, 8, 8, 64, 0, 1, 1, 0, 1, 0, 0) == 0
    _lib.plan(_lib.OP_EVICT, 1, 8, 8, 128, f32, torch.float16, 0, 4, 60, 1, 148)  # fp32 K, fp16 V
    with pytest.raises(RuntimeError):
        _lib.plan(_lib.OP_EVICT, 1, 8, 8, 128, torch.float16, bf16, 0, 4, 60, 1, 148)  # mixed 16-bit


@pytest.mark.parametrize("op,rows,n_sink,window,drop", [
    (_lib.OP_EVICT, 0, 4, 60, 1), (_lib.OP_EVICT, 0, 4, 32764, 1), (_lib.OP_EVICT, 0, 2, 7, 200),
    (_lib.OP_ATTEND, 1, 0, 1, 0), (_lib.OP_ATTEND, 4097, 0, 1, 0), (_lib.OP_FUSED_STEP, 1025, 4, 1020, 1),
    (_lib.OP_FUSED_STEP, 257, 4, 252, 0), (_lib.OP_EVICT, 0, 4, 4092, 512), (_lib.OP_EVICT, 0, 4, 32764, 512),
    (_lib.OP_FUSED_STEP, 4097, 4, 4092, 128),
])
@pytest.mark.parametrize("batch", [1, 8, 64])
@pytest.mark.parametrize("kdt", [torch.float32, torch.bfloat16], ids=["k32", "k16"])
def test_plan_covers_rows_exactly(op, rows, n_sink, window, drop, batch, kdt):
    """Splits tile each pair's rows with no gap and no empty split, in items of at most 32
    chunks (8 or more, or one split per pair, when the step takes several waves).  16-bit K attention plans
    for the persistent tensor-core kernel: 128-row chunks, one CTA per SM, items of 2 or
    more chunks."""
    p = _lib.plan(op, batch, 8, 16, 128, kdt, torch.bfloat16, rows, n_sink, window, drop, 148)
    if op == _lib.OP_ATTEND and kdt == torch.bfloat16:
        assert p["chunk_rows"] == 128 and p["stages"] == 3
    total = window if op == _lib.OP_EVICT else rows
    ns, rps, t = p["splits"], p["rows_per_split"], p["chunk_rows"]
    # items of at most 32 chunks, or, for a shift, 3 to 6 shifts long (short splits would
    # send most of the window through the halo copy)
    assert rps % t == 0 and 1 <= ns <= 256 and rps <= max(32 * t, 6 * drop + 2 * t)
    if drop > 0 and ns > 1 and op != _lib.OP_ATTEND:
        assert rps >= 3 * drop
    assert (ns - 1) * rps < total <= ns * rps
    slots = 148 * (233472 // (p["smem_bytes"] + 1024))  # CTA slots: SMs x CTAs per SM
    if batch * 8 * ns > slots:  # several waves: no more splits than items of 8 (tensor cores: 2) chunks give
        assert ns <= -(-(-(-total // t)) // (2 if t == 128 else 8))


@pytest.mark.parametrize("batch,slots,ns,mode", [
    (1, 256, 9, "cluster"), (1, 1024, 11, "cluster"), (2, 2047, 16, "cluster"), (7, 4096, 5, "cluster"),
    (8, 1024, 4, "cluster"), (2, 4096, 17, "split"), (4, 4096, 9, "split"), (2, 8192, 18, "split"),
    (4, 8192, 9, "split"), (1, 4096, 33, "split"), (64, 256, 1, "split"), (1, 32768, 37, "split"),
    (8, 4096, 9, "split"), (64, 32768, 33, "split"), (1, 16384, 37, "split"),
])
def test_plan_clusters_small_steps(batch, slots, ns, mode, built_lib):
    """Fused steps whose CTAs fit one wave with at most 16 splits per pair (or 16 splits
    that add at most 4 chunks per split) run as one clustered launch.  Clusters of more than
    8 CTAs only for splits of at most 4 chunks.  Several waves, or longer splits, keep the
    split launch with its halo pre-pass and combine.  Every split plan, clustered or not,
    has the split launch's partials and halo rows in its workspace."""
    f32, bf16 = torch.float32, torch.bfloat16
    args = (_lib.OP_FUSED_STEP, batch, 8, 16, 128, f32, bf16, slots + 1, 4, slots - 4, 1, 148)
    p = _lib.plan(*args)
    clustered = mode == "cluster"
    want = {"split": _lib.LAUNCH_SPLIT, "cluster": _lib.LAUNCH_CLUSTER}[mode]
    assert p["splits"] == ns and p["cluster_ctas"] == (ns if clustered else 1) and p["launch"] == want
    ws = _lib.workspace_bytes(*args)
    assert (ws == 256) == (ns == 1)  # the status word alone
    if clustered:  # the same plan split: partials of O, m, l and one halo row per split
        parts = batch * 8 * ns * 2
        halo = batch * 8 * ns * 128 * (4 + 2)
        assert ws >= 256 + parts * 128 * 4 + 2 * parts * 4 + halo
    # a shift of more than 4 rows, or 16-bit K attention on the tensor cores, is never clustered
    assert _lib.plan(_lib.OP_EVICT, batch, 8, 8, 128, f32, bf16, 0, 4, slots - 4, 5, 148)["cluster_ctas"] == 1
    assert _lib.plan(_lib.OP_ATTEND, batch, 8, 16, 128, bf16, bf16, slots, 0, 1, 0, 148)["cluster_ctas"] == 1


def test_argument_errors_return_codes_without_a_gpu(built_lib):
    """Rejected arguments come back as codes; nothing is launched."""
    kv = _lib.KVBuffers()  # null pointers
    rows = _lib.Rows()
    assert built_lib.sink_append(ctypes.byref(kv), ctypes.byref(rows), ctypes.byref(rows), 0, None) == -1
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 60, 1, None, None, 1, None, 0, None) == -1
    kv = _lib.KVBuffers(16, 32, 0, 1, 1, 8, 65, 96, 65 * 96 * 8, 65 * 96, 65 * 96 * 8, 65 * 96)
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 60, 1, None, None, 0, None, 0, None) == -3
    kv = _lib.KVBuffers(16, 32, 2, 1, 1, 8, 65, 128, 65 * 128 * 8, 65 * 128, 65 * 128 * 8, 65 * 128)
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 60, 1, None, None, 0, None, 0, None) == -2
    kv = _lib.KVBuffers(8, 32, 0, 1, 1, 8, 65, 128, 65 * 128 * 8, 65 * 128, 65 * 128 * 8, 65 * 128)
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 60, 1, None, None, 0, None, 0, None) == -5
    kv = _lib.KVBuffers(16, 32, 0, 1, 1, 8, 65, 128, 65 * 128 * 8, 65 * 128, 65 * 128 * 8, 65 * 128)
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 61, 1, None, None, 0, None, 0, None) == -1
    assert built_lib.sink_evict_rerotate(ctypes.byref(kv), 4, 60, 0, None, None, 0, None, 0, None) == 0


def test_product_refuses_cpu_tensors():
    """No CPU path: the kernels' wrappers reject host tensors instead of computing."""
    k = torch.zeros(1, 8, 65, 128)
    with pytest.raises(RuntimeError, match="CUDA"):
        _lib.kv_desc(k, k.bfloat16())
    from attention_sinks_b200 import SinkLayer
    layer = SinkLayer(4, 60, torch.ones(64))
    with pytest.raises(RuntimeError, match="CUDA"):
        layer.update(torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16), torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16))
