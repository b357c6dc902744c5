#!/usr/bin/env python
"""Benchmark of the sink-cache decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...          (one process per GPU)

A step is one layer of one decode step for every stream of this rank: the pending eviction
of one row with RoPE re-rotation by -1 of every window key (fp32), the append of the new
token (fp32 K / bf16 V), and GQA decode attention over the n_sink + window + 1 rows -- the
fused kernel pass of sink_fused_decode_step.  Shapes are one Qwen3-0.6B attention layer
(16 query heads, 8 KV heads, head_dim 128), n_sink 4, a 32,768-slot cache, 64 streams per
GPU; the state (12.9 GB per GPU) is far larger than L2, so consecutive steps read HBM.

`value` is the algorithmic bytes of all ranks' steps per second (GB/s) with inputs resident
in HBM; `e2e` is the same through the public API (SinkLayer.update + the attention backend)
with each step's q/k/v copied from pinned host memory and its output copied back.
Streams are independent: ranks split them with no collective on the hot path (weak
scaling: 64 streams per GPU).  `--impl reference` times the reference's CPU path (the
oracle port of it) on this host's cores instead.

The line's `model` object carries the model-level half of the metric at the same world
size (skip it with --no-model): a random-init Qwen3-0.6B with SinkCache(4, 1020) streamed
token by token from position 0 through the CUDA-graph StreamRunner, one stream per GPU
(tok/s, and the mean NLL against the reference's own CPU run of stream 0), and the same
model with 32,768 slots and 32 streams split over the GPUs (strong scaling: tok/s and
mean NLL of the same global streams at every world size).  Per-rank NLL sums and times
are gathered with NCCL after the timed regions.
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "decode-step µs/layer & achieved HBM GB/s (attn+evict/rerotate); streamed tok/s at 1/2/4/8 B200"
HQ, HKV, D, N_SINK = 16, 8, 128, 4
THETA = 1e6
L2_BYTES = 126 * 2 ** 20
FALLBACK_HBM_GBS = 6650.0


def alg_bytes(slots: int, n_sink: int = N_SINK, hq: int = HQ, hkv: int = HKV, d: int = D) -> int:
    """Algorithmic HBM bytes of one layer-step of one stream: every window row read and
    written once (K fp32 4+4 B, V bf16 2+2 B per element), sink rows read (6 B), the new
    token read (bf16 k, v) and stored (fp32 k, bf16 v), q read and the output written."""
    w, e = slots - n_sink, hkv * d
    return 12 * w * e + 6 * n_sink * e + 10 * e + 4 * hq * d


def alg_bytes_v2(slots: int, n_sink: int = N_SINK, hq: int = HQ, hkv: int = HKV, d: int = D) -> int:
    """Algorithmic HBM bytes of one ring-buffer (v2) layer-step of one stream, K and V in bf16:
    every window row read once (2 + 2 B per element), the new token read and stored in its
    ring slot (8 B), the region's original keys and values read and its rotated keys stored
    (6 B per region row element), q read and the output written.  The window is the same
    slots - n_sink rows the v1 step moves."""
    w, e = slots - n_sink, hkv * d
    return 4 * w * e + 8 * e + 6 * n_sink * e + 4 * hq * d


def inv_freq(d: int = D, theta: float = THETA) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32) / d))


def hbm_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(name: str = "sink_stream_kernel_traffic.txt") -> dict:
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary, if any
    (lines `traffic_bytes_per_launch: N` and `traffic_workload: ...`)."""
    path = os.path.join(ROOT, "profiles", name)
    out = {}
    try:
        with open(path) as f:
            for line in f:
                if ":" in line:
                    k, v = line.split(":", 1)
                    out[k.strip()] = v.strip()
    except OSError:
        pass
    return out


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.target = None
        try:
            props = torch.cuda.get_device_properties(device)
            uuid = str(getattr(props, "uuid", "") or "")
            self.target = uuid if uuid.startswith("GPU-") else (f"GPU-{uuid}" if uuid else None)
        except Exception:
            self.target = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.target:
            cmd += ["-i", self.target]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, maxes, reasons = [], [], set()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(self.REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


# ----------------------------------------------------------------------------- workload


class OpBench:
    """One layer of decode state for `batch` streams on one GPU, in the steady state (S + 1
    rows: S kept, one pending eviction), plus a small pool of per-step inputs."""

    POOL = 4

    def __init__(self, batch: int, slots: int, device: torch.device, seed: int):
        from attention_sinks_b200 import _lib
        self.lib = _lib
        self.batch, self.slots, self.device = batch, slots, device
        self.window = slots - N_SINK
        self.scale = D ** -0.5
        g = torch.Generator(device=device).manual_seed(seed)
        self.k = torch.empty(batch, HKV, slots + 1, D, dtype=torch.float32, device=device)
        self.v = torch.empty(batch, HKV, slots + 1, D, dtype=torch.bfloat16, device=device)
        inv = inv_freq().to(device)
        freqs = torch.arange(slots + 1, device=device, dtype=torch.float32)[:, None] * inv
        emb = torch.cat((freqs, freqs), -1)
        cos_t, sin_t = emb.cos(), emb.sin()
        for b in range(batch):  # keys ~ N(0,1) rotated at positions 0..S, one stream at a time
            raw = torch.randn(HKV, slots + 1, D, device=device, generator=g)
            x1, x2 = raw.chunk(2, -1)
            self.k[b] = raw * cos_t + torch.cat((-x2, x1), -1) * sin_t
            self.v[b] = torch.randn(HKV, slots + 1, D, device=device, generator=g).to(torch.bfloat16)
        del freqs, emb, cos_t, sin_t
        bf = torch.bfloat16
        self.q = [torch.randn(batch, HQ, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        self.kn = [torch.randn(batch, HKV, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        self.vn = [torch.randn(batch, HKV, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        cos, sin = torch.cat((-inv.cpu(), -inv.cpu())).cos(), torch.cat((-inv.cpu(), -inv.cpu())).sin()
        self.cos, self.sin = cos.to(device), sin.to(device)
        self.out = torch.empty(batch, 1, HQ, D, dtype=bf, device=device)
        self.ws = _lib.Workspace()
        sms = _lib.sm_count(device)
        need = _lib.workspace_bytes(_lib.OP_FUSED_STEP, batch, HKV, HQ, D, torch.float32, bf, slots + 1,
                                    N_SINK, self.window, 1, sms)
        self.ws.get(need, device)
        self.plan = _lib.plan(_lib.OP_FUSED_STEP, batch, HKV, HQ, D, torch.float32, bf, slots + 1,
                              N_SINK, self.window, 1, sms)

    def step(self, i: int) -> None:
        j = i % self.POOL
        self.lib.fused_decode_step(self.k, self.v, self.kn[j], self.vn[j], self.q[j], N_SINK, self.window, 1,
                                   self.slots, self.cos, self.sin, self.scale, self.out, self.ws)

    def state_bytes(self) -> int:
        return self.k.numel() * 4 + self.v.numel() * 2


class OpBenchV2:
    """One ring-buffer (v2) layer of decode state for `batch` streams on one GPU in the steady
    state: a ring of window + 1 slots holding keys rotated at their absolute positions, the
    n_sink region rows (original keys at positions 0..n_sink-1), the device position far
    from the origin, plus a small pool of per-step inputs.  A step is sink_v2_decode_step:
    the place work (ring write, region rotation, position advance) and split-K attention
    over the window + 1 + n_sink rows in one tensor-core launch, then the split combine
    unless the splits merge inside their clusters."""

    POOL = 4

    def __init__(self, batch: int, slots: int, device: torch.device, seed: int):
        from attention_sinks_b200 import _lib
        self.lib = _lib
        self.batch, self.slots, self.device = batch, slots, device
        self.window = slots - N_SINK
        self.ring = self.window + 1
        self.rows = self.ring + N_SINK
        self.scale = D ** -0.5
        bf = torch.bfloat16
        g = torch.Generator(device=device).manual_seed(seed)
        self.k = torch.empty(batch, HKV, self.rows, D, dtype=bf, device=device)
        self.v = torch.empty(batch, HKV, self.rows, D, dtype=bf, device=device)
        for b in range(batch):  # key and value contents do not change the work: N(0, 1)
            self.k[b] = torch.randn(HKV, self.rows, D, device=device, generator=g).to(bf)
            self.v[b] = torch.randn(HKV, self.rows, D, device=device, generator=g).to(bf)
        self.reg_k = torch.randn(batch, HKV, N_SINK, D, device=device, generator=g).to(bf)
        self.reg_pos = torch.arange(N_SINK, device=device)
        self.position = torch.tensor([10_000_000, 0], device=device)
        self.inv = inv_freq().to(device, torch.float64)
        self.q = [torch.randn(batch, HQ, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        self.kn = [torch.randn(batch, HKV, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        self.vn = [torch.randn(batch, HKV, 1, D, device=device, generator=g).to(bf) for _ in range(self.POOL)]
        self.out = torch.empty(batch, 1, HQ, D, dtype=bf, device=device)
        self.ws = _lib.Workspace()
        sms = _lib.sm_count(device)
        self.ws.get(_lib.workspace_bytes(_lib.OP_ATTEND, batch, HKV, HQ, D, bf, bf, self.rows, 0, 1, 0, sms), device)
        self.plan = _lib.plan(_lib.OP_ATTEND, batch, HKV, HQ, D, bf, bf, self.rows, 0, 1, 0, sms)

    def step(self, i: int) -> None:
        j = i % self.POOL
        self.lib.v2_decode_step(self.k, self.v, self.kn[j], self.vn[j], self.reg_k, self.reg_pos, N_SINK,
                                self.position, N_SINK, self.window, self.inv, self.q[j], self.scale, self.out,
                                self.ws)

    def state_bytes(self) -> int:
        return (self.k.numel() + self.v.numel()) * 2


def flush_l2(buf: torch.Tensor, i: int) -> None:
    """Evict the state from L2 between timed steps: write one half of `buf` (2x L2), then
    read the other half, so L2 is left holding clean lines and the timed step does not
    pay for writing back the flush's dirty lines."""
    half = buf.numel() // 2
    buf[:half].fill_(i & 0xFF)
    buf[half:].sum(dtype=torch.int64)


def time_device(bench: OpBench, steps: int, warmup: int, flush: torch.Tensor | None = None) -> float:
    """Mean ms per step with CUDA events on the launching stream.  When `flush` is given
    (state smaller than L2), L2 is overwritten between steps and each step timed alone."""
    for i in range(warmup):
        bench.step(i)
    torch.cuda.synchronize()
    if flush is None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            bench.step(i)
        end.record()
        end.synchronize()
        return start.elapsed_time(end) / steps
    total = 0.0
    for i in range(steps):
        flush_l2(flush, i)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        bench.step(i)
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return total / steps


class _Module:
    """What the attention backend reads from a Transformers attention module."""
    training = False
    num_key_value_groups = HQ // HKV
    is_causal = True


def run_e2e(bench: OpBench, steps: int, warmup: int) -> tuple[float, int, int]:
    """ms/step through the public API with host buffers: per step the new q/k/v are copied
    from pinned host memory, SinkLayer.update + the registered attention backend run the
    fused step, and the output is copied to pinned host memory."""
    from attention_sinks_b200 import SinkLayer
    from attention_sinks_b200.decode_attention import decode_attention_forward
    dev = bench.device
    layer = SinkLayer(N_SINK, bench.window, inv_freq(), key_dtype=torch.float32, fused=True)
    chunk = 4096
    for r0 in range(0, bench.slots + 1, chunk):  # prefill S + 1 rows through update()
        r1 = min(r0 + chunk, bench.slots + 1)
        layer.update(bench.k[:, :, r0:r1].to(torch.bfloat16), bench.v[:, :, r0:r1])
    assert layer.length == bench.slots + 1 and layer._kbuf.shape[-2] == bench.slots + 1
    pool = OpBench.POOL
    hq = [bench.q[j].cpu().pin_memory() for j in range(pool)]
    hk = [bench.kn[j].cpu().pin_memory() for j in range(pool)]
    hv = [bench.vn[j].cpu().pin_memory() for j in range(pool)]
    hout = [torch.empty(bench.out.shape, dtype=bench.out.dtype).pin_memory() for _ in range(pool)]
    module = _Module()

    def step(i):
        j = i % pool
        q = hq[j].to(dev, non_blocking=True)
        k = hk[j].to(dev, non_blocking=True)
        v = hv[j].to(dev, non_blocking=True)
        keys, values = layer.update(k, v)
        o, _ = decode_attention_forward(module, q, keys, values, None, scaling=bench.scale)
        hout[j].copy_(o, non_blocking=True)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step(i)
    end.record()
    end.synchronize()
    h2d = (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 2
    d2h = hout[0].numel() * 2
    del layer
    return start.elapsed_time(end) / steps, h2d, d2h


def cpu_streams(streams: int, state_bytes_per_stream: int) -> int:
    """Streams the CPU baseline holds at once: the workload's, unless five copies of that
    state (the buffers and the step's temporaries) would not fit this host's memory."""
    try:
        ram = os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError):
        return 1
    n = streams
    while n > 1 and 5 * n * state_bytes_per_stream > ram:
        n //= 2
    return n


def _time_cpu_steps(step, seconds: float) -> tuple[float, int]:
    """ms per step of `step()` after one warm-up call: as many calls as fit in `seconds` (at
    least one)."""
    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el > seconds or n >= 1000:
            return el * 1e3 / n, n


def cpu_baseline(slots: int, seconds: float = 15.0, streams: int = 1) -> dict:
    """The reference's CPU path (oracle port: SinkLayer.update on the PyTorch branch + SDPA
    attention) on this host's cores over the workload's streams as one batch, as many steps
    as fit in about `seconds`.  One stream's state is built and repeated over the batch (a
    step's work does not depend on the values)."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_streams = cpu_streams(streams, (slots + 1) * HKV * D * (4 + 2))
    layer = oracle.make_prefilled_cache(1, HKV, D, slots, N_SINK, inv_freq(), seed=0)
    layer.kbuf, layer.vbuf = layer.kbuf.repeat(n_streams, 1, 1, 1), layer.vbuf.repeat(n_streams, 1, 1, 1)
    g = torch.Generator().manual_seed(1)
    q = torch.randn(n_streams, HQ, 1, D, generator=g).bfloat16()
    kn = torch.randn(n_streams, HKV, 1, D, generator=g).bfloat16()
    vn = torch.randn(n_streams, HKV, 1, D, generator=g).bfloat16()
    ms, n = _time_cpu_steps(lambda: oracle.reference_cpu_step(layer, q, kn, vn, D ** -0.5), seconds)
    del layer
    rate = alg_bytes(slots) * n_streams / (ms * 1e-3) / 1e9
    scaled = "" if n_streams == streams else f"; host memory held {n_streams} of the {streams} streams, rate taken for all"
    return {"value": round(rate, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "ms_per_step": round(ms * streams / n_streams, 3),
            "sample": f"{n_streams} streams x {slots} slots as one batch, {n} steps after a warm-up, oracle port "
                      f"of SinkLayer.update (PyTorch path) + SDPA, torch threads={threads}{scaled}"}


def run_e2e_v2(bench: OpBenchV2, steps: int, warmup: int) -> tuple[float, int, int]:
    """ms/step of the ring-buffer step through the public API with host buffers: per step the
    new q/k/v are copied from pinned host memory, SinkLayerV2.update + the registered
    attention backend run the fused step, and the output is copied to pinned host memory."""
    from attention_sinks_b200 import SinkLayerV2
    from attention_sinks_b200.decode_attention import decode_attention_forward
    dev = bench.device
    layer = SinkLayerV2(N_SINK, bench.window, inv_freq(), fused=True)
    layer.update(bench.k[:, :, :bench.slots], bench.v[:, :, :bench.slots])  # one chunk fills the cache
    assert layer.t == bench.slots and layer.in_cache_length() == bench.slots
    torch.cuda.empty_cache()
    pool = OpBenchV2.POOL
    hq = [bench.q[j].cpu().pin_memory() for j in range(pool)]
    hk = [bench.kn[j].cpu().pin_memory() for j in range(pool)]
    hv = [bench.vn[j].cpu().pin_memory() for j in range(pool)]
    hout = [torch.empty(bench.out.shape, dtype=bench.out.dtype).pin_memory() for _ in range(pool)]
    module = _Module()

    def step(i):
        j = i % pool
        q = hq[j].to(dev, non_blocking=True)
        k = hk[j].to(dev, non_blocking=True)
        v = hv[j].to(dev, non_blocking=True)
        keys, values = layer.update(k, v)
        o, _ = decode_attention_forward(module, q, keys, values, None, scaling=bench.scale)
        hout[j].copy_(o, non_blocking=True)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step(i)
    end.record()
    end.synchronize()
    h2d = (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 2
    d2h = hout[0].numel() * 2
    del layer
    return start.elapsed_time(end) / steps, h2d, d2h


def cpu_baseline_v2(slots: int, seconds: float = 15.0, streams: int = 1) -> dict:
    """The reference's CPU path for the ring-buffer layer (oracle port: SinkLayerV2.update +
    SDPA attention) on this host's cores over the workload's streams as one batch (one
    stream's state repeated)."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_streams = cpu_streams(streams, (slots + N_SINK) * HKV * D * 4)
    layer = oracle.make_prefilled_cache_v2(1, HKV, D, slots, N_SINK, inv_freq(), seed=0)
    for name in ("kbuf", "vbuf", "reg_k"):
        setattr(layer, name, getattr(layer, name).repeat(n_streams, 1, 1, 1))
    g = torch.Generator().manual_seed(1)
    q = torch.randn(n_streams, HQ, 1, D, generator=g).bfloat16()
    kn = torch.randn(n_streams, HKV, 1, D, generator=g).bfloat16()
    vn = torch.randn(n_streams, HKV, 1, D, generator=g).bfloat16()
    ms, n = _time_cpu_steps(lambda: oracle.reference_cpu_step_v2(layer, q, kn, vn, D ** -0.5), seconds)
    del layer
    rate = alg_bytes_v2(slots) * n_streams / (ms * 1e-3) / 1e9
    scaled = "" if n_streams == streams else f"; host memory held {n_streams} of the {streams} streams, rate taken for all"
    return {"value": round(rate, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "ms_per_step": round(ms * streams / n_streams, 3),
            "sample": f"{n_streams} streams x {slots} slots as one batch, {n} steps after a warm-up, oracle port "
                      f"of SinkLayerV2.update (ring step) + SDPA, torch threads={threads}{scaled}"}


def time_graph(bench: OpBench, steps: int, flush: torch.Tensor | None) -> float:
    """Mean ms per step of one captured step replayed from a CUDA graph (how StreamRunner
    runs it: no host launch cost inside the step).  With `flush`, L2 is overwritten between
    replays and each replay is timed alone."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(3):
            bench.step(0)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        bench.step(0)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    if flush is None:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            graph.replay()
        end.record()
        end.synchronize()
        return start.elapsed_time(end) / steps
    total = 0.0
    for i in range(steps):
        flush_l2(flush, i)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return total / steps


def graph_floor(device: torch.device, flush: torch.Tensor, steps: int = 50) -> float:
    """µs of one CUDA-graph replay of a one-element kernel, timed like the sweep (CUDA events
    around the replay, L2 overwritten before each): the fixed cost inside every sweep number."""
    x = torch.zeros(1, device=device)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        x.add_(1)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        x.add_(1)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    total = 0.0
    for i in range(steps):
        flush_l2(flush, i)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    return round(total / steps * 1e3, 2)


def time_graph_layers(benches: list, reps: int = 30) -> float:
    """Mean ms per layer-step of one CUDA graph holding one step of every bench in turn (each
    its own state, like the layers of a model's decode step).  Their states together exceed
    2x L2, so every step reads its state from HBM with no flush in between."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for b in benches:
            b.step(0)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for b in benches:
            b.step(0)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / (reps * len(benches))


def sweep(device: torch.device, flush: torch.Tensor, cls=None, alg=None) -> dict:
    """µs per layer-step and GB/s over the op-bench grid (slots x streams), 1 GPU, from
    CUDA-graph replays.  `us_per_layer`: one step replayed alone, L2 overwritten before each
    replay when the state is smaller than 2x L2 (so it carries a graph launch per step).
    `us_per_layer_in_sequence`: for such states, the steps of as many independent layer
    states as exceed 2.5x L2 together, captured in one graph and replayed back to back, the
    way a model's layers run in one decode step; per layer-step."""
    cls, alg = cls or OpBench, alg or alg_bytes
    out = {}
    for slots in (256, 1024, 4096, 32768):
        for batch in (1, 8, 64):
            b = cls(batch, slots, device, seed=slots + batch)
            small = b.state_bytes() < 2 * L2_BYTES
            steps = 50 if small else max(10, min(200, int(2e9 / (alg(slots) * batch))))
            ms = time_graph(b, steps, flush if small else None)
            row = {"us_per_layer": round(ms * 1e3, 2), "GB_s": round(alg(slots) * batch / (ms * 1e-3) / 1e9, 1),
                   "l2_flushed": small}
            if small:
                n = min(320, max(2, math.ceil(2.5 * L2_BYTES / b.state_bytes())))
                layers = [b] + [cls(batch, slots, device, seed=slots + batch + 97 * i) for i in range(1, n)]
                ms_seq = time_graph_layers(layers)
                row["us_per_layer_in_sequence"] = round(ms_seq * 1e3, 2)
                row["GB_s_in_sequence"] = round(alg(slots) * batch / (ms_seq * 1e-3) / 1e9, 1)
                row["layers_in_sequence"] = n
                del layers
            out[f"S{slots}_B{batch}"] = row
            del b
            torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- chunk steps


def chunk_bench(args) -> None:
    """The general (multi-token) step on a full cache, one layer of the op-bench shape: a
    chunk of `n` tokens per stream through the public API -- SinkLayer.update (pending
    eviction of the previous chunk with re-rotation by -n, append, buffer growth and shrink)
    or SinkLayerV2.update (region rotation, window gather, ring stores) -- then the chunk's
    attention through the registered backend (SDPA over the returned K/V, as the
    reference).  Device-resident inputs, CUDA events around `steps` chunk steps."""
    from attention_sinks_b200 import SinkLayer, SinkLayerV2, streams
    from attention_sinks_b200.decode_attention import decode_attention_forward
    rank, world, local = streams.init_from_env("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    bf = torch.bfloat16
    for cache in ("v1", "v2"):
        for slots in (4096, 32768):
            for n in (16, 128, 512):
                b = 8
                if cache == "v1":
                    layer = SinkLayer(N_SINK, slots - N_SINK, inv_freq(), key_dtype=torch.float32, fused=True)
                else:
                    layer = SinkLayerV2(N_SINK, slots - N_SINK, inv_freq(), fused=True)
                for r0 in range(0, slots, 4096):  # fill the cache
                    r1 = min(r0 + 4096, slots)
                    layer.update(torch.randn(b, HKV, r1 - r0, D, device=dev, generator=g).to(bf),
                                 torch.randn(b, HKV, r1 - r0, D, device=dev, generator=g).to(bf))
                pool = [(torch.randn(b, HQ, n, D, device=dev, generator=g).to(bf),
                         torch.randn(b, HKV, n, D, device=dev, generator=g).to(bf),
                         torch.randn(b, HKV, n, D, device=dev, generator=g).to(bf)) for _ in range(2)]
                module = _Module()

                def step(i):
                    q, k, v = pool[i % 2]
                    keys, values = layer.update(k, v)
                    o, _ = decode_attention_forward(module, q, keys, values, None, scaling=D ** -0.5)
                    return o

                for i in range(3):
                    step(i)
                torch.cuda.synchronize()
                steps = 20
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                for i in range(steps):
                    step(i)
                end.record()
                end.synchronize()
                ms = start.elapsed_time(end) / steps
                out[f"{cache}_S{slots}_n{n}"] = {"us_per_chunk_step": round(ms * 1e3, 1),
                                                "tokens_per_s_per_layer": round(b * n / (ms * 1e-3), 0)}
                del layer, pool
                torch.cuda.empty_cache()
    if rank == 0:
        line = {"metric": "chunk step µs/layer (general path)", "value": None, "unit": "us", "n_gpus": world,
                "steps": 20, "warmup": 3, "higher_is_better": False, "dtype": "bf16 model / fp32 K (v1), bf16 K (v2)",
                "data": "synthetic", "config": {"workload": "chunk steps on a full cache, 8 streams, Qwen3-0.6B "
                                                             "layer shape", "n_sink": N_SINK},
                "chunks": out}
        print(json.dumps(line), flush=True)
    streams.shutdown()


# ----------------------------------------------------------------------------- model workloads


def model_configs():
    """The model-level configurations: random-init architectures (no weights available)."""
    from transformers import LlamaConfig, Qwen3Config
    qwen3_06b = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                     num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                     max_position_embeddings=40960, tie_word_embeddings=True, rms_norm_eps=1e-6)
    return {
        # Qwen3-0.6B, sink 4 + window 1020, one stream per GPU
        "qwen3-0.6b-1k": dict(cfg=lambda: Qwen3Config(**qwen3_06b), n_sink=4, window=1020, streams=1,
                              partition=False),
        # Llama-3.2-1B (llama3 rope scaling), 1K slots, 8 streams per GPU
        "llama3.2-1b-1k": dict(cfg=lambda: LlamaConfig(
            vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
            num_attention_heads=32, num_key_value_heads=8, head_dim=64, rope_theta=5e5,
            rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                          "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
            max_position_embeddings=131072, tie_word_embeddings=True, rms_norm_eps=1e-5),
            n_sink=4, window=1020, streams=8, partition=False),
        # Qwen3-0.6B with 32,768 slots, 32 streams split over the GPUs (16 per wave)
        "qwen3-0.6b-32k": dict(cfg=lambda: Qwen3Config(**qwen3_06b), n_sink=4, window=32764, streams=32,
                               partition=True, wave=16),
        # Qwen3-8B, 4,096 slots, 16 streams per GPU
        "qwen3-8b-4k": dict(cfg=lambda: Qwen3Config(
            vocab_size=151936, hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
            num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
            max_position_embeddings=40960, tie_word_embeddings=False, rms_norm_eps=1e-6),
            n_sink=4, window=4092, streams=16, partition=False),
    }


def build_model(spec: dict, device: torch.device, seed: int = 0):
    """Random-init bf16 model on `device` with the registered sink attention backend; the
    same seed gives the same weights on every rank."""
    from transformers import AutoModelForCausalLM

    from attention_sinks_b200 import register
    torch.manual_seed(seed)
    with torch.device(device):
        return AutoModelForCausalLM.from_config(spec["cfg"](), attn_implementation=register(),
                                                dtype=torch.bfloat16).eval()


class ModelBench:
    """One model replica and a sink cache for the streams `ids` (global stream indices) on one
    GPU, filled to the steady state (v1: n_sink + window kept rows + one pending; v2:
    n_sink + window tokens seen) through the layers' update with synthetic K/V, then
    streamed one token per step under the CUDA-graph StreamRunner.  Every stream's fill and
    tokens come from generators seeded by its global index, so a stream's data does not
    depend on how streams are split over GPUs or waves."""

    IDS = 64

    def __init__(self, spec: dict, model, stream_ids: list[int], device: torch.device, cache: str = "v1"):
        from attention_sinks_b200 import SinkCache, SinkCacheV2, StreamRunner
        self.model, self.cfg, self.batch, self.device = model, model.config, len(stream_ids), device
        cls = SinkCacheV2 if cache == "v2" else SinkCache
        self.cache = cls.from_model(self.model, n_sink=spec["n_sink"], window=spec["window"])
        hkv, d = self.cfg.num_key_value_heads, self.cfg.head_dim
        rows = spec["n_sink"] + spec["window"] + (0 if cache == "v2" else 1)
        gens = [torch.Generator(device=device).manual_seed(10_000 + s) for s in stream_ids]
        for layer in self.cache.layers:
            for r0 in range(0, rows, 4096):
                n = min(4096, rows - r0)
                k = torch.cat([torch.randn(1, hkv, n, d, device=device, generator=g) for g in gens]).bfloat16()
                v = torch.cat([torch.randn(1, hkv, n, d, device=device, generator=g) for g in gens]).bfloat16()
                layer.update(k, v)
        self.runner = StreamRunner(self.model, self.cache)
        self.ids = torch.cat([torch.randint(0, self.cfg.vocab_size, (1, self.IDS), device=device,
                                            generator=torch.Generator(device=device).manual_seed(20_000 + s))
                              for s in stream_ids])
        self.nll = torch.zeros(self.batch, device=device, dtype=torch.float64)

    def step(self, i: int) -> None:
        import torch.nn.functional as F
        j = i % (self.IDS - 1)
        logits = self.runner.step(self.ids[:, j:j + 1])[:, -1]
        self.nll += F.cross_entropy(logits.float(), self.ids[:, j + 1], reduction="none").double()

    def cache_bytes(self) -> int:
        return sum(l._kbuf.numel() * l._kbuf.element_size() + l._vbuf.numel() * l._vbuf.element_size()
                   for l in self.cache.layers)

    def step_kernels(self) -> int:
        """Sink-cache kernels per decode step: those the library launched while the replayed
        step was captured."""
        return self.runner.cache_kernels_per_replay


def stream_run(spec: dict, stream_ids: list[int], device: torch.device, steps: int, warmup: int,
               cache: str = "v1", wave: int | None = None) -> dict:
    """Steady-state streaming of this rank's streams in waves: per wave, `warmup` steps (the
    first eviction, the graph capture, replays), then `steps` timed graph-replayed steps.
    Returns this rank's seconds, tokens and NLL sum over the timed steps."""
    from attention_sinks_b200 import streams
    model = build_model(spec, device)
    wave = wave or max(len(stream_ids), 1)
    seconds, tokens, nll, launches, cache_gb = 0.0, 0, 0.0, 0, 0.0
    for w0 in range(0, len(stream_ids), wave):
        bench = ModelBench(spec, model, stream_ids[w0:w0 + wave], device, cache)
        for i in range(warmup):
            bench.step(i)
        assert bench.cache.is_steady and bench.runner.graph is not None
        bench.nll.zero_()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(steps):
            bench.step(warmup + i)
        end.record()
        end.synchronize()
        bench.cache.check_status()
        seconds += start.elapsed_time(end) / 1e3
        tokens += bench.batch * steps
        nll += float(bench.nll.sum())
        launches += bench.step_kernels() * steps
        cache_gb = bench.cache_bytes() / 1e9
        del bench
        torch.cuda.empty_cache()
    del model
    torch.cuda.empty_cache()
    streams.barrier()
    return {"seconds": seconds, "tokens": tokens, "nll_sum": nll, "launches": launches, "cache_gb": cache_gb}


def gather(local: dict) -> dict:
    """Job totals over ranks (NCCL, off the hot path): max of the seconds, sums of the rest."""
    from attention_sinks_b200 import streams
    t = streams.reduce_max(local["seconds"])
    tok, nll, launches = streams.reduce_sum([local["tokens"], local["nll_sum"], local["launches"]])
    return {"seconds": t, "tokens": int(tok), "nll_sum": nll, "launches": int(launches)}


def reference_stream_nll() -> dict:
    """The reference's own CPU run of the streamed Qwen3-0.6B / SinkCache(4, 1020) workload
    (committed fixture of tests/golden: mean NLL over 4,096 one-token steps)."""
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)["config1"]


def stream_qwen3_1k(device: torch.device, rank: int, world: int, steps: int = 4096) -> dict:
    """Qwen3-0.6B (random init, the weights of the reference fixture), SinkCache(4, 1020),
    one stream per GPU streamed token by token from position 0 through StreamRunner, the NLL
    of every next token buffered on the device (the shape of experiments/ppl.py:52-84).
    Stream r is the uniform token sequence of seed 1 + r; stream 0 is the reference run's."""
    import torch.nn.functional as F

    from attention_sinks_b200 import SinkCache, StreamRunner, register, streams
    from tests.golden import cases
    model, _ = cases.qwen3_0_6b(0, attn=register())
    model = model.to(device)
    ids = torch.randint(0, 151936, (1, steps + 1), generator=torch.Generator().manual_seed(1 + rank)).to(device)
    cache = SinkCache.from_model(model, n_sink=4, window=1020)
    runner = StreamRunner(model, cache)
    nll = torch.empty(steps, device=device)
    steady_from = 1200  # steps before this one fill the cache, evict eagerly, capture
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    torch.cuda.synchronize()
    streams.barrier()
    ev[0].record()
    with torch.inference_mode():
        for t in range(steps):
            if t == steady_from:
                ev[1].record()
            logits = runner.step(ids[:, t:t + 1])[0, -1]
            nll[t] = F.cross_entropy(logits.float()[None], ids[0, t + 1:t + 2])
    ev[2].record()
    ev[2].synchronize()
    cache.check_status()
    whole, steady = ev[0].elapsed_time(ev[2]) / 1e3, ev[1].elapsed_time(ev[2]) / 1e3
    own_mean = float(nll.double().mean())
    t_whole, t_steady = streams.reduce_max(whole), streams.reduce_max(steady)
    nll_sum = streams.reduce_sum([float(nll.double().sum())])[0]
    ref = reference_stream_nll()
    out = {"streams": world, "steps_per_stream": steps, "graph_replays_per_stream": runner.replays,
           "tok_s_stream": round(world * steps / t_whole, 1),
           "tok_s_steady": round(world * (steps - steady_from) / t_steady, 1),
           "ms_per_token_steady": round(t_steady * 1e3 / (steps - steady_from), 3),
           "mean_nll": round(nll_sum / (world * steps), 5)}
    if rank == 0:
        out["stream0_mean_nll"] = round(own_mean, 5)
        out["reference_stream0_mean_nll"] = round(ref["mean_nll"], 5)
        out["stream0_rel_to_reference"] = float(f"{abs(own_mean - ref['mean_nll']) / ref['mean_nll']:.3e}")
    del runner, cache, model
    torch.cuda.empty_cache()
    return out


def model_leg(device: torch.device, rank: int, world: int, steps: int, warmup: int) -> dict:
    """The model-level numbers of the metric at this world size: Qwen3-0.6B with 1,024 slots
    streamed token by token from position 0 (tok/s, mean NLL against the reference's run),
    and Qwen3-0.6B with 32,768 slots and 32 streams split over the ranks (strong scaling);
    per-rank NLL sums and times gathered over NCCL."""
    from attention_sinks_b200 import streams
    out = {"qwen3-0.6b-1k": stream_qwen3_1k(device, rank, world)}
    spec = model_configs()["qwen3-0.6b-32k"]
    mine = list(streams.shard(spec["streams"], rank, world))
    local = stream_run(spec, mine, device, steps, warmup, "v1", spec["wave"])
    tot = gather(local)
    out["qwen3-0.6b-32k"] = {
        "streams_total": spec["streams"], "streams_per_gpu": len(mine),
        "waves_per_gpu": -(-len(mine) // spec["wave"]), "steps_per_stream": steps,
        "tok_s": round(tot["tokens"] / tot["seconds"], 1),
        "ms_per_step": round(tot["seconds"] * 1e3 / (steps * -(-len(mine) // spec["wave"])), 3),
        "mean_nll": round(tot["nll_sum"] / tot["tokens"], 6), "scaling": "strong",
        "cache_gb_per_wave": round(local["cache_gb"], 2)}
    return out


def run_model(args, workload: str) -> None:
    from attention_sinks_b200 import streams
    spec = model_configs()[workload]
    rank, world, local_rank = streams.init_from_env("nccl")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if spec["partition"]:
        mine = list(streams.shard(spec["streams"], rank, world))
    else:
        mine = list(range(rank * spec["streams"], (rank + 1) * spec["streams"]))
    local = stream_run(spec, mine, device, args.steps, args.warmup, args.cache, spec.get("wave"))
    tot = gather(local)
    if rank == 0:
        total = spec["streams"] * (world if not spec["partition"] else 1)
        line = {"metric": METRIC, "value": round(tot["tokens"] / tot["seconds"], 1), "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(tot["seconds"] * 1e3 / args.steps, 4),
                "higher_is_better": True, "scaling": "strong" if spec["partition"] else "weak",
                "vs_baseline": None, "dtype": "bf16 model / fp32 K" if args.cache == "v1" else "bf16 model / bf16 K",
                "data": "synthetic (random-init weights, uniform tokens, cache filled to the steady state)",
                "config": {"workload": workload, "cache": args.cache, "streams_total": total,
                           "streams_per_gpu": len(mine), "waves_per_gpu": -(-len(mine) // (spec.get("wave") or len(mine))),
                           "n_sink": spec["n_sink"], "window": spec["window"],
                           "layers": spec["cfg"]().num_hidden_layers, "cache_gb_per_wave": round(local["cache_gb"], 2),
                           "runner": "StreamRunner (CUDA graph)"},
                "mean_nll": round(tot["nll_sum"] / tot["tokens"], 6), "gpu_launches": tot["launches"]}
        print(json.dumps(line), flush=True)
    streams.shutdown()


def op_kinds() -> dict:
    """The two cache layouts' layer-step benchmarks."""
    return {
        "v1": dict(cls=OpBench, alg=alg_bytes, e2e=run_e2e, cpu=cpu_baseline, traffic="sink_stream_kernel_traffic.txt",
                   workload=f"sink-cache fused decode layer-step: evict 1 + rerotate -1 + append + GQA decode "
                            f"attention, Qwen3-0.6B layer shape (Hq {HQ}, Hkv {HKV}, head_dim {D})",
                   key_dtype="fp32", dtype="f32",
                   kernel="sink_stream_kernel<float, bf16, 128, 2, true> (timed with its halo pre-pass and "
                          "split-combine launches: the whole fused step)",
                   api="SinkLayer.update + decode_attention_forward (fused step)"),
        "v2": dict(cls=OpBenchV2, alg=alg_bytes_v2, e2e=run_e2e_v2, cpu=cpu_baseline_v2,
                   traffic="sink_v2_decode_step_traffic.txt",
                   workload=f"ring-buffer (v2) decode layer-step: ring write + region rotation (fp64 angles) + "
                            f"GQA decode attention over window + 1 + n_sink rows, Qwen3-0.6B layer shape "
                            f"(Hq {HQ}, Hkv {HKV}, head_dim {D})",
                   key_dtype="bf16", dtype="bf16",
                   kernel="sink_attend_tc_kernel<bf16, 2, true> (tcgen05, persistent, place work in two of its warps; "
                          "timed with the split combine: the whole v2 step)",
                   api="SinkLayerV2.update + decode_attention_forward (fused step)"),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--slots", type=int, default=32768)
    ap.add_argument("--streams", type=int, default=64, help="streams per GPU")
    ap.add_argument("--cache", choices=("v1", "v2"), default="v1",
                    help="v1: SinkCache fused step (default); v2: SinkCacheV2 ring-buffer step")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the model-level leg (streamed tok/s and mean NLL of Qwen3-0.6B at 1K and 32K slots)")
    ap.add_argument("--model-steps", type=int, default=32,
                    help="timed steady steps per stream of the 32K-slot model leg")
    ap.add_argument("--workload", default="op", choices=["op", "chunk"] + sorted(model_configs()),
                    help="op: the layer-step (default); otherwise a model-level streamed run")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.workload == "chunk":
        return chunk_bench(args)
    if args.workload != "op":
        return run_model(args, args.workload)

    from attention_sinks_b200 import streams
    kind = op_kinds()[args.cache]
    alg = kind["alg"]
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    config = {"workload": kind["workload"], "cache": args.cache,
              "slots": args.slots, "n_sink": N_SINK, "window": args.slots - N_SINK,
              "streams_per_gpu": args.streams, "global_streams": args.streams * max(world_env, 1),
              "key_dtype": kind["key_dtype"], "value_dtype": "bf16",
              "parallelism": f"streams x{max(world_env, 1)} (no collective)",
              "l2": "state per GPU larger than L2: no flush between steps"}

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        steps = max(1, args.steps)
        seconds = min(120.0, 0.3 * steps + 5)
        cb = kind["cpu"](args.slots, seconds=seconds, streams=args.streams)
        v = cb["value"] * 1.0
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": kind["dtype"],
                "data": "synthetic", "config": config, "cpu_baseline": cb,
                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    rank, world, local = streams.init_from_env("nccl")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from attention_sinks_b200 import _lib, build
    build.build()  # no-op when the shipped library is current

    bench = kind["cls"](args.streams, args.slots, device, seed=1000 + rank)
    small = bench.state_bytes() < 2 * L2_BYTES
    if small:
        config["l2"] = ("state smaller than 2x L2: between steps 256 MB written then 256 MB read (L2 left "
                        "clean), each step timed alone")
    l2_flush = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device=device) if small else None
    for i in range(args.warmup):
        bench.step(i)
    torch.cuda.synchronize()
    streams.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(device)
    clocks.start()
    n_launched = _lib.launch_count()
    ms = time_device(bench, args.steps, 0, l2_flush)
    launches = _lib.launch_count() - n_launched  # the library's kernels in the timed region
    clk = clocks.stop()
    torch.cuda.synchronize()
    streams.barrier()
    ms_max = streams.reduce_max(ms)
    status = bench.ws.read_status()
    if status:
        raise SystemExit(f"kernel status word {status}: a bounded wait ran out")

    e2e_ms, h2d, d2h = kind["e2e"](bench, args.steps, args.warmup)
    streams.barrier()
    e2e_max = streams.reduce_max(e2e_ms)

    bytes_step = alg(args.slots) * args.streams
    total_bytes = bytes_step * world
    value = total_bytes / (ms_max * 1e-3) / 1e9
    e2e_value = total_bytes / (e2e_max * 1e-3) / 1e9
    peak, peak_kind = hbm_peak()
    per_gpu = bytes_step / (ms * 1e-3) / 1e9
    prof = profiled_traffic(kind["traffic"])
    traffic = None
    if "traffic_bytes_per_launch" in prof:
        try:
            traffic = float(prof["traffic_bytes_per_launch"])
        except ValueError:
            traffic = None
    roofline = {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                "frac": round(per_gpu / peak, 4), "traffic": traffic, "peak_source": peak_kind,
                "kernel": kind["kernel"], "algorithmic_bytes_per_launch": bytes_step}
    if "traffic_workload" in prof:
        roofline["traffic_workload"] = prof["traffic_workload"]

    plan = dict(bench.plan)
    del bench
    torch.cuda.empty_cache()
    extra = {}
    if world == 1 and rank == 0:
        if not args.no_sweep:
            flush = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device=device)
            extra["sweep"] = sweep(device, flush, kind["cls"], alg)
            extra["sweep_graph_floor_us"] = graph_floor(device, flush)
            del flush
            torch.cuda.empty_cache()
        if not args.no_cpu:
            extra["cpu_baseline"] = kind["cpu"](args.slots, streams=args.streams)
    if not args.no_model:  # every rank: per-rank NLL sums and times are gathered over NCCL
        extra["model"] = model_leg(device, rank, world, args.model_steps, args.warmup)
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
                "us_per_layer": round(ms_max * 1e3, 2), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": kind["dtype"], "data": "synthetic", "config": config,
                "roofline": roofline,
                "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_max, 4), "api": kind["api"]},
                "gpu_launches": launches, "clocks": clk, "plan": plan}
        line.update(extra)
        print(json.dumps(line), flush=True)
    streams.shutdown()


if __name__ == "__main__":
    main()
