"""Multi-GPU host logic on CPU `gloo` ranks (world size 2): stream partitioning, the max of
per-rank times and the sums of per-rank results that bench.py uses around its timed
region, and failure detection when a rank leaves between steps."""

import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from attention_sinks_b200 import streams


@pytest.mark.parametrize("n", [0, 1, 7, 32, 64, 128])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_covers_every_stream_once(n, world):
    parts = [streams.shard(n, r, world) for r in range(world)]
    assert [i for p in parts for i in p] == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_bad_partitions():
    with pytest.raises(ValueError):
        streams.shard(8, 2, 2)
    with pytest.raises(ValueError):
        streams.shard(8, 0, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exit_now(queue, msg):
    """Leave the process at once (no teardown), after the message is really sent."""
    queue.put(msg)
    queue.close()
    queue.join_thread()
    os._exit(0)


def _worker(rank, world, port, queue, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        r, w, _ = streams.init_from_env("gloo", timeout_s=10)
        if mode == "ok":
            mine = streams.shard(64, r, w)
            mx = streams.reduce_max(float(r + 1) * 1.5)         # per-rank "time"
            sums = streams.reduce_sum([len(mine), sum(mine)])   # e.g. token count, NLL sum
            streams.barrier()
            queue.put((r, mx, sums))
            streams.shutdown()
        else:  # a rank leaves between steps, with nothing in flight
            if r == 1:
                _exit_now(queue, (r, "left"))
            time.sleep(0.5)
            try:
                streams.reduce_max(1.0)
                msg = (r, "no error")
            except Exception as e:  # the next collective ends with an error, not a hang
                msg = (r, "error:" + type(e).__name__)
            _exit_now(queue, msg)
    except Exception as e:
        queue.put((rank, "setup:" + repr(e)))


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = [queue.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_gloo_ranks_reduce_times_and_results():
    out = _run("ok")
    assert [o[0] for o in out] == [0, 1]
    for _, mx, sums in out:
        assert mx == 3.0                      # the slowest rank's time
        assert sums == [64.0, float(sum(range(64)))]


def test_lost_rank_ends_the_next_collective_with_an_error():
    out = dict((r, msg) for r, msg in _run("lost"))
    assert out[1] == "left"
    assert out[0].startswith("error:"), out[0]
