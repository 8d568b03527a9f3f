"""Multi-process host logic on CPU (gloo, world size 2).

bench.py runs one independent decode replica per GPU; the only cross-rank
traffic is the timing reduction (max over ranks) and barriers.  These tests
run that plumbing as two CPU processes, including a rank that leaves between
steps: the survivor must get an error from its next collective (short
process-group timeout), not hang.
"""

import os
import socket

import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, q, fail_rank):
    import datetime
    import sys

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    os.environ.update(
        MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws), LOCAL_RANK=str(rank)
    )
    import bench

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    try:
        assert bench.dist_env() == (ws, rank, rank)
        bench.barrier(True)
        if rank == fail_rank:
            q.put((rank, "left", None))
            q.close()
            q.join_thread()  # flush the message before the abrupt exit
            os._exit(0)  # leaves between steps, nothing in flight
        v = bench.reduce_max(10.0 * (rank + 1), True)
        bench.barrier(True)
        q.put((rank, "ok", v))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(ws, fail_rank=-1, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q, fail_rank)) for r in range(ws)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(ws):
        r, status, v = q.get(timeout=timeout)
        out[r] = (status, v)
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_timing_reduction_is_max_over_ranks():
    out = _run(2)
    assert out[0] == ("ok", 20.0) and out[1] == ("ok", 20.0)


def test_rank_leaving_is_detected_not_hung():
    out = _run(2, fail_rank=1)
    assert out[1][0] == "left"
    assert out[0][0] == "error"


def test_bench_byte_accounting():
    import bench

    # 512 tokens at positions 1023..1534: each reads p cached positions, writes 1
    kv = bench.kv_bytes(1023, 512)
    assert kv == bench.KV_BYTES_PER_POS * sum(range(1024, 1536))
    assert bench.launch_bytes() == 512 * 1_192_101_888 + kv
    # weight bytes: 28 x 15,728,640 x 2 + norms + final norm + embed row + LM head
    assert bench.WEIGHT_BYTES == 28 * 15_728_640 * 2 + 28 * 4_608 + 2_048 + 2_048 + 151_936 * 1_024 * 2


@pytest.mark.parametrize("n", [1, 3])
def test_prompt_seeds_differ_per_rank(n):
    import bench

    a, b = bench.prompt_for_rank(0), bench.prompt_for_rank(n)
    assert len(a) == bench.PROMPT_LEN and a != b
    assert all(0 <= t < 151936 for t in a)


def test_clock_sampler_follows_visible_devices(monkeypatch):
    """Each rank samples the clocks of its own GPU: CUDA device i is entry i
    of CUDA_VISIBLE_DEVICES when that is set."""
    import sys

    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    assert bench.smi_gpu_id(1) == "1"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert bench.smi_gpu_id(0) == "3" and bench.smi_gpu_id(1) == "5"
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-aaaa, GPU-bbbb")
    assert bench.smi_gpu_id(1) == "GPU-bbbb"
