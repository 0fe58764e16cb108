"""Host-side logic of the N > 1 bench (one process per GPU, no collectives on
the data path) on CPU: world_size-2 `gloo` ranks check the max-over-ranks
timing that every rank agrees on, the whole-job throughput built from it, and
that the reference arm runs on rank 0 alone."""
import contextlib
import datetime
import io
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank, ws, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(ws), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        # each rank timed a different elapsed time for its own steps
        local_ms = 10.0 * (rank + 1)
        m = bench.max_over_ranks(local_ms, dist, "cpu")
        v = bench.job_throughput(ws, 8, 5, m)
        e_ws, e_rank, e_local = bench.dist_env()
        q.put((rank, m, v, (e_ws, e_rank, e_local)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_throughput_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert [p.exitcode for p in procs] == [0, 0]
    for rank, m, v, env in res:
        assert m == 20.0                          # the slowest rank's time, on every rank
        assert v == pytest.approx(2 * 8 * 5 / 0.020)   # all ranks' tokens over that time
        assert env == (2, rank, rank)


def test_single_process_needs_no_group():
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.job_throughput(1, 8, 50, 100.0) == pytest.approx(4000.0)


def test_reference_arm_runs_on_rank0_only(monkeypatch):
    """Under torchrun every rank starts the reference arm; ranks > 0 exit at
    once with no output and no CPU work."""
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    called = []
    monkeypatch.setattr(bench, "cpu_decode_rate", lambda *a, **k: called.append(a) or (1.0, "port"))

    class Args:
        steps, warmup, gpus = 2, 3, 2
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.reference_arm(Args())
    assert out.getvalue() == ""
    assert called == []


def test_reference_arm_rank0_line(monkeypatch):
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setattr(bench, "cpu_decode_rate", lambda threads, steps, warmup=0: (12.5, "reference"))

    class Args:
        steps, warmup, gpus = 2, 3, 2
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.reference_arm(Args())
    import json
    line = json.loads(out.getvalue())
    assert line["impl"] == "reference"
    assert line["value"] == 12.5 and line["e2e"]["value"] == 12.5
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "reference"
