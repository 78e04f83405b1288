"""Multi-process window partitioning on CPU (gloo, world size 2): the N > 1
plumbing of the throughput sweep, including host-side failure detection (a
rank that crashes or hangs between windows has its windows re-run)."""

import json
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

from fastdialoguesidon_b200.windows import WindowRunner, assign


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _window_record(w: int) -> float:
    """A deterministic per-window result: the oracle on a tiny seeded window."""
    from oracle import flexrel_oracle as O

    gen = torch.Generator().manual_seed(1000 + w)
    qkv = torch.randn(40, 3 * 64, generator=gen).half()
    rel = torch.randn(73, 64, generator=gen).half()
    return float(O.flexrel_attention(qkv, 1, 1, rel).double().sum())


def _worker(rank: int, world: int, port: int, n: int, mode: str, out_path: str):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    store = torch.distributed.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    torch.distributed.init_process_group("gloo", store=store, rank=rank, world_size=world,
                                         timeout=timedelta(seconds=30))
    torch.distributed.barrier()  # the data path itself has no collective; this only starts both ranks together
    done = []

    def process(w: int) -> float:
        if rank == 1 and mode == "crash" and len(done) == 1:
            os._exit(3)                      # the rank dies between windows
        if rank == 1 and mode == "hang" and len(done) == 1:
            time.sleep(3600)                 # the rank stops making progress
        if rank == 1 and mode == "slow_first" and not done:
            time.sleep(4.0)                  # a healthy but slow first window (> dead_after_s)
        done.append(w)
        return _window_record(w)

    if rank == 1 and mode == "late_start":
        time.sleep(4.0)                      # starts well after rank 0 (> dead_after_s)
    runner = WindowRunner(store, rank, world, n, heartbeat_s=0.05, dead_after_s=1.5,
                          window_timeout_s=2.5 if mode == "hang" else 30.0, start_grace_s=20.0,
                          deadline_s=60)
    rep = runner.run(process)
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump({"results": rep.results, "failed": rep.failed_ranks, "requeued": rep.requeued}, f)
    # no collective after a possible failure: rank 0 exits on its own
    os._exit(0)


def _run(mode: str, tmp_path, n: int = 7):
    ctx = mp.get_context("spawn")
    port = _free_port()
    out = str(tmp_path / f"{mode}.json")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, mode, out)) for r in range(2)]
    for p in procs:
        p.start()
    procs[0].join(timeout=120)
    for p in procs[1:]:
        p.join(timeout=1 if mode == "hang" else 60)
        if p.is_alive():
            p.kill()
            p.join()
    assert procs[0].exitcode == 0
    with open(out) as f:
        return json.load(f), procs


def test_assign_round_robin():
    assert assign(7, 2) == [[0, 2, 4, 6], [1, 3, 5]]
    assert sorted(sum(assign(64, 8), [])) == list(range(64))


def test_two_ranks_all_windows(tmp_path):
    rep, _ = _run("ok", tmp_path)
    assert rep["failed"] == [] and rep["requeued"] == {}
    assert {int(k): v for k, v in rep["results"].items()} == pytest.approx({w: _window_record(w) for w in range(7)})


@pytest.mark.parametrize("mode", ["crash", "hang"])
def test_failed_rank_windows_are_rerun(tmp_path, mode):
    rep, procs = _run(mode, tmp_path)
    assert rep["failed"] == [1]
    # rank 1 finished window 1, then failed: its remaining windows 3 and 5 were re-run by rank 0
    assert sorted(int(w) for w in rep["requeued"]) == [3, 5]
    assert {int(k): v for k, v in rep["results"].items()} == pytest.approx({w: _window_record(w) for w in range(7)})
    if mode == "crash":
        assert procs[1].exitcode == 3


@pytest.mark.parametrize("mode", ["slow_first", "late_start"])
def test_slow_healthy_rank_is_not_failed(tmp_path, mode):
    """No false positives: a rank whose first window outlasts dead_after_s, or
    that joins late, keeps its windows (heartbeat thread / start grace)."""
    rep, procs = _run(mode, tmp_path)
    assert rep["failed"] == [] and rep["requeued"] == {}
    assert {int(k): v for k, v in rep["results"].items()} == pytest.approx({w: _window_record(w) for w in range(7)})
