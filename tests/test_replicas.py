"""The replica plumbing of the multi-GPU runs (dinov3_b200/replicas.py, used by bench.py under
torchrun), as world-size-2 gloo process groups on the host: the barrier, the max over ranks,
each rank's image slice and work share, the whole-job throughput; a rank that leaves early makes
the other rank's next collective fail instead of hanging; and the reference arm's other ranks
exit without work."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _env(rank: int, world: int, port: int) -> dict:
    return {"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
            "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)}


def _rank_main(rank, world, port, mode, q):
    os.environ.update(_env(rank, world, port))
    try:
        from dinov3_b200 import synth
        from dinov3_b200.replicas import Replicas

        reps = Replicas("gloo", timeout_s=20)
        if mode == "leave" and rank == 1:
            os._exit(0)  # leaves between steps, without a word to the others
        reps.barrier()
        got = {"rank": reps.rank, "world": reps.world, "max": reps.max(1.5 * (rank + 1)),
               "first": reps.first_image(64), "share": reps.share(1001),
               "throughput": reps.throughput(64 * 10, 2.0),
               "image": synth.images(1000, 2, first=reps.first_image(2))[1]}
        reps.close()
        q.put(got)
    except Exception as e:  # reported to the parent
        q.put({"rank": rank, "error": repr(e)})


def _run(mode: str, world: int = 2, timeout: float = 120.0):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    expected = world if mode == "ok" else 1
    results = [q.get(timeout=timeout) for _ in range(expected)]
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r["rank"])


def test_two_gloo_ranks_barrier_max_slices_and_throughput():
    import numpy as np

    from dinov3_b200 import synth

    results = _run("ok")
    assert [r.get("error") for r in results] == [None, None]
    assert [(r["rank"], r["world"]) for r in results] == [(0, 2), (1, 2)]
    assert all(r["max"] == 3.0 for r in results)          # the slowest rank's value on every rank
    assert [r["first"] for r in results] == [0, 64]         # disjoint image slices
    assert sum(r["share"] for r in results) == 1001         # shares cover the job
    assert [r["share"] for r in results] == [501, 500]
    assert all(r["throughput"] == 640.0 for r in results)   # 2 ranks x 640 images / 2 s
    whole = synth.images(1000, 4)                           # rank r's images are images 2r, 2r+1
    np.testing.assert_array_equal(results[0]["image"], whole[1])
    np.testing.assert_array_equal(results[1]["image"], whole[3])


def test_a_rank_that_leaves_fails_the_next_collective():
    results = _run("leave")
    assert len(results) == 1 and results[0]["rank"] == 0
    assert "error" in results[0]  # an error from gloo (peer gone or timeout), not a hang


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, **_env(1, 2, _free_port()))
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "0"],
                         env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""
