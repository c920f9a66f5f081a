"""Data-parallel Lloyd host logic across 2 gloo ranks on CPU (no GPU): sharding, the
single all-reduce of the k x (d+1) statistics per iteration and the finalisation give
every rank the same centers, equal to the single-process result."""
import os
import socket
import subprocess
import sys
import time

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
WORKER = os.path.join(HERE, "dist_worker.py")


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def run_ranks(world, tmp_path, **extra_env):
    port = free_port()
    procs, outs = [], []
    for r in range(world):
        out = str(tmp_path / f"c_{world}_{r}.npy")
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="", **extra_env)
        procs.append(subprocess.Popen([sys.executable, WORKER, out], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT))
        outs.append(out)
    for p in procs:
        try:
            log, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail("gloo ranks did not finish")
        assert p.returncode == 0, log.decode()[-2000:]
    return [np.load(o) for o in outs]


def test_two_gloo_ranks_match_single_process(tmp_path):
    single = run_ranks(1, tmp_path)[0]
    two = run_ranks(2, tmp_path)
    np.testing.assert_array_equal(two[0], two[1])
    np.testing.assert_array_equal(two[0], single)


def test_rank_leaving_between_steps_ends_the_others_next_step(tmp_path):
    """Failure detection of the data-parallel loop, made on the host: rank 1 exits after
    its first Lloyd step.  Rank 0's next step (its all-reduce) must end with an error
    within the process group's timeout (10 s here), not wait for good."""
    port = free_port()
    procs, t0 = [], time.monotonic()
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", LOCAL_RANK=str(r), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="", LEAVE_AFTER="1", PG_TIMEOUT="10")
        procs.append(subprocess.Popen([sys.executable, WORKER, str(tmp_path / f"leave_{r}.npy")], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    try:
        logs = [p.communicate(timeout=120)[0].decode() for p in procs]
    except subprocess.TimeoutExpired:
        for q in procs:
            q.kill()
        pytest.fail("the surviving rank waited for good")
    elapsed = time.monotonic() - t0
    assert procs[1].returncode == 0, logs[1][-2000:]
    assert procs[0].returncode == 3, logs[0][-2000:]
    err = (tmp_path / "leave_0.npy.err").read_text()
    assert err.startswith("step 1:"), err
    assert elapsed < 60, elapsed


def test_shard_rows_cover_every_row_once():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "euclid-cuda_b200"))
    import kmeans
    for n in (0, 1, 7, 3001):
        for world in (1, 2, 3, 8):
            spans = [kmeans.shard_rows(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
