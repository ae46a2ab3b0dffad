"""Data parallelism (one process per GPU, images sharded contiguously, NCCL inside the session).

CPU: two gloo ranks exercise the host plumbing (shards, NCCL id broadcast, max over ranks).
GPU: two ranks on two GPUs step shards of a global batch; a single-GPU session stepping the whole
batch must give the same update (per-image BatchNorm statistics and loss normalisation make images
independent, DetectionLoss.cs:92-98), the same running statistics (folded in global image order,
HeadOperations.cs:164-165) and the same step statistics.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import dp_cases
from helpers import rel_l2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_contiguous_and_equal():
    from simdyolo_b200 import dp

    assert [dp.shard_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        dp.shard_range(6, 0, 4)
    with pytest.raises(ValueError):
        dp.shard_range(8, 4, 4)


def test_gloo_two_ranks_host_plumbing():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=dp_cases.gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get() for _ in range(2))
    for rank, ok_images, ok_boxes, ok_id, mx in res:
        assert ok_images and ok_boxes and ok_id
        assert mx == 3.0


@pytest.mark.gpu
def test_two_gpu_step_matches_single_gpu(tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import simdyolo_b200 as sy

    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", dp_cases.__file__, str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    ranks = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]

    cfg = sy.make_config("yolov8n", image_size=dp_cases.DP_IMAGE, max_batch=dp_cases.DP_GLOBAL, device=0)
    with sy.Session(cfg) as sess:
        dp_cases.init_session(sess, "yolov8n")
        p0 = sess.flat_params()
        single = dp_cases.run_steps(sess, dp_cases.global_batch())

    for r in ranks:
        # every rank holds the same replica after the update
        np.testing.assert_array_equal(r["params"], ranks[0]["params"])
        np.testing.assert_array_equal(r["buffers"], ranks[0]["buffers"])
        # per-image work is identical; only the order of the sum over images differs
        assert rel_l2(r["params"] - p0, single["params"] - p0) < 1e-4
        assert rel_l2(r["velocity"], single["velocity"]) < 1e-4
        assert rel_l2(r["grads"], single["grads"]) < 1e-4
        assert rel_l2(r["buffers"], single["buffers"]) < 1e-6
        np.testing.assert_allclose(r["stats"][:, :3], single["stats"][:, :3], rtol=1e-5)
        np.testing.assert_array_equal(r["stats"][:, 3:6], single["stats"][:, 3:6])
        np.testing.assert_allclose(r["stats"][:, 6], single["stats"][:, 6], rtol=1e-4)


@pytest.mark.gpu
def test_peer_that_leaves_ends_the_next_step_with_comm_error(tmp_path):
    """A rank that leaves between steps: the survivor's next collective is ended by the session's bounded
    wait (ncclCommAbort after comm_timeout_ms = 3 s) with SY_ERR_COMM instead of blocking forever
    (VulkanBackend.cs:323-style InvalidOperationException on the C# side)."""
    import json

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import simdyolo_b200 as sy

    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", dp_cases.__file__, "timeout", str(tmp_path)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads((tmp_path / "timeout.json").read_text())
    assert res["status"] == sy.SY_ERR_COMM, res
    assert 2.5 <= res["elapsed"] < 60, res
    assert res["second"] == sy.SY_ERR_COMM
    assert res["fresh_ok"]
