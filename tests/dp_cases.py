"""Worker bodies for the data-parallel tests (imported by spawned ranks; not a test module).

`gloo_rank` checks the host-side plumbing of simdyolo_b200.dp on CPU; `nccl_rank` (run under
torch.distributed.run on 2 GPUs) steps one shard of a global batch through a data-parallel session
and saves what a single-GPU session stepping the whole batch must reproduce.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# global batch of the GPU data-parallel parity case
DP_IMAGE = 256
DP_GLOBAL = 4
DP_STEPS = 2


def gloo_rank(rank: int, world: int, port: int, results):
    import torch.distributed as dist

    from simdyolo_b200 import data, dp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(7)
        imgs, boxes = data.synthetic_batch(rng, 6, 64, 80)
        mine, my_boxes = dp.shard(imgs, boxes, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, (mine.tobytes(), my_boxes))
        nid = dp.broadcast_nccl_id(dist, rank, make_id=lambda: bytes(range(128)))
        mx = dp.max_over_ranks(dist, float(rank + 1) * 1.5)
        ok_images = b"".join(g[0] for g in gathered) == imgs.tobytes()
        ok_boxes = [bx for g in gathered for bx in g[1]] == list(boxes)
        results.put((rank, ok_images, ok_boxes, nid == bytes(range(128)), mx))
    finally:
        dist.destroy_process_group()


def global_batch():
    from simdyolo_b200 import data

    rng = np.random.default_rng(11)
    return [data.synthetic_batch(rng, DP_GLOBAL, DP_IMAGE, 80) for _ in range(DP_STEPS)]


def init_session(sess, model):
    import simdyolo_b200 as sy
    from simdyolo_b200 import data

    params, buffers = data.head_params(sess, seed=0)
    sess.set_flat_params(params)
    sess.set_flat_buffers(buffers)
    sess.set_backbone(data.backbone_params(sy.MODELS[model], seed=0))


def run_steps(sess, batches, rank=0, world=1):
    from simdyolo_b200 import dp

    stats = []
    for imgs, boxes in batches:
        mine, my_boxes = dp.shard(imgs, boxes, rank, world)
        st = sess.step(mine, my_boxes)
        stats.append([st.box, st.cls, st.dfl, st.positives, st.images, st.box_has_grad, st.grad_checksum])
    return dict(params=sess.flat_params(), buffers=sess.flat_buffers(), velocity=sess.flat_velocity(),
                grads=sess.last_gradients(), stats=np.array(stats, np.float64))


def nccl_rank(out_dir: str):
    """One rank of the 2-GPU parity case (launched by torch.distributed.run)."""
    import torch
    import torch.distributed as dist

    from simdyolo_b200 import dp

    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    try:
        sess = dp.create_session(dist, "yolov8n", local_rank, DP_GLOBAL // world, image_size=DP_IMAGE)
        init_session(sess, "yolov8n")
        res = run_steps(sess, global_batch(), rank, world)
        sess.close()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def nccl_timeout_rank(out_dir: str):
    """Failure case (launched by torch.distributed.run on 2 GPUs, NCCL_NVLS_ENABLE=0): both ranks step once,
    then rank 1 leaves between steps, with nothing of its own in flight.  Rank 0's next step enqueues its
    collectives, which no peer completes: the session's bounded wait gives up after comm_timeout_ms, aborts
    the communicator and returns SY_ERR_COMM; the session refuses further steps, closes cleanly, and a fresh
    single-GPU session on the same device still steps."""
    import json
    import time

    import torch
    import torch.distributed as dist

    import simdyolo_b200 as sy
    from simdyolo_b200 import dp

    local_rank = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local_rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    sess = dp.create_session(dist, "yolov8n", local_rank, 1, image_size=128, comm_timeout_ms=3000)
    init_session(sess, "yolov8n")
    from simdyolo_b200 import data
    imgs, boxes = data.synthetic_batch(np.random.default_rng(5), world, 128, 80)
    mine, my_boxes = dp.shard(imgs, boxes, rank, world)
    sess.step(mine, my_boxes)
    torch.cuda.synchronize()
    dist.barrier()          # both ranks finished step 1: nothing is in flight
    if rank == 1:
        os._exit(0)         # leaves without another word to its peer
    time.sleep(1.0)
    res = {}
    t0 = time.monotonic()
    try:
        sess.step(mine, my_boxes)
        res["status"] = 0
    except sy.SyError as e:
        res["status"], res["message"] = e.status, str(e)
    res["elapsed"] = time.monotonic() - t0
    try:
        sess.step(mine, my_boxes)
        res["second"] = 0
    except sy.SyError as e:
        res["second"] = e.status
    sess.close()
    cfg = sy.make_config("yolov8n", image_size=128, max_batch=1, device=local_rank)
    with sy.Session(cfg) as fresh:
        init_session(fresh, "yolov8n")
        st = fresh.step(mine, my_boxes)
        res["fresh_ok"] = bool(np.isfinite(st.cls))
    with open(os.path.join(out_dir, "timeout.json"), "w") as f:
        json.dump(res, f)
    os._exit(0)             # the control-plane group has lost its peer: no collective teardown


if __name__ == "__main__":
    if sys.argv[1] == "timeout":
        nccl_timeout_rank(sys.argv[2])
    else:
        nccl_rank(sys.argv[1])
