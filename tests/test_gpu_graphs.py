"""The training step replayed from a CUDA graph (captured the second time a batch shape is seen) gives
bit-identical results to the eagerly launched step, over several steps, through the trunk and through
cached features."""
import os

import numpy as np
import pytest
import torch

import simdyolo_b200 as sy
from simdyolo_b200 import data

pytestmark = pytest.mark.gpu


def run(graphs: bool, backbone: bool, steps=4):
    old = os.environ.get("SIMDYOLO_CUDA_GRAPHS")
    os.environ["SIMDYOLO_CUDA_GRAPHS"] = "1" if graphs else "0"
    try:
        cfg = sy.make_config("yolov8n", image_size=128, max_batch=3, max_boxes=6, backbone=backbone)
        s = sy.Session(cfg)
    finally:
        if old is None:
            del os.environ["SIMDYOLO_CUDA_GRAPHS"]
        else:
            os.environ["SIMDYOLO_CUDA_GRAPHS"] = old
    params, buffers = data.head_params(s, 5)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    if backbone:
        s.set_backbone(data.backbone_params("yolov8n", 1))
    rng = np.random.default_rng(9)
    imgs, truth = data.synthetic_batch(rng, 3, 128, 80, (1, 5), (8.0, 64.0))
    dev = torch.from_numpy(imgs).cuda()
    feats = [(rng.standard_normal((3, cfg.feature_channels[l], 128 >> (3 + l), 128 >> (3 + l))) * 0.7)
             .astype(np.float32) for l in range(3)]
    losses = []
    for i in range(steps):
        # same inputs every step: steps 2.. replay (or capture) the same graph key
        st = s.step_device(dev.data_ptr(), 3, truth) if backbone else s.step_features(feats, truth)
        losses.append((st.box, st.cls, st.dfl, st.positives))
    return losses, s.flat_params(), s.flat_buffers(), s.flat_velocity()


@pytest.mark.parametrize("backbone", [True, False])
def test_graph_replay_is_bit_identical_to_eager_steps(backbone):
    eager = run(False, backbone)
    graph = run(True, backbone)
    assert eager[0] == graph[0]
    for a, b in zip(eager[1:], graph[1:]):
        assert a.tobytes() == b.tobytes()


def run_rotating(graphs: bool, buffers=3, steps=7):
    """Steps over several device image buffers in turn (a data loader's batches): the graph captured on
    one buffer replays on the others, since the stem reads the image address from device memory."""
    old = os.environ.get("SIMDYOLO_CUDA_GRAPHS")
    os.environ["SIMDYOLO_CUDA_GRAPHS"] = "1" if graphs else "0"
    try:
        cfg = sy.make_config("yolov8n", image_size=128, max_batch=3, max_boxes=6)
        s = sy.Session(cfg)
    finally:
        if old is None:
            del os.environ["SIMDYOLO_CUDA_GRAPHS"]
        else:
            os.environ["SIMDYOLO_CUDA_GRAPHS"] = old
    params, buffers_ = data.head_params(s, 5)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers_)
    s.set_backbone(data.backbone_params("yolov8n", 1))
    rng = np.random.default_rng(21)
    batches = [data.synthetic_batch(rng, 3, 128, 80, (1, 5), (8.0, 64.0)) for _ in range(buffers)]
    devs = [torch.from_numpy(imgs).cuda() for imgs, _ in batches]
    out = []
    for i in range(steps):
        st = s.step_device(devs[i % buffers].data_ptr(), 3, batches[i % buffers][1])
        out.append((st.box, st.cls, st.dfl, st.positives))
    return out, s.flat_params(), s.flat_buffers(), s.flat_velocity()


def test_graph_replays_on_other_image_buffers_bit_identically():
    eager = run_rotating(False)
    graph = run_rotating(True)
    assert eager[0] == graph[0]
    for a, b in zip(eager[1:], graph[1:]):
        assert a.tobytes() == b.tobytes()


def test_launch_count_includes_graph_replays():
    """sy_cuda_launch_count counts the kernels a replayed graph runs, so a replayed step adds as many
    launches as the eager step it was captured from."""
    cfg = sy.make_config("yolov8n", image_size=128, max_batch=3, max_boxes=6)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 5)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    s.set_backbone(data.backbone_params("yolov8n", 1))
    rng = np.random.default_rng(4)
    imgs, truth = data.synthetic_batch(rng, 3, 128, 80, (1, 5), (8.0, 64.0))
    dev = torch.from_numpy(imgs).cuda()
    deltas = []
    for _ in range(4):   # eager, capture + launch, replay, replay
        n0 = sy.launch_count()
        s.step_device(dev.data_ptr(), 3, truth)
        deltas.append(sy.launch_count() - n0)
    assert deltas[0] > 100
    assert deltas[1] == deltas[2] == deltas[3] == deltas[0]
