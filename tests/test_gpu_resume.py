"""Checkpoint / resume through the C ABI (YoloTrainer.cs:124-155 Resume, :265-306 checkpoint; the
reference's integration test requires the optimizer bytes to be identical after load and a resumed run to
continue like an uninterrupted one, tests/SimdYolo.Training.Tests/TrainingMatrix.cs:115-132).

k steps, export every parameter and buffer (sy_cuda_get_tensor, Snapshot order), every optimizer moment
(sy_cuda_get_optimizer_state) and, for AdamW, the per-group step counts; import them into a fresh session
and run m more steps.  The exported state must read back bit-identical, and because every kernel of the
step is deterministic the resumed run must end bit-identical to k + m uninterrupted steps.
"""
import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data

pytestmark = pytest.mark.gpu
SIZE, BATCH, K, M = 128, 2, 2, 3


def new_session(optimizer):
    cfg = sy.make_config("yolov8n", image_size=SIZE, max_batch=BATCH, max_boxes=6, optimizer=optimizer,
                         lr=1e-3 if optimizer == sy.SY_OPT_ADAMW else 0.01,
                         weight_decay=0.05 if optimizer == sy.SY_OPT_ADAMW else 5e-4)
    s = sy.Session(cfg)
    s.set_backbone(data.backbone_params("yolov8n", seed=0))
    return s, cfg


def batches(cfg):
    rng = np.random.default_rng(31)
    return [data.synthetic_batch(rng, BATCH, SIZE, cfg.num_classes, boxes=(1, 6), wh=(8.0, 64.0))
            for _ in range(K + M)]


def export(s):
    tensors = [s.get_tensor(t["index"]).copy() for t in s.tensors]
    moments = [[s.get_optimizer_state(t["index"], m) for t in s.params] for m in range(2)]
    return tensors, moments, s.optimizer_steps()


def load(s, snapshot):
    tensors, moments, steps = snapshot
    for t, v in zip(s.tensors, tensors):
        s.set_tensor(t["index"], v)
    for m in range(2):
        for t, v in zip(s.params, moments[m]):
            s.set_optimizer_state(t["index"], m, v)
    s.set_optimizer_steps(steps)


def same(a, b):
    ta, ma, sa = a
    tb, mb, sb = b
    return (all(x.tobytes() == y.tobytes() for x, y in zip(ta, tb)) and
            all(x.tobytes() == y.tobytes() for u, v in zip(ma, mb) for x, y in zip(u, v)) and sa == sb)


@pytest.mark.parametrize("optimizer", [sy.SY_OPT_SGD, sy.SY_OPT_ADAMW], ids=["sgd", "adamw"])
def test_resume_continues_bit_identical(optimizer):
    a, cfg = new_session(optimizer)
    params, buffers = data.head_params(a, seed=5)
    a.set_flat_params(params)
    a.set_flat_buffers(buffers)
    work = batches(cfg)
    for images, truth in work:
        a.step(images, truth)
    uninterrupted = export(a)
    a.close()

    b, _ = new_session(optimizer)
    b.set_flat_params(params)
    b.set_flat_buffers(buffers)
    for images, truth in work[:K]:
        b.step(images, truth)
    checkpoint = export(b)
    b.close()
    if optimizer == sy.SY_OPT_ADAMW:
        assert checkpoint[2][0] == K

    c, _ = new_session(optimizer)
    load(c, checkpoint)
    assert same(export(c), checkpoint)   # the state reads back byte for byte
    for images, truth in work[K:]:
        c.step(images, truth)
    resumed = export(c)
    c.close()
    assert same(resumed, uninterrupted)


def test_negative_step_counts_are_rejected():
    s, _ = new_session(sy.SY_OPT_ADAMW)
    with pytest.raises(ValueError):
        s.set_optimizer_steps([1, -1, 0])
    s.close()
