"""YoloTrainer.EvaluateLoss through the shim (sy_cuda_eval_loss*): BatchNorm with the running
statistics, the loss without gradients, nothing updated; against the oracle's evaluation-mode head."""
import ctypes as C

import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from oracle import oracle as O
from tests.helpers import head_desc

pytestmark = pytest.mark.gpu
TOL = 2e-3


def oracle_eval(cfg, params, buffers, feats, truth):
    d = head_desc(cfg)
    total = dict(box=0.0, cls=0.0, dfl=0.0, positives=0)
    for b in range(feats[0].shape[0]):
        fs = [np.ascontiguousarray(f[b], np.float32) for f in feats]
        fp = (C.c_void_p * 3)(*[f.ctypes.data_as(C.c_void_p) for f in fs])
        out = O.Loss()
        assert O.lib().syo_head_eval_image(C.byref(d), params, buffers.copy(), fp, O.boxes(truth[b]), len(truth[b]),
                                           C.byref(out)) == 0
        total["box"] += out.box
        total["cls"] += out.cls
        total["dfl"] += out.dfl
        total["positives"] += out.positives
    return total


@pytest.mark.parametrize("model", ["yolov8n", "yolo11s"])
def test_eval_loss_uses_running_statistics_and_changes_nothing(model):
    rng = np.random.default_rng(61)
    cfg = sy.make_config(model, image_size=128, max_batch=3, max_boxes=8, backbone=False)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 0)
    # running statistics away from the fresh (0, 1) so that evaluation mode is visible
    off = 0
    for t in s.tensors:
        if t["kind"] != 1:
            continue
        n = t["numel"]
        if t["name"].endswith("running_mean"):
            buffers[off:off + n] = rng.normal(0.0, 0.2, n)
        elif t["name"].endswith("running_var"):
            buffers[off:off + n] = rng.uniform(0.5, 2.0, n)
        off += n
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    feats = []
    for l in range(3):
        h = 128 >> (3 + l)
        feats.append((rng.standard_normal((3, cfg.feature_channels[l], h, h)) * 0.7 + 0.2).astype(np.float32))
    _, truth = data.synthetic_batch(rng, 3, 128, cfg.num_classes, boxes=(1, 8), wh=(8.0, 64.0))
    stats = s.eval_loss_features(feats, truth)
    want = oracle_eval(cfg, params, buffers, feats, truth)
    assert stats.images == 3
    assert stats.positives == want["positives"]
    assert abs(stats.cls - want["cls"]) <= TOL * abs(want["cls"])
    assert abs(stats.box - want["box"]) <= TOL * max(abs(want["box"]), 1.0)
    assert abs(stats.dfl - want["dfl"]) <= TOL * max(abs(want["dfl"]), 1.0)
    # evaluation mode differs from the training-mode loss of the same batch
    d = head_desc(cfg)
    fs = [np.ascontiguousarray(f[0], np.float32) for f in feats]
    fp = (C.c_void_p * 3)(*[f.ctypes.data_as(C.c_void_p) for f in fs])
    train0, eval0 = O.Loss(), O.Loss()
    O.lib().syo_head_image(C.byref(d), params, buffers.copy(), fp, O.boxes(truth[0]), len(truth[0]),
                           np.zeros_like(params), C.byref(train0), 0, None)
    O.lib().syo_head_eval_image(C.byref(d), params, buffers.copy(), fp, O.boxes(truth[0]), len(truth[0]),
                                C.byref(eval0))
    assert abs(train0.cls - eval0.cls) > 10 * TOL * abs(eval0.cls)
    # nothing moved
    assert s.flat_params().tobytes() == params.tobytes()
    assert s.flat_buffers().tobytes() == buffers.tobytes()
    assert not s.flat_velocity().any()
