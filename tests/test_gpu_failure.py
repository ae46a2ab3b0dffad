"""Failure paths of the step, made on the host or with a wait that is meant to run out.

* A non-finite loss or gradient stops the step before any update (YoloTrainer.cs:193,196;
  TrainingParameter.cs:40): the caller gets SY_ERR_NONFINITE (ArithmeticException), parameters, velocity,
  BatchNorm running statistics and AdamW step counts are bit-identical afterwards, and the session keeps
  working once the cause is gone.
* Every pipelined kernel bounds its mbarrier waits and reports a timed-out wait through an error flag
  instead of hanging; sy_cuda_wait_limit_selftest runs that path (TMEM allocated, a wait that nothing
  completes, TMEM freed) and the context stays usable.
"""
import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data

pytestmark = pytest.mark.gpu


def head_session(optimizer=sy.SY_OPT_SGD, seed=0):
    cfg = sy.make_config("yolov8n", image_size=128, max_batch=2, max_boxes=6, backbone=False, optimizer=optimizer,
                         lr=1e-3 if optimizer == sy.SY_OPT_ADAMW else 0.01)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, seed)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    return s, cfg


def batch(cfg, seed):
    rng = np.random.default_rng(seed)
    feats = [(rng.standard_normal((2, cfg.feature_channels[l], 128 >> (3 + l), 128 >> (3 + l))) * 0.7 + 0.2)
             .astype(np.float32) for l in range(3)]
    _, truth = data.synthetic_batch(rng, 2, 128, cfg.num_classes, boxes=(1, 5), wh=(8.0, 64.0))
    return feats, truth


def state(s):
    out = [s.flat_params(), s.flat_buffers(), s.flat_velocity(0), s.flat_velocity(1)]
    return [a.tobytes() for a in out] + [tuple(s.optimizer_steps())]


@pytest.mark.parametrize("optimizer", [sy.SY_OPT_SGD, sy.SY_OPT_ADAMW], ids=["sgd", "adamw"])
def test_nonfinite_step_changes_nothing_and_the_session_recovers(optimizer):
    s, cfg = head_session(optimizer)
    feats, truth = batch(cfg, 1)
    s.step_features(feats, truth)          # a finite step first: velocity and step counts are non-zero
    idx = next(t["index"] for t in s.tensors if t["name"] == "cv3.0.0.conv.weight")
    good = s.get_tensor(idx)
    bad = good.copy()
    bad.flat[7] = np.nan
    s.set_tensor(idx, bad)
    before = state(s)
    for _ in range(2):                     # the second attempt replays the captured step
        with pytest.raises(sy.NonFinite):
            s.step_features(feats, truth)
        assert state(s) == before
    s.set_tensor(idx, good)
    stats = s.step_features(feats, truth)
    assert np.isfinite(stats.cls) and stats.images == 2
    assert np.all(np.isfinite(s.flat_params()))
    s.close()


def test_nonfinite_input_features_are_reported_the_same_way():
    s, cfg = head_session()
    feats, truth = batch(cfg, 2)
    before = state(s)
    feats[1][0, 3, 2, 2] = np.inf
    with pytest.raises(sy.NonFinite):
        s.step_features(feats, truth)
    assert state(s) == before
    s.close()


def test_bounded_wait_gives_up_reports_and_frees_tmem():
    # a few thousand polls: the wait runs out within milliseconds
    assert sy.wait_limit_selftest(4096) == 21
    # TMEM was returned and the context is intact: run it again, then a tensor-core convolution
    assert sy.wait_limit_selftest(64) == 21
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 32, 8, 8)).astype(np.float32)
    w = rng.standard_normal((32, 32, 3, 3)).astype(np.float32)
    y = sy.conv2d_forward(x, w)
    assert np.all(np.isfinite(y))
    with pytest.raises(sy.InvalidArgument):
        sy.wait_limit_selftest(0)
