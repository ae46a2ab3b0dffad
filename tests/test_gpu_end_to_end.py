"""End-to-end detection heads through the session (C ABI) against the oracle: the one2one_cv2 /
one2one_cv3 branches after cv2 / cv3 (DetectionHead.cs:20-26), the second loss with its own top-k
(DetectionHead.cs:105-115), the progressive weight schedule (DetectionHead.cs:120) set through
sy_cuda_set_epoch, and separate optimizer groups for the two box branches (a box branch only steps
when its own loss assigned a positive).  Tolerances are the TF32 bound of the other step tests."""
import ctypes as C

import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from oracle import oracle as O
from tests.helpers import head_desc, oracle_head_step, oracle_head_step_adamw, rel_l2

pytestmark = pytest.mark.gpu
TOL = 2e-3


def make(model, reg_max, batch=2, image_size=128, schedule=5, optimizer=sy.SY_OPT_SGD, nc=80):
    kw = dict(optimizer=optimizer)
    if optimizer == sy.SY_OPT_ADAMW:
        kw.update(lr=1e-3, weight_decay=0.05)
    cfg = sy.make_config(model, image_size=image_size, max_batch=batch, max_boxes=8, num_classes=nc,
                         backbone=False, end_to_end=True, reg_max=reg_max, schedule_epochs=schedule, **kw)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 3)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    return s, cfg, params, buffers


def features(cfg, batch, rng):
    return [(rng.standard_normal((batch, cfg.feature_channels[l], cfg.image_size >> (3 + l),
                                  cfg.image_size >> (3 + l))) * 0.7 + 0.2).astype(np.float32) for l in range(3)]


def test_one_to_one_branches_follow_the_one_to_many_branches():
    s, cfg, params, _ = make("yolo11s", 1)
    names = [t["name"] for t in s.params]
    n = len(names) // 2
    assert names[:n] == [x for x in names if not x.startswith("one2one_")]
    assert names[n:] == ["one2one_" + x for x in names[:n]]
    assert names[n] == "one2one_cv2.0.0.conv.weight"
    last = next(t for t in s.params if t["name"] == "one2one_cv2.2.2.weight")
    assert tuple(last["shape"]) == (4, cfg.box_blocks[2][1].oc, 1, 1)   # reg_max 1: four distances
    buffers = [t["name"] for t in s.tensors if t["kind"] == 1]
    assert buffers[len(buffers) // 2] == "one2one_cv2.0.0.bn.running_mean"
    d = head_desc(cfg)
    assert O.lib().syo_head_param_count(C.byref(d)) == params.size


@pytest.mark.parametrize("model,reg_max,epoch", [("yolov8n", 16, 0), ("yolo11s", 1, 2), ("yolov8n", 1, 7)])
def test_end_to_end_step_matches_oracle(model, reg_max, epoch):
    rng = np.random.default_rng(40 + epoch)
    s, cfg, params, buffers = make(model, reg_max)
    s.set_epoch(epoch)
    feats = features(cfg, 2, rng)
    _, truth = data.synthetic_batch(rng, 2, cfg.image_size, cfg.num_classes, boxes=(1, 6), wh=(8.0, 64.0))
    stats = s.step_features(feats, truth)
    grad = s.last_gradients()
    losses, ograd, oparams, obuffers, ovel, conn = oracle_head_step(cfg, s.tensors, params, buffers,
                                                                    np.zeros_like(params), feats, truth, epoch)
    for k in ("box", "cls", "dfl"):
        want = sum(l[k] for l in losses)
        assert abs(getattr(stats, k) - want) <= TOL * max(abs(want), 1.0), k
    assert stats.positives == sum(l["positives"] for l in losses)
    assert stats.box_has_grad == conn == 3
    assert rel_l2(grad, ograd) < TOL
    assert rel_l2(s.flat_params() - params, oparams - params) < TOL
    assert rel_l2(s.flat_velocity(), ovel) < TOL
    assert rel_l2(s.flat_buffers(), obuffers) < TOL


def test_background_batch_leaves_both_box_branches():
    rng = np.random.default_rng(8)
    s, cfg, params, _ = make("yolov8n", 16)
    stats = s.step_features(features(cfg, 2, rng), [[], []])
    assert stats.positives == 0 and stats.box_has_grad == 0
    new = s.flat_params()
    off = 0
    for t in s.params:
        n = t["numel"]
        if sy.tensor_group(t["name"]):
            assert new[off:off + n].tobytes() == params[off:off + n].tobytes(), t["name"]
        off += n


def test_progressive_adamw_groups_match_oracle():
    """Two AdamW steps, the second without boxes: the class branches of both sets step twice, the
    two box groups once, each with its own step count."""
    rng = np.random.default_rng(21)
    s, cfg, params, buffers = make("yolo11s", 1, optimizer=sy.SY_OPT_ADAMW)
    p, m1, m2, steps, b = params.copy(), np.zeros_like(params), np.zeros_like(params), [0, 0, 0], buffers.copy()
    for it, nboxes in enumerate([(1, 6), (0, 0)]):
        s.set_epoch(it)
        feats = features(cfg, 2, rng)
        _, truth = data.synthetic_batch(rng, 2, cfg.image_size, cfg.num_classes, boxes=nboxes, wh=(8.0, 64.0))
        if nboxes == (0, 0):
            truth = [[], []]
        stats = s.step_features(feats, truth)
        # the oracle optimizer runs on this step's GPU gradient from the same starting state, so the
        # comparison isolates AdamW (it divides noise-level gradients by their own magnitude)
        _, ograd, _, b, _, _, _ = oracle_head_step_adamw(cfg, s.tensors, p, b, m1, m2, steps, feats, truth, it)
        g = s.last_gradients()
        assert rel_l2(g, ograd) < TOL
        connected = stats.box_has_grad
        assert connected == (3 if it == 0 else 0)
        off = 0
        for t in s.params:
            n = t["numel"]
            group = sy.tensor_group(t["name"])
            has = group == 0 or bool(connected >> (group - 1) & 1)
            decay = t["name"].endswith("conv.weight") or (t["name"].endswith(".weight") and len(t["shape"]) == 4)
            w, a, bb, gg = p[off:off + n].copy(), m1[off:off + n].copy(), m2[off:off + n].copy(), g[off:off + n].copy()
            assert O.lib().syo_adamw_update(w, a, bb, gg, n, cfg.lr, cfg.beta1, cfg.beta2, cfg.adam_eps,
                                            cfg.weight_decay if decay else 0.0, steps[group] + 1, 2, int(has)) == 0
            p[off:off + n], m1[off:off + n], m2[off:off + n] = w, a, bb
            off += n
        for gi in range(3):
            steps[gi] += int(gi == 0 or bool(connected >> (gi - 1) & 1))
        assert rel_l2(s.flat_params(), p) < 1e-5
        assert rel_l2(s.flat_velocity(0), m1) < 1e-5
        assert rel_l2(s.flat_velocity(1), m2) < 1e-5
    assert steps == [2, 1, 1]


def test_end_to_end_eval_loss_uses_epoch_zero():
    rng = np.random.default_rng(12)
    s, cfg, params, buffers = make("yolo11s", 1, schedule=4)
    s.set_epoch(3)   # evaluation ignores the training epoch (YoloTrainer.cs:243)
    feats = features(cfg, 2, rng)
    _, truth = data.synthetic_batch(rng, 2, cfg.image_size, cfg.num_classes, boxes=(1, 5), wh=(8.0, 64.0))
    stats = s.eval_loss_features(feats, truth)
    d = head_desc(cfg, 0)
    want = dict(box=0.0, cls=0.0, dfl=0.0, positives=0)
    for b in range(2):
        fs = [np.ascontiguousarray(f[b]) for f in feats]
        fp = (C.c_void_p * 3)(*[f.ctypes.data_as(C.c_void_p) for f in fs])
        out = O.Loss()
        assert O.lib().syo_head_eval_image(C.byref(d), params, buffers.copy(), fp, O.boxes(truth[b]), len(truth[b]),
                                           C.byref(out)) == 0
        for k in ("box", "cls", "dfl", "positives"):
            want[k] += getattr(out, k)
    assert stats.positives == want["positives"]
    for k in ("box", "cls", "dfl"):
        assert abs(getattr(stats, k) - want[k]) <= TOL * max(abs(want[k]), 1.0), k
    assert s.flat_params().tobytes() == params.tobytes()
