"""Configuration 0 of the benchmark contract, run on the GPU and on the CPU oracle side by side.

YOLOv8n (depth 0.33, width 0.25, 80 classes, reg_max 16), head fine-tune with the backbone+neck frozen,
random-init weights from seed 0, a batch of 8 synthetic 640x640 RGB24 images (bytes uniform in [0, 255],
1-8 boxes per image, class uniform in [0, 80), centre uniform, w/h log-uniform in [8, 320] px, clipped),
16 SGD steps (lr 0.01, momentum 0.937, weight decay 5e-4) over that batch.  Every step logs the loss parts,
the positives and the head-gradient checksum; both sides run the whole step from their own state (frozen
trunk on the RGB bytes, head forward with training BatchNorm, DetectionLoss, backward, update), exactly the
loop of YoloTrainer.Train (src/SimdYolo.Training/YoloTrainer.cs:185-199).  The oracle is the C restatement
of the reference's CPU trainer (oracle/step.c, syo_train_step).

Bounds.  The positives (the assigner's decisions) must match exactly in both precisions.

3xTF32 parity mode: loss parts within 1e-5 relative; the class loss is the reference's own float running
sum (DetectionLoss.cs:103-109), reproduced term by term.  Gradients, parameter updates, velocities and
BatchNorm buffers within 2e-5 relative L2.  That is twice the oracle's own distance from the exact gradient:
the first conv of every branch sums trunk features with a large per-channel mean against a zero-sum
BatchNorm gradient, so any FP32 evaluation order rounds by about 1e-5 there.
test_config0_head_gradients_against_float64 measures that distance from a float64 evaluation, and requires
the GPU to be within 1e-5 of the float64 result.

TF32 mode: loss parts within 2e-3 (the class loss is the exact sum of the terms, which differs from the
reference's float running sum by about 1.3e-3 at this size).  Every step's gradient is also checked against
the oracle's head run from the GPU's own state (its frozen features and its parameters before the step):
within 2.5e-3 (1.6-2.0e-3 measured, the TF32 operands' own error; test_config0_head_gradients_against_float64
evaluates the head in float64 with every conv operand rounded to TF32 as the tensor-core path stores it and
requires the GPU to sit within 10 % of that figure).  Against the oracle's independent trajectory the TF32
gradients agree to about 3.5e-3 on most steps, but on a few steps (2.5e-2 at most measured) a positive's
predicted box edge lies within TF32 noise of its ground-truth edge, where the reference's CIoU gradient
switches branch (the max / min of the enclosing and intersection boxes, DetectionLoss.cs:171-183): that step's
level gradient then differs by a few percent on one branch.  So the trajectory is held to a median of 4e-3
per step and 6e-3 on the final parameter update, velocity and BatchNorm buffers.
"""
import ctypes as C

import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from oracle import oracle as O
from tests.helpers import (backbone_desc, f64_head_gradient, head_desc, head_gradient_emulated, initial_head_state,
                           oracle_head_step, rel_l2)

pytestmark = pytest.mark.gpu

IMAGE, BATCH, STEPS, SEED = 640, 8, 16, 0
BOUNDS = {sy.SY_PRECISION_3XTF32: dict(loss=1e-5, cls=1e-5, features=1e-5, grad_state=2e-5, grad=2e-5, grad_median=2e-5,
                                       state=2e-5),
          sy.SY_PRECISION_TF32: dict(loss=2e-3, cls=2e-3, features=2e-3, grad_state=2.5e-3, grad=None, grad_median=4e-3,
                                     state=6e-3)}


def config0(precision, backbone=True):
    return sy.make_config("yolov8n", image_size=IMAGE, max_batch=BATCH, max_boxes=8, num_classes=80,
                          lr=0.01, momentum=0.937, weight_decay=5e-4, precision=precision, backbone=backbone)


def workload():
    rng = np.random.default_rng(SEED)
    images, truth = data.synthetic_batch(rng, BATCH, IMAGE, 80, boxes=(1, 8), wh=(8.0, 320.0))
    return images, truth


def initial_state(cfg):
    tensors, params, buffers = initial_head_state(cfg, SEED)
    return tensors, params, buffers, data.backbone_params("yolov8n", seed=SEED)


def oracle_trajectory():
    """The oracle's 16 steps: per step (box, cls, dfl, positives, summed gradient), final state."""
    cfg = config0(sy.SY_PRECISION_TF32)
    tensors, params, buffers, bparams = initial_state(cfg)
    images, truth = workload()
    bd, hd = backbone_desc(cfg), head_desc(cfg)
    p, b = params.copy(), buffers.copy()
    v, v2 = np.zeros_like(p), np.zeros_like(p)
    opt = O.Optim(cfg.lr, cfg.momentum, cfg.weight_decay, 0, cfg.beta1, cfg.beta2, cfg.adam_eps)
    flat = [bx for t in truth for bx in t]
    tb = O.boxes(flat)
    counts = np.array([len(t) for t in truth], np.int32)
    ptrs = (C.c_void_p * BATCH)(*[images[i].ctypes.data_as(C.c_void_p) for i in range(BATCH)])
    steps = []
    for _ in range(STEPS):
        grad = np.zeros_like(p)
        res = O.StepResult()
        O.lib().syo_train_step(C.byref(bd), bparams, C.byref(hd), p, b, v, v2, C.byref(opt), ptrs, tb, counts,
                               BATCH, 0, grad.ctypes.data_as(C.c_void_p), C.byref(res))
        assert res.status == 0
        steps.append(dict(box=res.box, cls=res.cls, dfl=res.dfl, positives=res.positives,
                          connected=res.box_has_grad, grad=grad))
    return dict(steps=steps, params=p, buffers=b, velocity=v, start=params, features=oracle_features(cfg, bparams, images))


def oracle_features(cfg, bparams, images):
    bd = backbone_desc(cfg)
    feats = [np.zeros((BATCH, cfg.feature_channels[l], IMAGE >> (3 + l), IMAGE >> (3 + l)), np.float32)
             for l in range(3)]
    for b in range(BATCH):
        f = [np.zeros(feats[l].shape[1:], np.float32) for l in range(3)]
        O.lib().syo_backbone_forward(C.byref(bd), bparams, images[b].ctypes.data_as(C.POINTER(C.c_uint8)), *f)
        for l in range(3):
            feats[l][b] = f[l]
    return feats


@pytest.fixture(scope="module")
def oracle_run():
    return oracle_trajectory()


@pytest.mark.parametrize("precision", [sy.SY_PRECISION_3XTF32, sy.SY_PRECISION_TF32], ids=["3xtf32", "tf32"])
def test_config0_sixteen_steps_match_oracle(oracle_run, precision):
    bound = BOUNDS[precision]
    cfg = config0(precision)
    tensors, params, buffers, bparams = initial_state(cfg)
    images, truth = workload()
    shapes = [(BATCH, cfg.feature_channels[l], IMAGE >> (3 + l), IMAGE >> (3 + l)) for l in range(3)]
    traj = []
    with sy.Session(cfg) as s:
        assert [(t["name"], t["shape"]) for t in s.tensors] == [(t["name"], t["shape"]) for t in tensors]
        s.set_flat_params(params)
        s.set_flat_buffers(buffers)
        s.set_backbone(bparams)
        for k, ref in enumerate(oracle_run["steps"]):
            p_before, b_before = s.flat_params(), s.flat_buffers()
            st = s.step(images, truth)
            g = s.last_gradients()
            feats = [s.last_features(l, shapes[l]) for l in range(3)]
            if k == 0:
                ferr = max(rel_l2(feats[l], oracle_run["features"][l]) for l in range(3))
                print(f"trunk features vs oracle: {ferr:.2e}")
                assert ferr <= bound["features"]
            # the oracle's head step from the GPU's own state (same features, same parameters)
            _, og, *_ = oracle_head_step(cfg, tensors, p_before, b_before, np.zeros_like(p_before), feats, truth)
            errs = dict(box=abs(st.box - ref["box"]) / max(abs(ref["box"]), 1e-6),
                        dfl=abs(st.dfl - ref["dfl"]) / max(abs(ref["dfl"]), 1e-6),
                        cls=abs(st.cls - ref["cls"]) / abs(ref["cls"]),
                        grad=rel_l2(g, ref["grad"]), grad_state=rel_l2(g, og))
            # checksum: sum |g| of the batch-averaged gradient, as sy_step_stats reports it
            want_sum = float(np.abs(ref["grad"].astype(np.float64)).sum()) / BATCH
            errs["checksum"] = abs(st.grad_checksum - want_sum) / want_sum
            print(f"step {k:2d}: box {st.box:.6f} cls {st.cls:.6f} dfl {st.dfl:.6f} pos {st.positives} | "
                  f"rel box {errs['box']:.2e} cls {errs['cls']:.2e} dfl {errs['dfl']:.2e} | gradient vs oracle "
                  f"at the GPU's state {errs['grad_state']:.2e}, vs the oracle's trajectory {errs['grad']:.2e} "
                  f"(checksum {errs['checksum']:.2e}); assigner near ties {st.near_ties}")
            assert st.positives == ref["positives"], (k, st.positives, ref["positives"])
            assert st.box_has_grad == ref["connected"]
            assert errs["box"] <= bound["loss"] and errs["dfl"] <= bound["loss"], (k, errs)
            assert errs["cls"] <= bound["cls"], (k, errs)
            assert errs["grad_state"] <= bound["grad_state"], (k, errs)
            if bound["grad"] is not None:
                assert errs["grad"] <= bound["grad"], (k, errs)
                assert errs["checksum"] <= bound["grad"], (k, errs)
            traj.append(errs["grad"])
        start = oracle_run["start"]
        state = dict(update=rel_l2(s.flat_params() - start, oracle_run["params"] - start),
                     velocity=rel_l2(s.flat_velocity(), oracle_run["velocity"]),
                     buffers=rel_l2(s.flat_buffers(), oracle_run["buffers"]))
    print(f"precision {precision}: trajectory gradient median {np.median(traj):.2e} max {max(traj):.2e}; "
          f"after {STEPS} steps {state}")
    assert np.median(traj) <= bound["grad_median"]
    for key, err in state.items():
        assert err <= bound["state"], (key, err)


def test_config0_head_gradients_against_float64():
    """Step 0 of configuration 0, head only, on the oracle's own frozen features: the GPU in both
    precisions, the oracle, and the head evaluated in float64 (exact up to 1e-15) and in float64 with
    TF32-rounded conv operands (the TF32 format's own error for this workload)."""
    cfg = config0(sy.SY_PRECISION_TF32)
    tensors, params, buffers, bparams = initial_state(cfg)
    images, truth = workload()
    feats = oracle_features(cfg, bparams, images)
    exact, positives = f64_head_gradient(cfg, tensors, params, feats, truth)
    _, ograd, *_ = oracle_head_step(cfg, tensors, params, buffers, np.zeros_like(params), feats, truth)
    tf32_floor = rel_l2(head_gradient_emulated(cfg, tensors, params, feats, truth, tf32=True,
                                               center_first=False)[0], exact)
    oracle_err = rel_l2(ograd, exact)
    got = {}
    for precision in (sy.SY_PRECISION_3XTF32, sy.SY_PRECISION_TF32):
        with sy.Session(config0(precision, backbone=False)) as s:
            s.set_flat_params(params)
            s.set_flat_buffers(buffers)
            st = s.step_features(feats, truth)
            assert st.positives == positives
            got[precision] = rel_l2(s.last_gradients(), exact)
    print(f"distance from the float64 head gradient: oracle (FP32) {oracle_err:.2e}, GPU 3xTF32 "
          f"{got[sy.SY_PRECISION_3XTF32]:.2e}, GPU TF32 {got[sy.SY_PRECISION_TF32]:.2e}, "
          f"TF32 operands emulated in float64 {tf32_floor:.2e}")
    assert oracle_err <= 2e-5
    assert got[sy.SY_PRECISION_3XTF32] <= 1e-5
    assert got[sy.SY_PRECISION_TF32] <= 1.1 * tf32_floor
    # the contract's TF32 figure of 2e-3 lies below the format's own error on this workload
    assert tf32_floor > 2e-3
