"""Config 3 pieces on the GPU: the YOLO11 Detect head (class branch with depthwise 3x3 convs,
HeadOperations.GroupedConv HeadOperations.cs:88-133, flattened to five blocks) and the AdamW
optimizer, against the CPU oracle on identical seeded features, within the TF32 bound of 2e-3."""
import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from tests.helpers import oracle_head_step, rel_l2

pytestmark = pytest.mark.gpu
TOL = 2e-3


def session(image_size, batch, optimizer=sy.SY_OPT_SGD, **kw):
    cfg = sy.make_config("yolo11s", image_size=image_size, max_batch=batch, max_boxes=20, backbone=False,
                         optimizer=optimizer, **kw)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 2)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    return s, cfg, params, buffers


def features(cfg, batch, rng):
    out = []
    for l in range(3):
        h = cfg.image_size >> (3 + l)
        out.append((rng.standard_normal((batch, cfg.feature_channels[l], h, h)) * 0.7 + 0.2).astype(np.float32))
    return out


def test_yolo11s_head_tensors_follow_the_snapshot_layout():
    s, cfg, params, _ = session(128, 1)
    names = [t["name"] for t in s.params if t["name"].startswith("cv3.0.")]
    assert names == ["cv3.0.0.0.conv.weight", "cv3.0.0.0.bn.weight", "cv3.0.0.0.bn.bias",
                     "cv3.0.0.1.conv.weight", "cv3.0.0.1.bn.weight", "cv3.0.0.1.bn.bias",
                     "cv3.0.1.0.conv.weight", "cv3.0.1.0.bn.weight", "cv3.0.1.0.bn.bias",
                     "cv3.0.1.1.conv.weight", "cv3.0.1.1.bn.weight", "cv3.0.1.1.bn.bias",
                     "cv3.0.2.weight", "cv3.0.2.bias"]
    dw = next(t for t in s.params if t["name"] == "cv3.0.0.0.conv.weight")
    assert dw["shape"] == (128, 1, 3, 3)


@pytest.mark.parametrize("image_size,batch", [(128, 2), (256, 2)])
def test_yolo11s_head_step_matches_oracle(image_size, batch):
    rng = np.random.default_rng(31)
    s, cfg, params, buffers = session(image_size, batch)
    feats = features(cfg, batch, rng)
    _, truth = data.synthetic_batch(rng, batch, image_size, cfg.num_classes, boxes=(1, 20), wh=(8.0, image_size / 2))
    stats = s.step_features(feats, truth)
    losses, ograd, oparams, obuffers, ovel, conn = oracle_head_step(cfg, s.tensors, params, buffers,
                                                                    np.zeros_like(params), feats, truth)
    ocls = sum(l["cls"] for l in losses)
    assert abs(stats.cls - ocls) <= TOL * abs(ocls)
    assert stats.positives == sum(l["positives"] for l in losses)
    assert rel_l2(s.last_gradients(), ograd) < TOL
    assert rel_l2(s.flat_params() - params, oparams - params) < TOL
    assert rel_l2(s.flat_buffers(), obuffers) < TOL


def test_adamw_steps_match_oracle():
    """Config-3 optimizer: AdamW lr 1e-3, weight decay 0.05 over three steps, one of them without boxes
    (the box group then keeps its parameters, moments and step count).  AdamW divides every update by
    the root of its second moment, so a parameter whose true gradient is almost zero moves by +-lr in
    the direction of its TF32 rounding noise; the update is therefore checked on the GPU's own
    gradients (the oracle's AdamW applied to them), and the gradients against the oracle's."""
    from oracle import oracle as O
    rng = np.random.default_rng(41)
    s, cfg, params, buffers = session(128, 2, optimizer=sy.SY_OPT_ADAMW, lr=1e-3, weight_decay=0.05)
    p, m1, m2, steps = params.copy(), np.zeros_like(params), np.zeros_like(params), [0, 0]
    for k in range(3):
        feats = features(cfg, 2, rng)
        truth = [[], []] if k == 1 else data.synthetic_batch(rng, 2, 128, cfg.num_classes, boxes=(1, 20),
                                                             wh=(8.0, 64.0))[1]
        stats = s.step_features(feats, truth)
        grad = s.last_gradients()
        _, ograd, *_ = oracle_head_step(cfg, s.tensors, p, s.flat_buffers(), np.zeros_like(p), feats, truth)
        off = 0
        for t in s.params:
            n = t["numel"]
            box = t["name"].startswith("cv2")
            decay = t["name"].endswith("conv.weight") or (t["name"].endswith(".weight") and len(t["shape"]) == 4)
            w, a, b, g = p[off:off + n].copy(), m1[off:off + n].copy(), m2[off:off + n].copy(), grad[off:off + n].copy()
            has = stats.box_has_grad if box else 1
            assert O.lib().syo_adamw_update(w, a, b, g, n, cfg.lr, cfg.beta1, cfg.beta2, cfg.adam_eps,
                                            cfg.weight_decay if decay else 0.0, steps[1 if box else 0] + 1, 2,
                                            int(has)) == 0
            p[off:off + n], m1[off:off + n], m2[off:off + n] = w, a, b
            off += n
        steps[0] += 1
        steps[1] += int(stats.box_has_grad)
        assert rel_l2(s.flat_params() - params, p - params) < 1e-5
        assert rel_l2(s.flat_velocity(0), m1) < 1e-5
        assert rel_l2(s.flat_velocity(1), m2) < 1e-5
        assert rel_l2(grad, ograd) < TOL
        p = s.flat_params()   # next step from the GPU's parameters (the gradients are compared per step)
        m1, m2 = s.flat_velocity(0), s.flat_velocity(1)


def test_yolo11s_full_step_trunk_and_head_match_oracle():
    """The YOLO11s trunk (C3k2 / C3k / SPPF / C2PSA with attention) from RGB24 on the GPU, then the
    head step, against the oracle's trunk and head."""
    import ctypes as C

    from oracle import oracle as O
    from tests.helpers import backbone_desc
    image_size, batch = 128, 2
    rng = np.random.default_rng(51)
    cfg = sy.make_config("yolo11s", image_size=image_size, max_batch=batch, max_boxes=20)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 2)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    bparams = data.backbone_params("yolo11s", seed=2)
    bd = backbone_desc(cfg)
    assert s.backbone_param_count() == O.lib().syo_backbone_param_count(C.byref(bd)) == bparams.size
    s.set_backbone(bparams)
    images, truth = data.synthetic_batch(rng, batch, image_size, cfg.num_classes, boxes=(1, 20), wh=(8.0, 64.0))
    stats = s.step(images, truth)
    gpu_feats = []
    for l in range(3):
        h = image_size >> (3 + l)
        want = np.zeros((batch, cfg.feature_channels[l], h, h), np.float32)
        gpu_feats.append(s.last_features(l, want.shape))
    for b in range(batch):
        f = [np.zeros((cfg.feature_channels[l], image_size >> (3 + l), image_size >> (3 + l)), np.float32)
             for l in range(3)]
        O.lib().syo_backbone_forward(C.byref(bd), bparams, images[b].ctypes.data_as(C.POINTER(C.c_uint8)), *f)
        for l in range(3):
            # the trunk chains ~90 TF32 convolutions
            assert rel_l2(gpu_feats[l][b], f[l]) < 1.5 * TOL, f"image {b} level {l}"
    losses, ograd, oparams, obuffers, ovel, conn = oracle_head_step(cfg, s.tensors, params, buffers,
                                                                    np.zeros_like(params), gpu_feats, truth)
    ocls = sum(l["cls"] for l in losses)
    assert abs(stats.cls - ocls) <= TOL * abs(ocls)
    assert rel_l2(s.last_gradients(), ograd) < 2.5 * TOL
