"""Head convs with general group counts (groups dividing both channel counts, HeadOperations.cs:88-133)
through the session against the oracle's grouped convolution: the GPU runs them on the tensor-core conv
with block-diagonal dense weights and keeps the diagonal blocks of the dense weight gradient.  TF32 at the
step tests' 2e-3; 3xTF32 at 1e-5 (class loss 1e-4, as the other 3xTF32 tests)."""
import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from tests.helpers import oracle_head_step, rel_l2

pytestmark = pytest.mark.gpu


def grouped_session(precision, image_size=128, batch=2):
    cfg = sy.make_config("yolov8n", image_size=image_size, max_batch=batch, max_boxes=8, backbone=False,
                         precision=precision)
    for l in range(3):
        cfg.box_blocks[l][1].groups = 4   # 3x3 64 -> 64 in four groups
        cfg.cls_blocks[l][0].groups = 2   # 3x3 C_l -> 80 in two groups (reads the features)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 11)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    return s, cfg, params, buffers


# update_tol: the first SGD step's update is lr (g / N + wd w); where the two terms nearly cancel, the same
# gradient difference is a larger relative difference of the update (3xTF32: gradients 1e-5, update 2e-5)
@pytest.mark.parametrize("precision,tol,cls_tol,update_tol", [(sy.SY_PRECISION_TF32, 2e-3, 2e-3, 2e-3),
                                                              (sy.SY_PRECISION_3XTF32, 1e-5, 1e-4, 2e-5)])
def test_grouped_head_step_matches_oracle(precision, tol, cls_tol, update_tol):
    rng = np.random.default_rng(23)
    s, cfg, params, buffers = grouped_session(precision)
    shapes = {t["name"]: tuple(t["shape"]) for t in s.params}
    assert shapes["cv2.0.1.conv.weight"] == (64, 16, 3, 3)
    assert shapes["cv3.2.0.conv.weight"] == (80, cfg.feature_channels[2] // 2, 3, 3)
    feats = [(rng.standard_normal((2, cfg.feature_channels[l], 128 >> (3 + l), 128 >> (3 + l))) * 0.7 + 0.2)
             .astype(np.float32) for l in range(3)]
    _, truth = data.synthetic_batch(rng, 2, 128, cfg.num_classes, boxes=(1, 6), wh=(8.0, 64.0))
    stats = s.step_features(feats, truth)
    losses, ograd, oparams, obuffers, ovel, conn = oracle_head_step(cfg, s.tensors, params, buffers,
                                                                    np.zeros_like(params), feats, truth)
    ocls = sum(l["cls"] for l in losses)
    obox = sum(l["box"] for l in losses)
    assert abs(stats.cls - ocls) <= cls_tol * abs(ocls)
    assert abs(stats.box - obox) <= tol * max(abs(obox), 1.0)
    assert stats.positives == sum(l["positives"] for l in losses)
    assert rel_l2(s.last_gradients(), ograd) < tol
    assert rel_l2(s.flat_params() - params, oparams - params) < update_tol
    assert rel_l2(s.flat_buffers(), obuffers) < tol


def test_group_count_must_divide_the_channels():
    cfg = sy.make_config("yolov8n", image_size=128, max_batch=2, backbone=False)
    cfg.box_blocks[0][1].groups = 3   # 64 channels
    with pytest.raises(sy.UnsupportedShape):
        sy.Session(cfg)
