"""The head's pyramid levels run on separate streams (forward: from the trunk op that finishes each
level's feature map to the loss; backward: from the loss to the parameter-gradient fold), each with its
own scratch.  Nothing else changes, so a session on those streams (and in a CUDA graph) must give results
bit-identical to the same session run serially on one stream (conv-launch profiling switches the level
streams and the graphs off).  A buffer shared by two levels shows up here as a difference."""
import numpy as np
import pytest
import torch

import simdyolo_b200 as sy
from simdyolo_b200 import data

pytestmark = pytest.mark.gpu


def run(model, image_size, batch, serial, backbone=True, end_to_end=False, reg_max=16, steps=4):
    cfg = sy.make_config(model, image_size=image_size, max_batch=batch, max_boxes=12, backbone=backbone,
                         end_to_end=end_to_end, reg_max=reg_max)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, 7)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    if backbone:
        s.set_backbone(data.backbone_params(model, 3))
    if serial:
        s.conv_profile(True)
    rng = np.random.default_rng(17)
    imgs, truth = data.synthetic_batch(rng, batch, image_size, 80, (1, 12), (8.0, image_size / 2))
    feats = [(rng.standard_normal((batch, cfg.feature_channels[l], image_size >> (3 + l), image_size >> (3 + l)))
              * 0.7).astype(np.float32) for l in range(3)]
    dev = torch.from_numpy(imgs).cuda()
    out = []
    for _ in range(steps):
        st = s.step_device(dev.data_ptr(), batch, truth) if backbone else s.step_features(feats, truth)
        out.append((st.box, st.cls, st.dfl, st.positives))
        out.append(s.last_gradients().tobytes())
    out += [s.flat_params().tobytes(), s.flat_buffers().tobytes(), s.flat_velocity().tobytes()]
    return out


@pytest.mark.parametrize("model,image_size,batch,backbone,end_to_end,reg_max", [
    ("yolov8n", 320, 8, True, False, 16),
    ("yolo11s", 256, 4, True, False, 16),
    ("yolo11s", 128, 2, True, False, 16),
    ("yolov8n", 256, 4, False, True, 1),
])
def test_level_streams_match_one_stream_bitwise(model, image_size, batch, backbone, end_to_end, reg_max):
    laned = run(model, image_size, batch, False, backbone, end_to_end, reg_max)
    serial = run(model, image_size, batch, True, backbone, end_to_end, reg_max)
    assert len(laned) == len(serial)
    for i, (a, b) in enumerate(zip(laned, serial)):
        assert a == b, f"item {i} differs"
