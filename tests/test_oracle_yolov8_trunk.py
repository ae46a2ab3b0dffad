"""The oracle's YOLOv8 trunk (oracle/step.c: the C restatement of PtModel.cs Conv / C2f / Bottleneck / SPPF /
Upsample / Concat, :267-342, with BatchNorm folded as PtModel.cs:128-144 does) against a torch restatement of
the public YOLOv8 detection model definition written from that definition alone: the backbone
(Conv 64/3/2, Conv 128/3/2, C2f 128 x3 shortcut, Conv 256/3/2, C2f 256 x6, Conv 512/3/2, C2f 512 x6,
Conv 1024/3/2, C2f 1024 x3, SPPF 1024/5) and the neck (Upsample, Concat with layer 6, C2f 512 x3, Upsample,
Concat with layer 4, C2f 256 x3 -> P3, Conv 256/3/2, Concat with layer 12, C2f 512 x3 -> P4, Conv 512/3/2,
Concat with layer 9, C2f 1024 x3 -> P5), channels make_divisible(min(c, max) * width, 8), repeats
max(round(n * depth), 1).  Both consume the same flat folded parameters in the order the C ABI documents
(every conv in call order, OIHW weight then bias; C2f = cv1, bottlenecks, cv2; SPPF = cv1, cv2).  The torch
side runs in float64, so the comparison bounds the oracle's float32 rounding."""
import ctypes as C
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import simdyolo_b200 as sy
from simdyolo_b200 import data
from oracle import oracle as O
from tests.helpers import backbone_desc, rel_l2


class Params:
    def __init__(self, flat):
        self.flat, self.off = torch.from_numpy(flat.astype(np.float64)), 0

    def take(self, shape):
        n = int(np.prod(shape))
        t = self.flat[self.off:self.off + n].reshape(shape)
        self.off += n
        return t


def conv(p, x, c2, k, s=1):
    """Conv: conv2d (BatchNorm folded into weight and bias) + SiLU."""
    w = p.take((c2, x.shape[1], k, k))
    b = p.take((c2,))
    return F.silu(F.conv2d(x, w, b, stride=s, padding=k // 2))


def c2f(p, x, c2, n, shortcut):
    c = int(c2 * 0.5)
    y = list(conv(p, x, 2 * c, 1).chunk(2, 1))
    for _ in range(n):
        t = conv(p, conv(p, y[-1], c, 3), c, 3)       # Bottleneck(c, c, shortcut, k=(3, 3), e=1.0)
        y.append(y[-1] + t if shortcut else t)
    return conv(p, torch.cat(y, 1), c2, 1)


def sppf(p, x, c2, k=5):
    x = conv(p, x, x.shape[1] // 2, 1)
    y = [x]
    for _ in range(3):
        y.append(F.max_pool2d(y[-1], k, 1, k // 2))
    return conv(p, torch.cat(y, 1), c2, 1)


def yolov8_trunk(flat, rgb, width, depth, max_channels):
    ch = lambda c: math.ceil(min(c, max_channels) * width / 8) * 8
    rep = lambda n: max(round(n * depth), 1)
    p = Params(flat)
    up = lambda t: F.interpolate(t, scale_factor=2, mode="nearest")
    x = torch.from_numpy(rgb.astype(np.float64) / 255.0).permute(2, 0, 1)[None]
    x = conv(p, x, ch(64), 3, 2)
    x = conv(p, x, ch(128), 3, 2)
    x = c2f(p, x, ch(128), rep(3), True)
    x = conv(p, x, ch(256), 3, 2)
    l4 = c2f(p, x, ch(256), rep(6), True)
    x = conv(p, l4, ch(512), 3, 2)
    l6 = c2f(p, x, ch(512), rep(6), True)
    x = conv(p, l6, ch(1024), 3, 2)
    x = c2f(p, x, ch(1024), rep(3), True)
    l9 = sppf(p, x, ch(1024))
    l12 = c2f(p, torch.cat([up(l9), l6], 1), ch(512), rep(3), False)
    p3 = c2f(p, torch.cat([up(l12), l4], 1), ch(256), rep(3), False)
    p4 = c2f(p, torch.cat([conv(p, p3, ch(256), 3, 2), l12], 1), ch(512), rep(3), False)
    p5 = c2f(p, torch.cat([conv(p, p4, ch(512), 3, 2), l9], 1), ch(1024), rep(3), False)
    assert p.off == p.flat.numel(), "parameter count"
    return [t[0].numpy() for t in (p3, p4, p5)]


@pytest.mark.parametrize("model,size", [("yolov8n", 96), ("yolov8l", 64)])
def test_oracle_yolov8_trunk_matches_torch_restatement(model, size):
    width, depth, max_ch = sy.MODELS[model]
    cfg = sy.make_config(model, image_size=size, max_batch=1)
    bparams = data.backbone_params(model, seed=3)
    bd = backbone_desc(cfg)
    assert O.lib().syo_backbone_param_count(C.byref(bd)) == bparams.size
    rng = np.random.default_rng(4)
    rgb = rng.integers(0, 256, size=(size, size, 3), dtype=np.uint8)
    feats = [np.zeros((cfg.feature_channels[l], size >> (3 + l), size >> (3 + l)), np.float32) for l in range(3)]
    O.lib().syo_backbone_forward(C.byref(bd), bparams, rgb.ctypes.data_as(C.POINTER(C.c_uint8)), *feats)
    want = yolov8_trunk(bparams, rgb, width, depth, max_ch)
    for l in range(3):
        assert feats[l].shape == want[l].shape
        assert rel_l2(feats[l], want[l]) < 2e-6, (model, l, rel_l2(feats[l], want[l]))
