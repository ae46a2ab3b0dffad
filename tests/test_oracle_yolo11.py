"""The oracle's YOLO11 trunk (C restatement of PtModel.cs C3k2 / C3k / Bottleneck / SPPF / C2PSA /
PSABlock / Attention, :299-342, :429-439) against an independent torch restatement of the same layer
graph that consumes the same flat, BN-folded parameters in the same order."""
import ctypes as C

import numpy as np
import torch
import torch.nn.functional as F

import simdyolo_b200 as sy
from simdyolo_b200 import data
from oracle import oracle as O
from tests.helpers import backbone_desc, rel_l2


class Params:
    def __init__(self, flat):
        self.flat, self.off = torch.from_numpy(flat), 0

    def take(self, shape):
        n = int(np.prod(shape))
        t = self.flat[self.off:self.off + n].reshape(shape)
        self.off += n
        return t


def conv(p, x, oc, k, s=1, act=True, groups=1):
    ic = x.shape[1]
    w = p.take((oc, ic // groups, k, k))
    b = p.take((oc,))
    y = F.conv2d(x, w, b, stride=s, padding=k // 2, groups=groups)
    return F.silu(y) if act else y


def bottleneck(p, x, c2, e, shortcut=True):
    y = conv(p, conv(p, x, int(c2 * e), 3), c2, 3)
    return x + y if shortcut and x.shape[1] == c2 else y


def c3k(p, x, c2, n):
    c_ = int(c2 * 0.5)
    a = conv(p, x, c_, 1)
    for _ in range(n):
        a = bottleneck(p, a, c_, 1.0)
    b = conv(p, x, c_, 1)
    return conv(p, torch.cat([a, b], 1), c2, 1)


def c3k2(p, x, c2, n, use_c3k, e):
    c = int(c2 * e)
    ys = list(conv(p, x, 2 * c, 1).split(c, 1))
    for _ in range(n):
        ys.append(c3k(p, ys[-1], c, 2) if use_c3k else bottleneck(p, ys[-1], c, 0.5))
    return conv(p, torch.cat(ys, 1), c2, 1)


def attention(p, x, heads):
    b, c, h, w = x.shape
    hd, n = c // heads, h * w
    kd = int(hd * 0.5)
    qkv = conv(p, x, c + 2 * kd * heads, 1, act=False).view(b, heads, 2 * kd + hd, n)
    q, k, v = qkv.split([kd, kd, hd], 2)
    attn = ((q.transpose(-2, -1) @ k) * kd ** -0.5).softmax(-1)
    out = (v @ attn.transpose(-2, -1)).view(b, c, h, w) + conv(p, v.reshape(b, c, h, w), c, 3, act=False, groups=c)
    return conv(p, out, c, 1, act=False)


def c2psa(p, x, n):
    c1 = x.shape[1]
    c = int(c1 * 0.5)
    a, b = conv(p, x, 2 * c, 1).split(c, 1)
    for _ in range(n):
        b = b + attention(p, b, max(c // 64, 1))
        b = b + conv(p, conv(p, b, 2 * c, 1), c, 1, act=False)
    return conv(p, torch.cat([a, b], 1), c1, 1)


def sppf(p, x, c2):
    y = [conv(p, x, x.shape[1] // 2, 1)]
    for _ in range(3):
        y.append(F.max_pool2d(y[-1], 5, 1, 2))
    return conv(p, torch.cat(y, 1), c2, 1)


def trunk(p, img, ch, n2):
    up = lambda t: F.interpolate(t, scale_factor=2, mode="nearest")
    x = conv(p, img, ch(64), 3, 2)
    x = conv(p, x, ch(128), 3, 2)
    x = c3k2(p, x, ch(256), n2, False, 0.25)
    x = conv(p, x, ch(256), 3, 2)
    l4 = c3k2(p, x, ch(512), n2, False, 0.25)
    x = conv(p, l4, ch(512), 3, 2)
    l6 = c3k2(p, x, ch(512), n2, True, 0.5)
    x = conv(p, l6, ch(1024), 3, 2)
    x = c3k2(p, x, ch(1024), n2, True, 0.5)
    x = sppf(p, x, ch(1024))
    l10 = c2psa(p, x, n2)
    l13 = c3k2(p, torch.cat([up(l10), l6], 1), ch(512), n2, False, 0.5)
    p3 = c3k2(p, torch.cat([up(l13), l4], 1), ch(256), n2, False, 0.5)
    p4 = c3k2(p, torch.cat([conv(p, p3, ch(256), 3, 2), l13], 1), ch(512), n2, False, 0.5)
    p5 = c3k2(p, torch.cat([conv(p, p4, ch(512), 3, 2), l10], 1), ch(1024), n2, True, 0.5)
    return p3, p4, p5


def test_yolo11s_trunk_matches_torch_restatement():
    size = 128
    cfg = sy.make_config("yolo11s", image_size=size, max_batch=1)
    width, depth, max_ch = sy.MODELS["yolo11s"]
    params = data.backbone_params("yolo11s", seed=2)
    bd = backbone_desc(cfg)
    assert O.lib().syo_backbone_param_count(C.byref(bd)) == params.size
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, (size, size, 3), dtype=np.uint8)
    feats = [np.zeros((cfg.feature_channels[l], size >> (3 + l), size >> (3 + l)), np.float32) for l in range(3)]
    O.lib().syo_backbone_forward(C.byref(bd), params, img.ctypes.data_as(C.POINTER(C.c_uint8)), *feats)
    ch = lambda c: sy._make_div8(np.float32(min(c, max_ch)) * np.float32(width))
    p = Params(params)
    with torch.no_grad():
        x = torch.from_numpy(img).permute(2, 0, 1)[None].float() / 255.0
        ref = trunk(p, x, ch, max(int(np.floor(2 * depth + 0.5)), 1))
    assert p.off == params.size
    for l in range(3):
        assert rel_l2(feats[l], ref[l][0].numpy()) < 1e-5, f"level {l}"
