"""Inputs and independent expectations for the inference post-processing tests.

The input generators restate the fixtures of the reference's own tests (paths inside the reference project):
  head_coordinate_case  tests/SimdYolo.Tests/CpuHeadCoordinatesTests.cs:15-20 and :43-47
  e2e_case              tests/SimdYolo.Tests/CpuPtEndToEndTests.cs:53-85
  mask_pipeline_case    tests/SimdYolo.Tests/MaskPipelineTests.cs:90-103
  nms_case              tests/SimdYolo.Tests/Program.cs:227-233
The expectations are written independently of the oracle: the coordinate formula of
CpuHeadCoordinatesTests, the full sorts of CpuPtEndToEndTests.Reference, and a scalar float32 restatement
of YoloDetector.DecodeIndexed (src/SimdYolo/YoloDetector.cs:539-652) in plain Python.
"""
from __future__ import annotations

import math
import struct

import numpy as np

f32 = np.float32


def bits_to_f32(u: int) -> np.float32:
    return np.frombuffer(struct.pack("<I", u & 0xffffffff), np.float32)[0]


def f32_bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------------- head decode

def head_coordinate_case(width: int, bins: int, batch: int = 2, height: int = 3, classes: int = 3):
    """CpuHeadCoordinatesTests.cs:17-20: box logits sin(a + side * .3 + b) * 4 (bins 1) or .2 (bins 16)."""
    spatial = width * height
    boxes = np.zeros((batch, 4 * bins, height, width), np.float32)
    flat = boxes.reshape(batch, 4, bins, spatial)
    for b in range(batch):
        for side in range(4):
            for r in range(bins):
                for a in range(spatial):
                    flat[b, side, r, a] = (f32(math.sin(f32(a + side * f32(.3) + b))) * f32(4)) if bins == 1 else f32(.2)
    scores = np.zeros((batch, classes, height, width), np.float32)
    return boxes, scores


def expected_coordinates(distance, width: int, spatial: int, stride, xyxy: bool):
    """The scalar expectation of CpuHeadCoordinatesTests.cs:25-28 for one image: [4][spatial] float32."""
    s = f32(stride)
    out = np.zeros((4, spatial), np.float32)
    with np.errstate(all="ignore"):
        for a in range(spatial):
            col, row = f32(a % width), f32(a // width)
            x1 = (col + f32(.5) - distance(0, a)) * s
            y1 = (row + f32(.5) - distance(1, a)) * s
            x2 = (col + f32(.5) + distance(2, a)) * s
            y2 = (row + f32(.5) + distance(3, a)) * s
            out[:, a] = [x1 if xyxy else (x1 + x2) * f32(.5), y1 if xyxy else (y1 + y2) * f32(.5),
                         x2 if xyxy else x2 - x1, y2 if xyxy else y2 - y1]
    return out


SPECIAL = [bits_to_f32(0x7fc12345), bits_to_f32(0xffc54321), f32(np.inf), f32(-np.inf), f32(0.0), f32(-0.0),
           f32(.1234567), f32(-2.345678)]


def special_case(width: int = 19, height: int = 2):
    """CpuHeadCoordinatesTests.cs:46-47: NaN payloads, infinities and signed zeros, bins 1, one class."""
    spatial = width * height
    data = np.array([SPECIAL[i % len(SPECIAL)] for i in range(4 * spatial)], np.float32)
    return data.reshape(1, 4, height, width), np.zeros((1, 1, height, width), np.float32)


# ---------------------------------------------------------------- end-to-end top-k

def e2e_case(batch: int, classes: int, anchors: int, frame: int) -> np.ndarray:
    """CpuPtEndToEndTests.Input (CpuPtEndToEndTests.cs:53-85)."""
    x = np.zeros((batch, classes + 4, anchors), np.float32)
    for b in range(batch):
        for c in range(4):
            for a in range(anchors):
                x[b, c, a] = b * 10000 + c * 1000 + a + frame * 100000
        for c in range(classes):
            for a in range(anchors):
                score = f32(((a * 7 + c * 3 + frame) % 17 - 8)) / f32(10)
                k = (a + c * 3 + frame) % 13
                score = {0: bits_to_f32(0x7fc00001 + a + c), 1: f32(np.inf), 2: f32(-np.inf), 3: f32(0.0),
                         4: bits_to_f32(0x80000000), 5: bits_to_f32(1), 6: bits_to_f32(0x80000001)}.get(k, score)
                if frame == 3:
                    score = f32(a % 7) * f32(.1) if c == 0 else f32(.25)
                x[b, c + 4, a] = score
    return x


def _net_max(a, b):
    """MathF.Max (and the IEEE 754:2019 Vector.Max of .NET 9+): NaN propagates, +0 above -0."""
    if a != a:
        return a
    if b != b:
        return b
    if a > b:
        return a
    if b > a:
        return b
    return b if math.copysign(1.0, float(a)) < 0 else a


def _desc_key(score):
    """Comparer<float>.Default in descending order: NaN below every number, -0 equal to +0."""
    return (1, 0.0) if score != score else (0, -float(score))


def e2e_expected(x: np.ndarray, maximum: int, classes: int) -> np.ndarray:
    """CpuPtEndToEndTests.Reference (CpuPtEndToEndTests.cs:93-121): two full sorts."""
    batch, _, anchors = x.shape
    count = min(maximum, anchors)
    out = np.zeros((batch, count, 6), np.float32)
    for b in range(batch):
        maxima = [f32(-np.inf)] * anchors
        for c in range(classes):
            for a in range(anchors):
                maxima[a] = _net_max(maxima[a], x[b, c + 4, a])
        chosen = sorted(range(anchors), key=lambda a: (_desc_key(maxima[a]), a))[:count]
        pairs = [(a, c, x[b, c + 4, a]) for a in chosen for c in range(classes)]
        pairs.sort(key=lambda p: (_desc_key(p[2]), p[0], p[1]))
        for i, (a, c, s) in enumerate(pairs[:count]):
            out[b, i, :4] = x[b, :4, a]
            out[b, i, 4] = s
            out[b, i, 5] = c
    return out


# ---------------------------------------------------------------- DecodeIndexed

def nms_case():
    """Program.cs:227-233: channels-last [3][6] raw output and a two-row end-to-end output."""
    raw = np.array([10, 10, 10, 10, .9, .1, 10, 10, 10, 10, .8, .1, 10, 10, 10, 10, .1, .95], np.float32).reshape(3, 6)
    end = np.array([1, 1, 10, 10, .9, 0, 1, 1, 10, 10, .8, 0], np.float32).reshape(2, 6)
    return raw, end


def mask_pipeline_case():
    """MaskPipelineTests.cs:90-103: the same rows channels-first [9][35] and channels-last [35][9]."""
    anchors, fields = 35, 9
    first = np.zeros((fields, anchors), np.float32)
    for a in range(anchors):
        first[:, a] = [a * 3 + 4, 5, 7, 3, np.nan if a % 5 == 0 else .5, .5,
                       np.inf if a % 7 == 0 else f32(.7) * f32(a % 2), 100, 100]
    return first, np.ascontiguousarray(first.T)


def _iou(a, b):
    """YoloDetector.Iou (YoloDetector.cs:648-652) on (x, y, w, h) float32 tuples."""
    w = _net_max(f32(0), _net_min(a[0] + a[2], b[0] + b[2]) - _net_max(a[0], b[0]))
    h = _net_max(f32(0), _net_min(a[1] + a[3], b[1] + b[3]) - _net_max(a[1], b[1]))
    inter = w * h
    return inter / _net_max(bits_to_f32(1), a[2] * a[3] + b[2] * b[3] - inter)


def _net_min(a, b):
    if a != a:
        return a
    if b != b:
        return b
    if a < b:
        return a
    if b < a:
        return b
    return a if math.copysign(1.0, float(a)) < 0 else b


def decode_expected(output: np.ndarray, layout: int, class_count: int = 0, letterbox=(1 << 20, 1 << 20, 1., 1., 0, 0),
                    confidence=.25, iou_threshold=.45, max_detections=300, max_candidates=30000, agnostic=False):
    """YoloDetector.DecodeIndexed restated in scalar float32 Python; letterbox = (source_w, source_h, scale_x,
    scale_y, pad_x, pad_y).  Returns [(class_id, confidence, x, y, w, h)]."""
    cf, e2e = layout == 1, layout == 3
    dim1, dim2 = output.shape
    count, fields = (dim2, dim1) if cf else (dim1, dim2)
    class_fields = 4 + class_count if class_count > 0 else fields
    at = (lambda a, c: output[c, a]) if cf else (lambda a, c: output[a, c])
    thr, iou_thr = f32(confidence), f32(iou_threshold)
    cand = []
    with np.errstate(all="ignore"):
        for a in range(count):
            cls = 0
            if e2e:
                conf, cv = at(a, 4), at(a, 5)
                if not np.isfinite(cv) or cv < 0 or cv != np.trunc(cv):
                    continue
                cls = int(cv)
            else:
                conf = f32(-np.inf)
                for c in range(4, class_fields):
                    if at(a, c) > conf:
                        conf, cls = at(a, c), c - 4
            if not np.isfinite(conf) or conf < thr:
                continue
            x, y, w, h = at(a, 0), at(a, 1), at(a, 2), at(a, 3)
            if not all(np.isfinite(v) for v in (x, y, w, h)):
                continue
            if e2e:
                w, h = w - x, h - y
            else:
                x, y = x - w * f32(.5), y - h * f32(.5)
            if w <= 0 or h <= 0:
                continue
            cand.append((cls, conf, x, y, w, h, a))
        cand.sort(key=lambda d: (-float(d[1]), d[6]))
        kept = []
        for d in cand[:max_candidates]:
            if not e2e and any((agnostic or k[0] == d[0]) and _iou(k[2:6], d[2:6]) > iou_thr for k in kept):
                continue
            kept.append(d)
            if len(kept) >= max_detections:
                break
        sw, sh, sx, sy, px, py = letterbox
        sw, sh, sx, sy, px, py = f32(sw), f32(sh), f32(sx), f32(sy), f32(px), f32(py)

        def clamp(v, hi):
            return f32(0) if v < 0 else hi if v > hi else v

        out = []
        for cls, conf, x, y, w, h, _ in kept:
            x1, y1 = clamp((x - px) / sx, sw), clamp((y - py) / sy, sh)
            x2, y2 = clamp((x + w - px) / sx, sw), clamp((y + h - py) / sy, sh)
            if x2 - x1 > 0 and y2 - y1 > 0:
                out.append((cls, float(conf), float(x1), float(y1), float(x2 - x1), float(y2 - y1)))
    return out


def random_raw_output(rng, anchors: int, nc: int, image: float = 640.0, dup: float = 0.3) -> np.ndarray:
    """A channels-first raw output [4 + nc][anchors] with clustered boxes (so NMS has work), repeated
    confidences (ties) and scores spread over (0, 1)."""
    out = np.zeros((4 + nc, anchors), np.float32)
    centres = rng.uniform(0, image, (max(1, anchors // 20), 2))
    pick = rng.integers(0, len(centres), anchors)
    out[0] = centres[pick, 0] + rng.normal(0, 4, anchors)
    out[1] = centres[pick, 1] + rng.normal(0, 4, anchors)
    out[2] = np.exp(rng.uniform(np.log(4), np.log(200), anchors))
    out[3] = np.exp(rng.uniform(np.log(4), np.log(200), anchors))
    scores = rng.uniform(0, 1, (nc, anchors)).astype(np.float32) ** 4
    ties = rng.uniform(0, 1, anchors) < dup
    scores[:, ties] = np.round(scores[:, ties] * 8) / 8
    out[4:] = scores
    return out
