"""Inference post-processing on the GPU through the C ABI, against the CPU oracle (oracle/detect.c), bit for
bit: sy_cuda_head_decode (CpuHead.DecodeInto), sy_cuda_end_to_end_topk (PtModel.EndToEndTopK),
sy_cuda_decode_detections (YoloDetector.DecodeIndexed) and the session's sy_cuda_detect / _features
(YoloDetector.Detect on the fine-tuned model), plus the evaluator on GPU detections.

The post-processing is integer and ordering work on float inputs evaluated with round-to-nearest
intrinsics and the same exp as the oracle, so every comparison here is exact; the one exception is the
NaN payload, which GPU arithmetic replaces by the canonical NaN (compared as NaN).  The session test
checks the head's raw outputs against the oracle's evaluation-mode head within the conv precision, and
the detections bit for bit against the oracle's decode of the GPU's own head outputs.
"""
import ctypes as C

import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data
from simdyolo_b200 import evaluate as E
from oracle import oracle as O
from tests import detect_cases as D
from tests.helpers import head_desc, rel_l2

pytestmark = pytest.mark.gpu
f32 = np.float32


def same_bits(a, b):
    return np.array_equal(D.f32_bits(a), D.f32_bits(b))


def same_or_both_nan(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    nan = np.isnan(a)
    return np.array_equal(nan, np.isnan(b)) and np.array_equal(D.f32_bits(a[~nan]), D.f32_bits(b[~nan]))


def as_array(dets):
    return np.array(dets, np.float64).reshape(-1, 6)


# ---------------------------------------------------------------- head decode

@pytest.mark.parametrize("width", [1, 3, 19, 80])
@pytest.mark.parametrize("bins", [1, 16])
@pytest.mark.parametrize("xyxy", [False, True])
def test_head_decode_coordinates(width, bins, xyxy):
    boxes, scores = D.head_coordinate_case(width, bins)
    got = sy.head_decode([(boxes, scores, 8.0)], bins, 3, xyxy)
    assert same_bits(got, O.head_decode([(boxes, scores, 8.0)], bins, 3, xyxy))


@pytest.mark.parametrize("stride", [1.25, -3.75, 0.0])
@pytest.mark.parametrize("xyxy", [False, True])
def test_head_decode_special_values(stride, xyxy):
    boxes, scores = D.special_case()
    got = sy.head_decode([(boxes, scores, stride)], 1, 1, xyxy)
    assert same_or_both_nan(got, O.head_decode([(boxes, scores, stride)], 1, 1, xyxy))


@pytest.mark.parametrize("bins,nc,size", [(16, 80, 640), (1, 3, 96), (16, 7, 200)])
def test_head_decode_three_levels(bins, nc, size):
    rng = np.random.default_rng(bins + nc)
    levels = []
    for l in range(3):
        h = (size + (8 << l) - 1) // (8 << l)
        levels.append(((rng.standard_normal((2, 4 * bins, h, h)) * 3).astype(np.float32),
                       (rng.standard_normal((2, nc, h, h)) * 4).astype(np.float32), float(8 << l)))
    for xyxy in (False, True):
        assert same_bits(sy.head_decode(levels, bins, nc, xyxy), O.head_decode(levels, bins, nc, xyxy))


# ---------------------------------------------------------------- end-to-end top-k

@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("classes", [1, 3, 7])
@pytest.mark.parametrize("anchors", [1, 7, 8, 9, 37])
@pytest.mark.parametrize("maximum", [1, 8, 49])
def test_end_to_end_topk_reference_cases(batch, classes, anchors, maximum):
    for frame in range(4):
        x = D.e2e_case(batch, classes, anchors, frame)
        got = sy.end_to_end_topk(x, classes, maximum)
        assert same_bits(got, O.end_to_end_topk(x, classes, maximum))   # scores are copied, payloads included


@pytest.mark.parametrize("anchors,nc,maximum,extra", [(8400, 80, 300, 0), (2100, 1, 300, 2), (33600, 80, 1024, 0),
                                                      (500, 3, 700, 1)])
def test_end_to_end_topk_large(anchors, nc, maximum, extra):
    rng = np.random.default_rng(anchors)
    x = rng.standard_normal((3, 4 + nc + extra, anchors)).astype(np.float32)
    x[:, 4:4 + nc] = np.round(rng.uniform(0, 1, (3, nc, anchors)) * 64) / 64   # many equal scores
    assert same_bits(sy.end_to_end_topk(x, nc, maximum), O.end_to_end_topk(x, nc, maximum))


# ---------------------------------------------------------------- DecodeIndexed

def oracle_decode(output, layout, class_count, lb, o):
    return O.decode_detections(output, layout, class_count, O.Letterbox(*lb), o.confidence, o.iou_threshold,
                               o.max_detections, o.max_candidates, bool(o.class_agnostic))


def test_decode_known_answer():
    raw, end = D.nms_case()
    lb = [sy.Letterbox(20, 20, 20, 20, 1, 1, 0, 0)]
    assert len(sy.decode_detections(raw, sy.SY_LAYOUT_CHANNELS_LAST, transforms=lb)[0]) == 2
    assert len(sy.decode_detections(end, sy.SY_LAYOUT_END_TO_END, transforms=lb)[0]) == 2


@pytest.mark.parametrize("confidence", [.25, .6, float("nan")])
def test_decode_channels_first_and_last(confidence):
    first, last = D.mask_pipeline_case()
    lb = (128, 32, 128, 32, 1., 1., 0, 0)
    o = sy.detect_options(confidence, .3, 300, 23)
    a = sy.decode_detections(first, sy.SY_LAYOUT_CHANNELS_FIRST, 3, [sy.Letterbox(*lb)], o)[0]
    b = sy.decode_detections(last, sy.SY_LAYOUT_CHANNELS_LAST, 3, [sy.Letterbox(*lb)], o)[0]
    want = oracle_decode(first, 1, 3, lb, o)
    assert a and np.array_equal(as_array(a), as_array(want)) and np.array_equal(as_array(b), as_array(want))
    # Auto resolves [1, 9, 35] with ClassCount 3 to channels-first
    assert np.array_equal(as_array(sy.decode_detections(first, sy.SY_LAYOUT_AUTO, 3, [sy.Letterbox(*lb)], o)[0]),
                          as_array(want))


CASES = [  # (confidence, iou, max_detections, max_candidates, agnostic)
    (.001, .7, 300, 30000, False), (.25, .45, 300, 30000, False), (.05, .5, 50, 400, False),
    (0.0, .3, 1000, 2000, True), (.1, .6, 7, 30000, False), (.5, 1.0, 300, 3, False)]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_decode_raw_head_outputs(case):
    conf, iou, max_det, max_cand, agnostic = CASES[case]
    rng = np.random.default_rng(100 + case)
    images, anchors, nc = 3, 8400, 80
    out = np.stack([D.random_raw_output(rng, anchors, nc) for _ in range(images)])
    lbs = [(640 + 13 * b, 360 + 7 * b, float(f32(0.5 + 0.25 * b)), float(f32(0.5 + 0.2 * b)), 4 * b, 140 - b)
           for b in range(images)]
    o = sy.detect_options(conf, iou, max_det, max_cand, agnostic)
    got = sy.decode_detections(out, sy.SY_LAYOUT_CHANNELS_FIRST, nc,
                               [sy.Letterbox(l[0], l[1], 640, 640, *l[2:]) for l in lbs], o)
    for b in range(images):
        want = oracle_decode(out[b], 1, nc, (lbs[b][0], lbs[b][1], 640, 640, *lbs[b][2:]), o)
        assert len(got[b]) == len(want) and np.array_equal(as_array(got[b]), as_array(want)), b


@pytest.mark.parametrize("max_candidates", [30000, 20000])
def test_decode_more_candidates_than_shared_memory_sorts(max_candidates):
    """33,600 anchors (a 1280 x 1280 input) all above the threshold: the kernel's second path (radix-select
    MaxCandidates, then repeated maxima) instead of the shared-memory sort, which holds 16,384 keys."""
    rng = np.random.default_rng(max_candidates)
    out = np.stack([D.random_raw_output(rng, 33600, 3, image=1280.0) for _ in range(2)])
    o = sy.detect_options(0.0, 0.6, 300, max_candidates)
    got = sy.decode_detections(out, sy.SY_LAYOUT_CHANNELS_FIRST, 3, None, o)
    lb = (1 << 20, 1 << 20, 1 << 20, 1 << 20, 1., 1., 0, 0)
    for b in range(2):
        assert np.array_equal(as_array(got[b]), as_array(oracle_decode(out[b], 1, 3, lb, o))), b


def test_decode_end_to_end_rows():
    rng = np.random.default_rng(7)
    rows = rng.uniform(0, 600, (2, 300, 6)).astype(np.float32)
    rows[..., 2:4] = rows[..., :2] + rng.uniform(-5, 80, (2, 300, 2)).astype(np.float32)
    rows[..., 4] = np.round(rng.uniform(0, 1, (2, 300)) * 16) / 16
    rows[..., 5] = rng.integers(0, 80, (2, 300))
    rows[0, 5, 5] = 2.5          # non-integer class: skipped
    rows[1, 9, 5] = -1           # negative class: skipped
    o = sy.detect_options(.2, .45, 100, 250)
    got = sy.decode_detections(rows, sy.SY_LAYOUT_END_TO_END, 0, None, o)
    lb = (1 << 20, 1 << 20, 1 << 20, 1 << 20, 1., 1., 0, 0)
    for b in range(2):
        assert np.array_equal(as_array(got[b]), as_array(oracle_decode(rows[b], 3, 0, lb, o)))
    rows[1, 3, 5] = 3e9          # the reference's checked conversion throws
    with pytest.raises(sy.InvalidArgument):
        sy.decode_detections(rows, sy.SY_LAYOUT_END_TO_END, 0, None, o)


def test_decode_rejects_bad_arguments():
    out = np.zeros((1, 84, 100), np.float32)
    with pytest.raises(sy.InvalidArgument):
        sy.decode_detections(out, 7, 80)
    with pytest.raises(sy.InvalidArgument):
        sy.decode_detections(out, sy.SY_LAYOUT_CHANNELS_FIRST, 90)
    with pytest.raises(sy.InvalidArgument):
        sy.decode_detections(out, sy.SY_LAYOUT_CHANNELS_FIRST, 80, options=sy.detect_options(max_detections=0))
    with pytest.raises(sy.InvalidArgument):
        sy.decode_detections(out, sy.SY_LAYOUT_CHANNELS_FIRST, 80,
                             transforms=[sy.Letterbox(0, 10, 10, 10, 1, 1, 0, 0)])
    with pytest.raises(sy.InvalidArgument):   # [84, 84] is ambiguous without a class count
        sy.decode_detections(np.zeros((1, 84, 84), np.float32), sy.SY_LAYOUT_AUTO, 0)


# ---------------------------------------------------------------- session inference

def oracle_head_outputs(cfg, params, buffers, feats, set_=0):
    d = head_desc(cfg)
    images = feats[0].shape[0]
    box = [np.zeros((images, 4 * cfg.reg_max) + f.shape[2:], np.float32) for f in feats]
    cls = [np.zeros((images, cfg.num_classes) + f.shape[2:], np.float32) for f in feats]
    for b in range(images):
        fs = [np.ascontiguousarray(f[b], np.float32) for f in feats]
        bo = [np.zeros(x.shape[1:], np.float32) for x in box]
        co = [np.zeros(x.shape[1:], np.float32) for x in cls]
        P = C.c_void_p * 3
        assert O.lib().syo_head_eval_outputs(C.byref(d), params, buffers, P(*[f.ctypes.data for f in fs]), set_,
                                             P(*[x.ctypes.data for x in bo]), P(*[x.ctypes.data for x in co])) == 0
        for l in range(3):
            box[l][b], cls[l][b] = bo[l], co[l]
    return box, cls


def oracle_detect(cfg, box, cls, o, transforms=None):
    """PtModel.Detect + DecodeIndexed on given head outputs, per image, in the oracle."""
    levels = [(box[l], cls[l], float(8 << l)) for l in range(3)]
    e2e = bool(cfg.end_to_end)
    dec = O.head_decode(levels, cfg.reg_max, cfg.num_classes, xyxy=e2e)
    s = cfg.image_size
    out = []
    for b in range(dec.shape[0]):
        lb = transforms[b] if transforms else (s, s, s, s, 1., 1., 0, 0)
        if e2e:
            rows = O.end_to_end_topk(dec[b:b + 1], cfg.num_classes, 300)[0]
            out.append(oracle_decode(rows, 3, 0, lb, o))
        else:
            out.append(oracle_decode(dec[b], 1, cfg.num_classes, lb, o))
    return out


def session_with_state(cfg, seed):
    s = sy.Session(cfg)
    rng = np.random.default_rng(seed)
    params, buffers = data.head_params(s, seed, cfg.image_size)
    params = params + (rng.standard_normal(params.size) * 0.05).astype(np.float32)
    off = 0
    for t in s.tensors:   # class biases around sigmoid(-2.5), so that a few hundred anchors pass 0.01
        if t["kind"] == 0:
            if t["name"].endswith(".bias") and not t["name"].endswith("bn.bias") and "cv3" in t["name"].split(".")[0]:
                params[off:off + t["numel"]] = rng.normal(-2.5, 1.5, t["numel"])
            off += t["numel"]
    off = 0
    for t in s.tensors:
        if t["kind"] == 1:
            n = t["numel"]
            if t["name"].endswith("running_mean"):
                buffers[off:off + n] = rng.normal(0.0, 0.2, n)
            elif t["name"].endswith("running_var"):
                buffers[off:off + n] = rng.uniform(0.5, 2.0, n)
            off += n
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    return s, params, buffers


@pytest.mark.parametrize("model,end_to_end,reg_max", [("yolov8n", False, 16), ("yolo11s", False, 16),
                                                       ("yolov8n", True, 16), ("yolov8n", True, 1)])
def test_session_detect_features(model, end_to_end, reg_max):
    image, images = 256, 3
    cfg = sy.make_config(model, image_size=image, max_batch=4, max_boxes=8, backbone=False, num_classes=20,
                         reg_max=reg_max, end_to_end=end_to_end, precision=sy.SY_PRECISION_3XTF32)
    s, params, buffers = session_with_state(cfg, 5)
    rng = np.random.default_rng(11)
    feats = [(rng.standard_normal((images, cfg.feature_channels[l], image >> (3 + l), image >> (3 + l))) * 0.7
              + 0.2).astype(np.float32) for l in range(3)]
    lbs = [(500, 400, image, image, float(f32(image / 500)), float(f32(image / 500)), 0, 28 + b) for b in range(images)]
    o = sy.detect_options(0.01, 0.5, 300)
    before_p, before_b = s.flat_params(), s.flat_buffers()
    got = s.detect_features(feats, o, [sy.Letterbox(*lb) for lb in lbs])
    set_ = 1 if end_to_end else 0
    box = [None] * 3
    cls = [None] * 3
    for l in range(3):
        box[l], cls[l] = s.last_head_outputs(l, images, set_)
    wb, wc = oracle_head_outputs(cfg, params, buffers, feats, set_)
    err = max(max(rel_l2(box[l], wb[l]), rel_l2(cls[l], wc[l])) for l in range(3))
    print(f"head outputs vs oracle (3xTF32): {err:.2e}; detections per image {[len(g) for g in got]}")
    assert err <= 1e-5
    want = oracle_detect(cfg, box, cls, o, lbs)
    for b in range(images):
        assert len(got[b]) > 0
        assert np.array_equal(as_array(got[b]), as_array(want[b])), b
    assert s.flat_params().tobytes() == before_p.tobytes() and s.flat_buffers().tobytes() == before_b.tobytes()
    s.close()


def test_session_detect_rgb_and_evaluate():
    image, images = 256, 4
    cfg = sy.make_config("yolov8n", image_size=image, max_batch=images, max_boxes=8, num_classes=80)
    s, params, buffers = session_with_state(cfg, 9)
    s.set_backbone(data.backbone_params("yolov8n", seed=9))
    rng = np.random.default_rng(2)
    imgs, _ = data.synthetic_batch(rng, images, image, 80, boxes=(1, 4), wh=(8.0, 128.0))
    o = sy.evaluation_options()
    got = s.detect(imgs, o)
    box, cls = zip(*[s.last_head_outputs(l, images) for l in range(3)])
    want = oracle_detect(cfg, list(box), list(cls), o)
    for b in range(images):
        assert np.array_equal(as_array(got[b]), as_array(want[b])), b
    # the detections as ground truth: every prediction matches its own box at IoU 1
    truths = [[(d[0], d[2], d[3], f32(d[2]) + f32(d[4]), f32(d[3]) + f32(d[5])) for d in g] for g in got]
    r = E.evaluate(s, imgs, truths, [str(i) for i in range(80)])
    assert sum(len(g) for g in got) > 0
    assert r.map50 == 1.0 and r.map50_95 == 1.0
    with pytest.raises(sy.InvalidArgument):
        s.detect(imgs, sy.detect_options(confidence=1.5))
    s.close()
