"""Pins the oracle's inference post-processing (oracle/detect.c) and the host evaluator
(simdyolo_b200/evaluate.py) to the reference's own tests and to independent restatements.

Reference tests restated (paths inside the reference project):
  tests/SimdYolo.Tests/Program.cs:227-233                 class-aware NMS, end-to-end rows skip NMS
  tests/SimdYolo.Tests/CpuHeadCoordinatesTests.cs:12-57   head coordinates (bit-exact for bins 1)
  tests/SimdYolo.Tests/CpuPtEndToEndTests.cs:13-26        end-to-end top-k against full sorts, bitwise
  tests/SimdYolo.Tests/MaskPipelineTests.cs:89-110        channels-first and channels-last decode agree
  tests/SimdYolo.Training.Tests/FeatureTests.cs:14-21     AP101 known answers
"""
import numpy as np
import pytest

from oracle import oracle as O
from simdyolo_b200 import evaluate as E
from tests import detect_cases as D

f32 = np.float32


def same_bits(a, b):
    return np.array_equal(D.f32_bits(a), D.f32_bits(b))


def test_nms_known_answer():
    raw, end = D.nms_case()
    lb = O.Letterbox(20, 20, 20, 20, 1, 1, 0, 0)
    got = O.decode_detections(raw, 2, 0, lb)
    assert len(got) == 2                       # the 0.8 box of class 0 is suppressed by the 0.9 one
    assert [d[0] for d in got] == [1, 0]
    assert len(O.decode_detections(end, 3, 0, lb)) == 2   # end-to-end rows are not suppressed


@pytest.mark.parametrize("width", [1, 3, 19, 80])
@pytest.mark.parametrize("bins", [1, 16])
@pytest.mark.parametrize("xyxy", [False, True])
def test_head_coordinates(width, bins, xyxy):
    boxes, scores = D.head_coordinate_case(width, bins)
    batch, height = boxes.shape[0], boxes.shape[2]
    spatial = width * height
    saved = boxes.copy()
    out = O.head_decode([(boxes, scores, 8.0)], bins, 3, xyxy)
    assert np.array_equal(boxes, saved)
    flat = saved.reshape(batch, 4, bins, spatial)
    for b in range(batch):
        want = D.expected_coordinates(lambda side, a: flat[b, side, 0, a] if bins == 1 else f32(7.5), width, spatial,
                                      8.0, xyxy)
        got = out[b, :4]
        if bins == 1:
            assert same_bits(got, want)
        else:
            assert np.all(np.isfinite(got))
            assert np.all(np.abs(got - want) <= 2e-5 * np.maximum(1, np.abs(want)))
        assert np.all(out[b, 4:] == f32(.5))   # sigmoid(0)


@pytest.mark.parametrize("stride", [1.25, -3.75, 0.0])
@pytest.mark.parametrize("xyxy", [False, True])
def test_head_coordinates_special_values(stride, xyxy):
    boxes, scores = D.special_case()
    width, spatial = boxes.shape[3], boxes.shape[2] * boxes.shape[3]
    out = O.head_decode([(boxes, scores, stride)], 1, 1, xyxy)
    flat = boxes.reshape(4, spatial)
    want = D.expected_coordinates(lambda side, a: flat[side, a], width, spatial, stride, xyxy)
    assert same_bits(out[0, :4], want)


def test_head_decode_joins_levels_in_order():
    rng = np.random.default_rng(3)
    levels = [(rng.normal(size=(2, 64, 3, w)).astype(np.float32), rng.normal(size=(2, 5, 3, w)).astype(np.float32),
               float(8 << i)) for i, w in enumerate((19, 17))]
    joined = O.head_decode(levels, 16, 5)
    parts = [O.head_decode([lv], 16, 5) for lv in levels]
    assert same_bits(joined, np.concatenate(parts, axis=2))


@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("classes", [1, 3, 7])
@pytest.mark.parametrize("anchors", [1, 7, 8, 9, 37])
@pytest.mark.parametrize("maximum", [1, 8, 49])
def test_end_to_end_topk(batch, classes, anchors, maximum):
    for frame in range(4):
        x = D.e2e_case(batch, classes, anchors, frame)
        assert same_bits(O.end_to_end_topk(x, classes, maximum), D.e2e_expected(x, maximum, classes))


@pytest.mark.parametrize("confidence", [.25, .6, float("nan")])
def test_channels_first_and_last_agree(confidence):
    first, last = D.mask_pipeline_case()
    lb = O.Letterbox(128, 32, 128, 32, 1, 1, 0, 0)
    kw = dict(class_count=3, letterbox=lb, confidence=confidence, iou_threshold=.3, max_candidates=23)
    a = O.decode_detections(first, 1, **kw)
    b = O.decode_detections(last, 2, **kw)
    assert a and a == b
    want = D.decode_expected(first, 1, 3, (128, 32, 1., 1., 0, 0), confidence, .3, 300, 23)
    assert np.array_equal(np.array(a, np.float64), np.array(want, np.float64))


@pytest.mark.parametrize("seed", range(6))
def test_decode_matches_scalar_restatement(seed):
    rng = np.random.default_rng(seed)
    nc, anchors = [(1, 50), (3, 200), (80, 300), (5, 400), (2, 120), (7, 333)][seed]
    out = D.random_raw_output(rng, anchors, nc)
    lb = (640 + seed * 7, 480 - seed * 5, float(f32(0.75 + seed * 0.1)), float(f32(0.75 + seed * 0.05)), 3 * seed, 40)
    opts = dict(confidence=[.001, .25, .05, 0, .5, .1][seed], iou_threshold=[.7, .45, .5, .3, 1.0, .6][seed],
                max_detections=[300, 20, 50, 7, 300, 100][seed], max_candidates=[30000, 100, 37, 30000, 5, 60][seed],
                class_agnostic=seed in (2, 5))
    got = O.decode_detections(out, 1, nc, O.Letterbox(lb[0], lb[1], 640, 640, lb[2], lb[3], lb[4], lb[5]), **opts)
    want = D.decode_expected(out, 1, nc, lb, opts["confidence"], opts["iou_threshold"], opts["max_detections"],
                             opts["max_candidates"], opts["class_agnostic"])
    assert np.array_equal(np.array(got, np.float64).reshape(-1, 6), np.array(want, np.float64).reshape(-1, 6))


# ---------------------------------------------------------------- evaluator

def test_ap101_known_answers():
    truth = [(0, 0, 0, 10, 10)]
    hit = (0, .9, 0, 0, 10, 10)
    assert abs(E.calculate(["a"], [(truth, [hit])]).map50_95 - 1) <= 1e-12
    duplicate = E.calculate(["a"], [(truth, [hit, (0, .8, 0, 0, 10, 10)])])
    assert abs(duplicate.precision - .5) <= 1e-12 and abs(duplicate.map50 - 1) <= 1e-12
    false_first = E.calculate(["a"], [(truth, [(0, .99, 20, 0, 10, 10), hit])])
    assert abs(false_first.map50 - .5) <= 1e-12
    wrong = E.calculate(["a", "b"], [(truth, [(1, .9, 0, 0, 10, 10)])])
    assert wrong.map50 == 0 and wrong.confusion_matrix[0][1] == 1
    assert E.calculate(["a"], [([], [hit])]).map50 == 0


def test_evaluator_rejects_invalid_samples():
    with pytest.raises(ValueError):
        E.calculate(["a"], [([(0, 0, 0, 10, 10)], [(0, 1.5, 0, 0, 10, 10)])])
    with pytest.raises(ValueError):
        E.calculate(["a"], [([(1, 0, 0, 10, 10)], [])])
    with pytest.raises(ValueError):
        E.calculate(["a"], [([(0, 0, 0, 0, 10)], [])])
    with pytest.raises(ValueError):
        E.calculate([], [])


def test_evaluator_partial_matches_and_thresholds():
    """A box at IoU 0.68 matches at thresholds 0.50..0.65 only: AP50-95 = 4 / 10 of AP50; a lower-ranked
    duplicate is a false positive; the confusion matrix counts the background column for a missed truth."""
    truth = [(0, 0, 0, 10, 10), (1, 50, 50, 60, 60)]
    pred = [(0, .9, 0, 0, 10, 6.8), (0, .5, 0, 0, 10, 10), (1, .1, 50, 50, 10, 10)]
    r = E.calculate(["a", "b"], [(truth, pred)])
    a = r.classes[0]
    assert a.map50 == 1.0 and abs(a.map50_95 - 0.4 * 1.0 - 0.6 * 0.5) < 1e-12   # the 0.5 box matches above 0.65
    assert (a.true_positive, a.false_positive, a.false_negative) == (1, 1, 0)
    b = r.classes[1]
    assert b.map50_95 == 1.0 and (b.true_positive, b.false_negative) == (0, 1)   # below the operating confidence
    assert r.confusion_matrix[1][2] == 1 and r.confusion_matrix[0][0] == 1 and r.confusion_matrix[2][0] == 1
