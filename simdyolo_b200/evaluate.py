"""Detection validation: DetectionEvaluator (src/SimdYolo.Training/DetectionEvaluator.cs) on this library.

``calculate`` restates ``DetectionEvaluator.Calculate`` (DetectionEvaluator.cs:72-122): per class, the
predictions of every image ranked by confidence (then image, then prediction index), greedy one-to-one
matching against the unused ground truth of that class at the ten IoU thresholds 0.50:0.05:0.95, 101-point
interpolated AP (:129-138), precision / recall / TP / FP / FN at the operating confidence (IoU 0.5), the
confusion matrix with a background row and column, and macro averages over the classes that have ground
truth.  IoU (:124-128) and the thresholds are evaluated in single precision as the reference does; AP and the
averages in double.

``evaluate`` restates ``DetectionEvaluator.Evaluate`` (:45-66) for a session: inference on the GPU
(``Session.detect`` with the evaluator's detector settings, confidence 0.001, IoU 0.7, 300 detections), then
``calculate``.  The session's classes are the dataset's classes, so the reference's remapping of a
pretrained model's class names onto the dataset's is the identity here.

Ground truth is ``(class_id, x1, y1, x2, y2)`` (TrainingBox) and predictions ``(class_id, confidence, x, y,
width, height)`` (Detection), both in source-image pixels.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List, Sequence

import numpy as np

f32 = np.float32


@dataclass
class ClassEvaluation:
    class_id: int
    name: str
    ground_truth: int
    true_positive: int
    false_positive: int
    false_negative: int
    precision: float
    recall: float
    map50: float
    map50_95: float


@dataclass
class EvaluationResult:
    images: int
    precision: float
    recall: float
    map50: float
    map50_95: float
    classes: List[ClassEvaluation]
    confusion_matrix: List[List[int]]
    samples: list = field(default_factory=list)
    elapsed_ms: float = 0.0


def iou(prediction, truth) -> np.float32:
    """DetectionEvaluator.Iou (DetectionEvaluator.cs:124-128) in single precision."""
    _, _, x, y, w, h = prediction
    _, x1, y1, x2, y2 = truth
    x, y, w, h, x1, y1, x2, y2 = map(f32, (x, y, w, h, x1, y1, x2, y2))
    ix = max(f32(0), min(x + w, x2) - max(x, x1))
    iy = max(f32(0), min(y + h, y2) - max(y, y1))
    inter = f32(ix * iy)
    return f32(inter / max(f32(1e-12), w * h + (x2 - x1) * (y2 - y1) - inter))


def average_precision(matches: Sequence[bool], truths: int) -> float:
    """101-point interpolated AP (DetectionEvaluator.cs:129-138)."""
    if truths == 0 or len(matches) == 0:
        return 0.0
    n = len(matches)
    precision, recall = [0.0] * n, [0.0] * n
    tp = 0
    for i, m in enumerate(matches):
        tp += 1 if m else 0
        precision[i] = tp / (i + 1)
        recall[i] = tp / truths
    for i in range(n - 2, -1, -1):
        precision[i] = max(precision[i], precision[i + 1])
    total, index = 0.0, 0
    for r in range(101):
        while index < n and recall[index] < r / 100.0:
            index += 1
        if index < n:
            total += precision[index]
    return total / 101


def _finite(*v) -> bool:
    return all(np.isfinite(f32(x)) for x in v)


def _best_match(prediction, truths, used, threshold, cls=None) -> int:
    """Unused truth with the largest IoU >= threshold (the first one reaching it, then strictly larger)."""
    best, chosen = f32(threshold), -1
    for j, t in enumerate(truths):
        if used[j] or (cls is not None and t[0] != cls):
            continue
        overlap = iou(prediction, t)
        if overlap >= best and (chosen < 0 or overlap > best):
            best, chosen = overlap, j
    return chosen


def calculate(class_names: Sequence[str], samples, operating_confidence: float = 0.25) -> EvaluationResult:
    """DetectionEvaluator.Calculate.  samples: list of (truth boxes, predictions) per image."""
    nc = len(class_names)
    if not 1 <= nc <= 1000 or not np.isfinite(operating_confidence) or not 0 <= operating_confidence <= 1:
        raise ValueError("invalid evaluation classes or confidence")
    data = [(list(t), list(p)) for t, p in samples]
    for truth, preds in data:
        for c, x1, y1, x2, y2 in truth:
            if c < 0 or c >= nc or not _finite(x1, y1, x2, y2) or f32(x2) <= f32(x1) or f32(y2) <= f32(y1):
                raise ValueError("evaluation sample holds an invalid class or box")
        for c, conf, x, y, w, h in preds:
            if (c < 0 or c >= nc or not _finite(x, y, w, h, conf) or f32(w) <= 0 or f32(h) <= 0 or
                    not 0 <= f32(conf) <= 1):
                raise ValueError("evaluation sample holds an invalid class or box")
    operating = f32(operating_confidence)
    metrics = []
    for cls in range(nc):
        truths = sum(1 for truth, _ in data for t in truth if t[0] == cls)
        ranked = [(p, image, index) for image, (_, preds) in enumerate(data) for index, p in enumerate(preds)
                  if p[0] == cls]
        ranked.sort(key=lambda r: (-f32(r[0][1]), r[1], r[2]))
        aps = [0.0] * 10
        tp = fp = 0
        for threshold in range(10):
            used = [[False] * len(truth) for truth, _ in data]
            matches = [False] * len(ranked)
            limit = f32(f32(0.5) + f32(threshold) * f32(0.05))
            for i, (prediction, image, _) in enumerate(ranked):
                chosen = _best_match(prediction, data[image][0], used[image], limit, cls)
                if chosen >= 0:
                    matches[i] = True
                    used[image][chosen] = True
            aps[threshold] = average_precision(matches, truths)
            if threshold == 0:
                for i, (prediction, _, _) in enumerate(ranked):
                    if f32(prediction[1]) >= operating:
                        if matches[i]:
                            tp += 1
                        else:
                            fp += 1
        metrics.append(ClassEvaluation(cls, class_names[cls], truths, tp, fp, max(0, truths - tp),
                                       tp / (tp + fp) if tp + fp > 0 else 0.0, tp / truths if truths > 0 else 0.0,
                                       aps[0], sum(aps) / len(aps)))
    matrix = [[0] * (nc + 1) for _ in range(nc + 1)]
    for truth, preds in data:
        used = [False] * len(truth)
        kept = sorted((p for p in preds if f32(p[1]) >= operating), key=lambda p: -f32(p[1]))
        for prediction in kept:
            chosen = _best_match(prediction, truth, used, 0.5)
            if chosen < 0:
                matrix[nc][prediction[0]] += 1
            else:
                used[chosen] = True
                matrix[truth[chosen][0]][prediction[0]] += 1
        for j, t in enumerate(truth):
            if not used[j]:
                matrix[t[0]][nc] += 1
    present = [m for m in metrics if m.ground_truth > 0]

    def mean(key):
        return sum(getattr(m, key) for m in present) / len(present) if present else 0.0

    return EvaluationResult(len(data), mean("precision"), mean("recall"), mean("map50"), mean("map50_95"), metrics,
                            matrix, data)


def evaluate(session, images: np.ndarray, truths, class_names: Sequence[str], operating_confidence: float = 0.25,
             batch: int = 0, transforms=None) -> EvaluationResult:
    """DetectionEvaluator.Evaluate on the GPU: letterboxed uint8 images [N, S, S, 3], truths[N] lists of
    (class_id, x1, y1, x2, y2) in source pixels, transforms[N] (Letterbox records, None: identity)."""
    from . import evaluation_options

    if not np.isfinite(operating_confidence) or not 0 <= operating_confidence <= 1:
        raise ValueError("P/R confidence must be between 0 and 1")
    start = time.perf_counter()
    batch = batch or int(session.config.max_batch)
    predictions = []
    for i in range(0, len(images), batch):
        tf = None if transforms is None else list(transforms[i:i + batch])
        predictions += session.detect(images[i:i + batch], evaluation_options(), tf)
    result = calculate(class_names, list(zip(truths, predictions)), operating_confidence)
    result.elapsed_ms = (time.perf_counter() - start) * 1e3
    return result
