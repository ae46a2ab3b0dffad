"""Seeded synthetic workloads and random initialisation (no datasets or checkpoints are available).

Images: RGB24 bytes uniform in [0, 255].  Boxes: per image a uniform count in [lo, hi], class uniform
in [0, nc), centre uniform over the image, width/height log-uniform in [wmin, wmax] pixels, clipped
to the image (the synthetic distributions the benchmark configurations name).
"""
from __future__ import annotations

import numpy as np

from . import MODELS, Session, model_family, yolo11_backbone_convs, yolov8_backbone_convs


def synthetic_batch(rng: np.random.Generator, batch: int, size: int, nc: int, boxes=(1, 8), wh=(8.0, 320.0)):
    images = rng.integers(0, 256, size=(batch, size, size, 3), dtype=np.uint8)
    truth = []
    for _ in range(batch):
        n = int(rng.integers(boxes[0], boxes[1] + 1))
        per = []
        for _ in range(n):
            w, h = np.exp(rng.uniform(np.log(wh[0]), np.log(wh[1]), 2))
            cx, cy = rng.uniform(0, size, 2)
            x1, y1 = max(0.0, cx - w / 2), max(0.0, cy - h / 2)
            x2, y2 = min(float(size), cx + w / 2), min(float(size), cy + h / 2)
            per.append((int(rng.integers(0, nc)), float(np.float32(x1)), float(np.float32(y1)),
                        float(np.float32(x2)), float(np.float32(y2))))
        truth.append(per)
    return images, truth


def backbone_params(model, seed: int) -> np.ndarray:
    """Random frozen trunk (BatchNorm folded): He-normal weights, small biases, trunk order.
    `model`: a name from MODELS, or a (width, depth, max_channels) tuple of the YOLOv8 family."""
    if isinstance(model, str):
        width, depth, max_ch = MODELS[model]
        convs = (yolo11_backbone_convs if model_family(model) == "yolo11" else yolov8_backbone_convs)(width, depth,
                                                                                                      max_ch)
    else:
        width, depth, max_ch = model
        convs = yolov8_backbone_convs(width, depth, max_ch)
    rng = np.random.default_rng(seed)
    parts = []
    for oc, ic, k in convs:
        std = np.sqrt(2.0 / (ic * k * k)) * 0.8
        parts.append((rng.standard_normal(oc * ic * k * k) * std).astype(np.float32))
        parts.append((rng.standard_normal(oc) * 0.05).astype(np.float32))
    return np.concatenate(parts)


def head_params(session: Session, seed: int, image_size: int = 640) -> tuple[np.ndarray, np.ndarray]:
    """Random head in Snapshot order: conv weights uniform(+-1/sqrt(fan_in)) (torch Conv2d default),
    BN gamma 1 / beta 0, final box bias 1.0, final class bias log(5 / nc / (640 / s)^2)
    (the reference's class re-initialisation, DetectionHead.cs:52-54).  Buffers: mean 0, var 1, tracked 0."""
    rng = np.random.default_rng(seed)
    nc = session.config.num_classes
    params, buffers = [], []
    for t in session.tensors:
        name, shape, n = t["name"], t["shape"], t["numel"]
        if t["kind"] == 0:
            if name.endswith("conv.weight") or (name.endswith(".weight") and len(shape) == 4):
                fan_in = shape[1] * shape[2] * shape[3]
                bound = 1.0 / np.sqrt(fan_in)
                v = rng.uniform(-bound, bound, n)
            elif name.endswith("bn.weight"):
                v = np.ones(n)
            elif name.endswith("bn.bias"):
                v = np.zeros(n)
            else:  # final conv bias
                level = int(name.split(".")[1])
                stride = 8 << level
                box = "cv2" in name.split(".")[0]
                v = np.full(n, 1.0) if box else np.full(n, np.log(5.0 / nc / (640.0 / stride) ** 2))
            params.append(v.astype(np.float32))
        else:
            v = np.ones(n) if name.endswith("running_var") else np.zeros(n)
            buffers.append(v.astype(np.float32))
    return np.concatenate(params), np.concatenate(buffers)
