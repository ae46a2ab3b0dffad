"""End-to-end (dual-branch) detection heads in the oracle (DetectionHead.cs:20-26, :105-120;
TrainingHeadSchema.cs:7-21) against a torch restatement of the head branches whose outputs feed the
oracle's DetectionLoss once per branch set (that loss is pinned on its own against autograd and the
reference's known answers): the one-to-many set with top-k 10 / 10, the one-to-one set with top-k 1
(7 when progressive) and a second top-1, each set's output gradient scaled by its weight and the
reported parts summed with the same weights.  Also the head-schema checks of the C ABI, which run
before any device call."""
import ctypes as C

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import simdyolo_b200 as sy
from oracle import oracle as O
from tests.helpers import head_desc, rel_l2


def block_path(i, n):
    return ["0.0", "0.1", "1.0", "1.1", "2"][i] if n == 5 else str(i)


def head_layout(cfg):
    """(name, shape, block, set, box, level) of every parameter in Snapshot order, restated from
    DetectionHead.BuildBranch (DetectionHead.cs:28-75): cv2, cv3, then one2one_cv2, one2one_cv3."""
    out = []
    sets = 2 if cfg.end_to_end else 1
    for st in range(sets):
        for box in (True, False):
            for lvl in range(3):
                prefix = ("one2one_" if st else "") + ("cv2" if box else "cv3") + f".{lvl}"
                n = cfg.n_box_blocks if box else cfg.n_cls_blocks
                blocks = cfg.box_blocks[lvl] if box else cfg.cls_blocks[lvl]
                for i in range(n):
                    b = blocks[i]
                    path = f"{prefix}.{block_path(i, n)}"
                    conv = path + (".conv" if b.has_bn else "")
                    out.append((conv + ".weight", (b.oc, b.ic // b.groups, b.k, b.k), b, st, box, lvl))
                    if b.has_bias:
                        out.append((conv + ".bias", (b.oc,), b, st, box, lvl))
                    if b.has_bn:
                        out.append((path + ".bn.weight", (b.oc,), b, st, box, lvl))
                        out.append((path + ".bn.bias", (b.oc,), b, st, box, lvl))
    return out


def random_head(cfg, rng):
    params = []
    for name, shape, *_ in head_layout(cfg):
        n = int(np.prod(shape))
        if len(shape) == 4:
            params.append(rng.uniform(-1, 1, n) / np.sqrt(np.prod(shape[1:])))
        elif name.endswith("bn.weight"):
            params.append(rng.uniform(0.8, 1.2, n))
        elif name.endswith("bn.bias"):
            params.append(rng.normal(0, 0.1, n))
        else:
            params.append(np.full(n, 1.0 if "cv2" in name.split(".")[0] else -4.0) + rng.normal(0, 0.1, n))
    return np.concatenate(params).astype(np.float32)


def torch_head(cfg, flat, feats):
    """Branch outputs [set][box/cls][level] of one image with training BatchNorm (batch statistics of
    this image, HeadOperations.cs:158-166), plus the per-block (mean, biased var) for the running fold."""
    layout = head_layout(cfg)
    tensors, off = {}, 0
    for name, shape, *_ in layout:
        n = int(np.prod(shape))
        tensors[name] = torch.tensor(flat[off:off + n].reshape(shape), requires_grad=True)
        off += n
    outs, stats = {}, []
    sets = 2 if cfg.end_to_end else 1
    for st in range(sets):
        for box in (True, False):
            for lvl in range(3):
                prefix = ("one2one_" if st else "") + ("cv2" if box else "cv3") + f".{lvl}"
                n = cfg.n_box_blocks if box else cfg.n_cls_blocks
                blocks = cfg.box_blocks[lvl] if box else cfg.cls_blocks[lvl]
                x = torch.tensor(feats[lvl])[None]
                for i in range(n):
                    b = blocks[i]
                    path = f"{prefix}.{block_path(i, n)}"
                    conv = path + (".conv" if b.has_bn else "")
                    x = F.conv2d(x, tensors[conv + ".weight"], tensors.get(conv + ".bias"), padding=b.k // 2,
                                 groups=b.groups)
                    if b.has_bn:
                        mean = x.mean((0, 2, 3))
                        var = x.var((0, 2, 3), unbiased=False)
                        stats.append((mean.detach().numpy(), var.detach().numpy()))
                        x = (x - mean[None, :, None, None]) / torch.sqrt(var[None, :, None, None] + cfg.bn_eps)
                        x = x * tensors[path + ".bn.weight"][None, :, None, None] + \
                            tensors[path + ".bn.bias"][None, :, None, None]
                        x = F.silu(x)
                outs[(st, box, lvl)] = x[0]
    return tensors, layout, outs, stats


def progressive_weight(epoch, epochs):
    t = np.float32(max(np.float32(1) - np.float32(epoch) / np.float32(max(epochs - 1, 1)), 0))
    return np.float32(np.float32(t * np.float32(0.7)) + np.float32(0.1))


CASES = [
    # model head, reg_max, epoch, schedule: YOLOv10 v10Detect (legacy end to end) and the YOLO26-style
    # progressive loss at the start, middle and past the end of its schedule
    ("yolov8n", 16, 0, 100),
    ("yolo11s", 1, 0, 5),
    ("yolo11s", 1, 2, 5),
    ("yolov8n", 1, 9, 5),
]


@pytest.mark.parametrize("model,reg_max,epoch,schedule", CASES)
def test_end_to_end_head_matches_torch_restatement(model, reg_max, epoch, schedule):
    rng = np.random.default_rng(17 + epoch + reg_max)
    cfg = sy.make_config(model, image_size=64, max_batch=1, max_boxes=6, num_classes=5, backbone=False,
                         end_to_end=True, reg_max=reg_max, schedule_epochs=schedule)
    d = head_desc(cfg, epoch)
    flat = random_head(cfg, rng)
    assert O.lib().syo_head_param_count(C.byref(d)) == flat.size
    feats = [(rng.standard_normal((cfg.feature_channels[l], 64 >> (3 + l), 64 >> (3 + l))) * 0.8 + 0.1)
             .astype(np.float32) for l in range(3)]
    truth = [(1, 6.0, 9.0, 30.0, 41.0), (3, 33.0, 4.0, 60.0, 22.0), (0, 20.0, 40.0, 50.0, 62.0)]
    # oracle
    nb = O.lib().syo_head_buffer_count(C.byref(d))
    buffers = np.zeros(nb, np.float32)
    grad = np.zeros_like(flat)
    fp = (C.c_void_p * 3)(*[f.ctypes.data_as(C.c_void_p) for f in feats])
    loss = O.Loss()
    conn = np.zeros(1, np.int32)
    assert O.lib().syo_head_image(C.byref(d), flat, buffers, fp, O.boxes(truth), len(truth), grad, C.byref(loss), 1,
                                  conn.ctypes.data_as(C.POINTER(C.c_int32))) == 0
    # torch branches + the oracle loss per set
    tensors, layout, outs, stats = torch_head(cfg, flat, feats)
    progressive = reg_max == 1
    w = progressive_weight(epoch, schedule) if progressive else np.float32(1)
    weights = [w, np.float32(1) - w] if progressive else [np.float32(1), np.float32(1)]
    parts, grads_out, connected = [], [], 0
    for st in range(2):
        bl = [outs[(st, True, l)].detach().numpy() for l in range(3)]
        cl = [outs[(st, False, l)].detach().numpy() for l in range(3)]
        topk, topk2 = (10, 10) if st == 0 else ((7 if progressive else 1), 1)
        part, db, dc, _, _ = O.detection_loss(bl, cl, [8.0, 16.0, 32.0], truth, cfg.num_classes, bins=reg_max,
                                              topk=topk, topk2=topk2, grad_scale=float(weights[st]))
        parts.append(part)
        connected |= int(bool(part["connected"])) << st
        for l in range(3):
            grads_out += [(outs[(st, True, l)], torch.tensor(db[l])), (outs[(st, False, l)], torch.tensor(dc[l]))]
    torch.autograd.backward([o for o, _ in grads_out], [g for _, g in grads_out])
    ref = np.concatenate([tensors[name].grad.numpy().ravel() for name, *_ in layout])
    assert connected == 3 and conn[0] == 3
    for k in ("box", "cls", "dfl"):
        want = np.float32(np.float32(parts[0][k] * weights[0]) + np.float32(parts[1][k] * weights[1]))
        assert abs(getattr(loss, k) - want) <= 1e-6 * max(1.0, abs(want)), k
    assert loss.positives == parts[0]["positives"] + parts[1]["positives"]
    # the one-to-one assigner keeps one anchor per truth box unless progressive (top 7, then top 1)
    assert parts[1]["positives"] <= len(truth)
    assert rel_l2(grad, ref) < 1e-4
    # every branch, one-to-one included, folded its batch statistics into the running buffers
    # (from zero: mean 0.03 * batch mean, variance 0.03 * unbiased batch variance, one batch tracked)
    off, si = 0, 0
    for name, shape, b, st, box, lvl in layout:
        if not name.endswith("bn.weight"):
            continue
        mean, var = stats[si]
        si += 1
        c, n = shape[0], (64 >> (3 + lvl)) ** 2
        assert np.allclose(buffers[off:off + c], 0.03 * mean, rtol=1e-4, atol=1e-7), name
        assert np.allclose(buffers[off + c:off + 2 * c], 0.03 * var * n / (n - 1), rtol=1e-4, atol=1e-7), name
        assert buffers[off + 2 * c] == 1.0
        off += 2 * c + 1
    assert si == len(stats) and off == nb


def test_schema_is_checked_before_the_device():
    """TrainingHeadSchema.Read: reg_max is 1 or 16 and one bin needs the one-to-one branches; the C
    ABI refuses other heads while validating the description, before any CUDA call."""
    L = sy.lib()
    for kwargs in (dict(reg_max=1), dict(reg_max=8, end_to_end=True)):
        cfg = sy.make_config("yolov8n", image_size=64, max_batch=1, backbone=False, **kwargs)
        h = C.c_void_p()
        assert L.sy_cuda_create(C.byref(cfg), C.byref(h)) == sy.SY_ERR_UNSUPPORTED_SHAPE
        assert not h.value
    cfg = sy.make_config("yolov8n", image_size=64, max_batch=1, backbone=False, end_to_end=True, reg_max=1,
                         schedule_epochs=-1)
    h = C.c_void_p()
    assert L.sy_cuda_create(C.byref(cfg), C.byref(h)) == sy.SY_ERR_INVALID_ARGUMENT


def test_progressive_weight_schedule_matches_reference_formula():
    for epoch, epochs in [(0, 5), (1, 5), (2, 5), (4, 5), (7, 5), (0, 1), (3, 1), (50, 100)]:
        assert O.lib().syo_progressive_weight(epoch, epochs) == progressive_weight(epoch, epochs)
