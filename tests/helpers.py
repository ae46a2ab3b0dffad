"""Shared test helpers: build oracle descriptors from the product's model description, and run the
oracle's head-only step (YoloTrainer.cs:185-197 with cached features) for parity checks."""
from __future__ import annotations

import ctypes as C

import numpy as np

import simdyolo_b200 as sy
from oracle import oracle as O


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def head_desc(cfg: sy.Config, epoch: int = 0) -> O.HeadDesc:
    d = O.HeadDesc()
    d.levels = 3
    d.nc = cfg.num_classes
    d.bins = cfg.reg_max
    for l in range(3):
        s = cfg.image_size >> (3 + l)
        d.hs[l] = s
        d.ws[l] = s
        d.strides[l] = float(8 << l)
    d.n_box_blocks = cfg.n_box_blocks
    d.n_cls_blocks = cfg.n_cls_blocks
    for l in range(3):
        for i in range(cfg.n_box_blocks):
            b = cfg.box_blocks[l][i]
            d.box_blocks[l][i] = O.Block(b.ic, b.oc, b.k, b.groups, b.has_bn, b.has_bias)
        for i in range(cfg.n_cls_blocks):
            b = cfg.cls_blocks[l][i]
            d.cls_blocks[l][i] = O.Block(b.ic, b.oc, b.k, b.groups, b.has_bn, b.has_bias)
    d.bn_eps = cfg.bn_eps
    d.bn_momentum = cfg.bn_momentum
    d.end_to_end = cfg.end_to_end
    d.epoch = epoch
    d.schedule_epochs = cfg.schedule_epochs
    return d


def backbone_desc(cfg: sy.Config) -> O.BackboneDesc:
    return O.BackboneDesc(cfg.image_size, cfg.width_mult, cfg.depth_mult, cfg.max_channels,
                          1 if cfg.backbone == sy.SY_BACKBONE_YOLO11 else 0)


def oracle_head_step(cfg: sy.Config, tensors, params, buffers, velocity, features, truth, epoch: int = 0):
    """Head forward / loss / backward per image, gradients summed in image order, then
    TrainingParameter.Update for every tensor.  Returns (losses[B] dicts, grad, params, buffers,
    velocity, connected) with arrays updated copies; connected: bit 0 cv2, bit 1 one2one_cv2."""
    L = O.lib()
    d = head_desc(cfg, epoch)
    params = params.astype(np.float32).copy()
    buffers = buffers.astype(np.float32).copy()
    velocity = velocity.astype(np.float32).copy()
    grad = np.zeros_like(params)
    losses = []
    connected_any = 0
    B = features[0].shape[0]
    for b in range(B):
        feats = [np.ascontiguousarray(f[b], np.float32) for f in features]
        VP = C.c_void_p * 3
        fp = VP(*[f.ctypes.data_as(C.c_void_p) for f in feats])
        out = O.Loss()
        conn = np.zeros(1, np.int32)
        tb = O.boxes(truth[b])
        rc = L.syo_head_image(C.byref(d), params, buffers, fp, tb, len(truth[b]), grad, C.byref(out), 1,
                              conn.ctypes.data_as(C.POINTER(C.c_int32)))
        assert rc == 0
        losses.append(dict(box=out.box, cls=out.cls, dfl=out.dfl, positives=out.positives))
        connected_any |= int(conn[0])
    summed = grad.copy()
    off = 0
    for t in tensors:
        if t["kind"] != 0:
            continue
        n = t["numel"]
        group = sy.tensor_group(t["name"])
        decay = t["name"].endswith("conv.weight") or (t["name"].endswith(".weight") and len(t["shape"]) == 4)
        has = bool((connected_any >> (group - 1)) & 1) if group else True
        w, v, g = params[off:off + n].copy(), velocity[off:off + n].copy(), grad[off:off + n].copy()
        rc = O.sgd_update(w, v, g, cfg.lr, cfg.momentum, cfg.weight_decay if decay else 0.0, B, has)
        assert rc == 0
        params[off:off + n], velocity[off:off + n] = w, v
        off += n
    return losses, summed, params, buffers, velocity, connected_any


def oracle_head_step_adamw(cfg: sy.Config, tensors, params, buffers, m1, m2, steps, features, truth, epoch=0):
    """Same head step followed by AdamW (torch.optim.AdamW form, lr / betas / eps / weight decay of the
    config) for every tensor; steps = per optimizer group (class branches, cv2, one2one_cv2) counts
    before this step, a box group stepping only when an image connected it.  Returns (losses, grad,
    params, buffers, m1, m2, steps) as updated copies."""
    losses, grad, _, buffers_out, _, connected = oracle_head_step(cfg, tensors, params, buffers,
                                                                  np.zeros_like(params), features, truth, epoch)
    params, m1, m2 = params.astype(np.float32).copy(), m1.astype(np.float32).copy(), m2.astype(np.float32).copy()
    steps = list(steps) + [0] * (3 - len(steps))
    has_group = [True, bool(connected & 1), bool(connected & 2)]
    B = features[0].shape[0]
    off = 0
    for t in tensors:
        if t["kind"] != 0:
            continue
        n = t["numel"]
        group = sy.tensor_group(t["name"])
        decay = t["name"].endswith("conv.weight") or (t["name"].endswith(".weight") and len(t["shape"]) == 4)
        has = has_group[group]
        w, a, b, g = params[off:off + n].copy(), m1[off:off + n].copy(), m2[off:off + n].copy(), grad[off:off + n].copy()
        rc = O.lib().syo_adamw_update(w, a, b, g, n, cfg.lr, cfg.beta1, cfg.beta2, cfg.adam_eps,
                                      cfg.weight_decay if decay else 0.0, steps[group] + 1, B, int(has))
        assert rc == 0
        params[off:off + n], m1[off:off + n], m2[off:off + n] = w, a, b
        off += n
    for gi in range(3):
        steps[gi] += int(has_group[gi])
    return losses, grad, params, buffers_out, m1, m2, steps
