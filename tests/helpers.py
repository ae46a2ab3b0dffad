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


def _block_path(i: int, n: int) -> str:
    return ["0.0", "0.1", "1.0", "1.1", "2"][i] if n == 5 else str(i)


def snapshot_tensors(cfg: sy.Config):
    """The session's tensor list (DetectionHead.Snapshot order, DetectionHead.cs:124-130) restated on the
    host: every parameter (cv2.0-2, cv3.0-2, then one2one_cv2 / one2one_cv3; per block weight, [bias],
    [bn gamma, beta]), then per BatchNorm block running_mean, running_var, num_batches_tracked.  Same
    dict layout as Session.tensors, so seeded initial states can be built without a GPU."""
    params, buffers = [], []
    for st in range(2 if cfg.end_to_end else 1):
        for box in (True, False):
            for lvl in range(3):
                prefix = ("one2one_" if st else "") + ("cv2" if box else "cv3") + f".{lvl}"
                n = cfg.n_box_blocks if box else cfg.n_cls_blocks
                blocks = cfg.box_blocks[lvl] if box else cfg.cls_blocks[lvl]
                for i in range(n):
                    b = blocks[i]
                    path = f"{prefix}.{_block_path(i, n)}"
                    conv = path + (".conv" if b.has_bn else "")
                    params.append((conv + ".weight", (b.oc, b.ic // b.groups, b.k, b.k)))
                    if b.has_bias:
                        params.append((conv + ".bias", (b.oc,)))
                    if b.has_bn:
                        params.append((path + ".bn.weight", (b.oc,)))
                        params.append((path + ".bn.bias", (b.oc,)))
                        buffers += [(path + ".bn.running_mean", (b.oc,)), (path + ".bn.running_var", (b.oc,)),
                                    (path + ".bn.num_batches_tracked", ())]
    out = []
    for kind, items in ((0, params), (1, buffers)):
        for name, shape in items:
            out.append(dict(index=len(out), name=name, kind=kind, shape=shape,
                            numel=int(np.prod(shape, dtype=np.int64))))
    return out


def initial_head_state(cfg: sy.Config, seed: int):
    """data.head_params for `cfg` without a session: (tensors, params, buffers)."""
    from types import SimpleNamespace

    from simdyolo_b200 import data
    tensors = snapshot_tensors(cfg)
    params, buffers = data.head_params(SimpleNamespace(config=cfg, tensors=tensors), seed)
    return tensors, params, buffers


def tf32_rna(t):
    """Round a float64 torch tensor to float32, then to the nearest TF32 value (10 mantissa bits, ties away
    from zero): the rounding cvt.rna.tf32.f32 applies to every tensor-core operand in TF32 mode."""
    import torch
    f = t.to(torch.float32).contiguous()
    bits = f.view(torch.int32)
    r = torch.bitwise_and(bits + 0x1000, ~0x1FFF)
    return r.view(torch.float32).to(torch.float64)


def _tf32_conv():
    import torch
    import torch.nn.functional as F

    class Tf32Conv(torch.autograd.Function):
        """conv2d in float64 whose operands are TF32-rounded in the forward (input, weight) and in both
        backward GEMMs (output gradient and weight for the data gradient, input and output gradient for the
        weight gradient), as the TF32 tensor-core path stores them.  `center` applies the first-conv
        weight-gradient identity with the exact zero total: the input is centred per channel before the
        rounding and mean * (-edge strip sums of dy) is added back."""

        @staticmethod
        def forward(ctx, x, w, pad, center):
            ctx.save_for_backward(x, w)
            ctx.pad, ctx.center = pad, center
            return F.conv2d(tf32_rna(x), tf32_rna(w), padding=pad)

        @staticmethod
        def backward(ctx, dy):
            x, w = ctx.saved_tensors
            dyr = tf32_rna(dy)
            dx = torch.nn.grad.conv2d_input(x.shape, tf32_rna(w), dyr, padding=ctx.pad)
            if not ctx.center:
                dw = torch.nn.grad.conv2d_weight(tf32_rna(x), w.shape, dyr, padding=ctx.pad)
            else:
                mu = x.mean((2, 3), keepdim=True)
                dw = torch.nn.grad.conv2d_weight(tf32_rna(x - mu), w.shape, dyr, padding=ctx.pad)
                k = w.shape[-1]
                H, W = dy.shape[2], dy.shape[3]
                # T[t][o] = -(sum of dy over the pixels whose tap-t source leaves the map)
                T = torch.zeros(dy.shape[1], k, k, dtype=dy.dtype)
                for ky in range(k):
                    for kx in range(k):
                        sy_, sx = ky - k // 2, kx - k // 2
                        mask = torch.zeros(H, W, dtype=torch.bool)
                        if sy_ < 0:
                            mask[:-sy_, :] = True
                        if sy_ > 0:
                            mask[H - sy_:, :] = True
                        if sx < 0:
                            mask[:, :-sx] = True
                        if sx > 0:
                            mask[:, W - sx:] = True
                        T[:, ky, kx] = -(dyr[0][:, mask].sum(-1))
                dw = dw + mu[0, :, 0, 0][None, :, None, None] * T[:, None, :, :]
            return dx, dw, None, None

    return Tf32Conv


def head_gradient_emulated(cfg: sy.Config, tensors, params, features, truth, tf32: bool, center_first: bool = True):
    """The head gradient of one step in float64: per image the head forward with training BatchNorm
    (HeadOperations.cs:158-166) and the backward by torch autograd, fed with the oracle's DetectionLoss
    gradient (DetectionLoss.cs:19-149, float32, evaluated on the float64 outputs rounded to float32),
    summed over images.  With `tf32`, every conv of the head is evaluated like the TF32 tensor-core path
    (operands rounded to TF32 in the forward and both backward GEMMs; with `center_first` the first conv
    of each branch uses the centred weight gradient).  Returns (gradient, positives)."""
    import torch
    import torch.nn.functional as F
    assert not cfg.end_to_end
    conv = _tf32_conv() if tf32 else None
    names = [t for t in tensors if t["kind"] == 0]
    total = np.zeros(sum(t["numel"] for t in names), np.float64)
    positives = 0
    for b in range(features[0].shape[0]):
        ts, off = {}, 0
        for t in names:
            ts[t["name"]] = torch.tensor(params[off:off + t["numel"]].astype(np.float64).reshape(t["shape"]),
                                         requires_grad=True)
            off += t["numel"]
        outs = {}
        for box in (True, False):
            for lvl in range(3):
                prefix = ("cv2" if box else "cv3") + f".{lvl}"
                n = cfg.n_box_blocks if box else cfg.n_cls_blocks
                blocks = cfg.box_blocks[lvl] if box else cfg.cls_blocks[lvl]
                x = torch.tensor(features[lvl][b].astype(np.float64))[None]
                if tf32:
                    x = tf32_rna(x)
                for i in range(n):
                    blk = blocks[i]
                    assert blk.groups == 1
                    path = f"{prefix}.{_block_path(i, n)}"
                    cname = path + (".conv" if blk.has_bn else "")
                    if tf32:
                        x = conv.apply(x, ts[cname + ".weight"], blk.k // 2, center_first and i == 0 and bool(blk.has_bn))
                        if cname + ".bias" in ts:
                            x = x + ts[cname + ".bias"][None, :, None, None]
                    else:
                        x = F.conv2d(x, ts[cname + ".weight"], ts.get(cname + ".bias"), padding=blk.k // 2)
                    if blk.has_bn:
                        mean = x.mean((0, 2, 3))
                        var = x.var((0, 2, 3), unbiased=False)
                        x = (x - mean[None, :, None, None]) / torch.sqrt(var[None, :, None, None] + cfg.bn_eps)
                        x = x * ts[path + ".bn.weight"][None, :, None, None] + ts[path + ".bn.bias"][None, :, None, None]
                        x = F.silu(x)
                outs[(box, lvl)] = x[0]
        bl = [outs[(True, l)].detach().numpy().astype(np.float32) for l in range(3)]
        cl = [outs[(False, l)].detach().numpy().astype(np.float32) for l in range(3)]
        part, db, dc, _, _ = O.detection_loss(bl, cl, [8.0, 16.0, 32.0], truth[b], cfg.num_classes, bins=cfg.reg_max)
        positives += part["positives"]
        pairs = [(outs[(True, l)], torch.tensor(db[l].astype(np.float64))) for l in range(3)]
        pairs += [(outs[(False, l)], torch.tensor(dc[l].astype(np.float64))) for l in range(3)]
        torch.autograd.backward([o for o, _ in pairs], [g for _, g in pairs])
        total += np.concatenate([ts[t["name"]].grad.numpy().ravel() if ts[t["name"]].grad is not None
                                 else np.zeros(t["numel"]) for t in names])
    return total, positives


def f64_head_gradient(cfg: sy.Config, tensors, params, features, truth):
    """head_gradient_emulated without TF32 rounding: the exact (float64) head gradient of one step given
    the oracle's loss gradient.  Sums that cancel heavily (the first conv of every branch reads trunk
    features with a large per-channel mean against a zero-mean BatchNorm gradient) carry FP32 rounding
    of about 1e-5 in any FP32 evaluation order; this one has none, so FP32 implementations can be compared
    by their distance from it."""
    return head_gradient_emulated(cfg, tensors, params, features, truth, tf32=False)
