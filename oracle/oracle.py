"""ctypes bindings for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` as the checker and by
``bench.py``'s cpu_baseline / ``--impl reference`` legs.  The product package never imports it.
See ``oracle/syo.h`` for which reference file each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class Box(C.Structure):
    _fields_ = [("cls", C.c_int32), ("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float)]


class Loss(C.Structure):
    _fields_ = [("box", C.c_float), ("cls", C.c_float), ("dfl", C.c_float), ("positives", C.c_int32),
                ("connected", C.c_int32)]


class Block(C.Structure):
    _fields_ = [("ic", C.c_int32), ("oc", C.c_int32), ("k", C.c_int32), ("groups", C.c_int32),
                ("has_bn", C.c_int32), ("has_bias", C.c_int32)]


class HeadDesc(C.Structure):
    _fields_ = [("levels", C.c_int32), ("nc", C.c_int32), ("bins", C.c_int32), ("hs", C.c_int32 * 3),
                ("ws", C.c_int32 * 3), ("strides", C.c_float * 3), ("n_box_blocks", C.c_int32),
                ("n_cls_blocks", C.c_int32), ("box_blocks", (Block * 8) * 3), ("cls_blocks", (Block * 8) * 3),
                ("bn_eps", C.c_float), ("bn_momentum", C.c_float), ("end_to_end", C.c_int32),
                ("epoch", C.c_int32), ("schedule_epochs", C.c_int32)]


class BackboneDesc(C.Structure):
    _fields_ = [("image", C.c_int32), ("width_mult", C.c_float), ("depth_mult", C.c_float),
                ("max_channels", C.c_int32), ("family", C.c_int32)]


class Optim(C.Structure):
    _fields_ = [("lr", C.c_float), ("momentum", C.c_float), ("weight_decay", C.c_float), ("optimizer", C.c_int32),
                ("beta1", C.c_float), ("beta2", C.c_float), ("adam_eps", C.c_float), ("adam_step", C.c_int32 * 3)]


class StepResult(C.Structure):
    _fields_ = [("box", C.c_double), ("cls", C.c_double), ("dfl", C.c_double), ("positives", C.c_int64),
                ("box_has_grad", C.c_int32), ("status", C.c_int32)]


class Detection(C.Structure):
    _fields_ = [("class_id", C.c_int32), ("confidence", C.c_float), ("x", C.c_float), ("y", C.c_float),
                ("width", C.c_float), ("height", C.c_float)]


class Letterbox(C.Structure):
    _fields_ = [("source_width", C.c_int32), ("source_height", C.c_int32), ("target_width", C.c_int32),
                ("target_height", C.c_int32), ("scale_x", C.c_float), ("scale_y", C.c_float), ("pad_x", C.c_int32),
                ("pad_y", C.c_int32)]


class DetectOptions(C.Structure):
    _fields_ = [("confidence", C.c_float), ("iou_threshold", C.c_float), ("max_detections", C.c_int32),
                ("max_candidates", C.c_int32), ("class_agnostic", C.c_int32)]


def build() -> None:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        fp, ip, vp = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.c_void_p
        L.syo_expf.argtypes = [C.c_float]; L.syo_expf.restype = C.c_float
        L.syo_atanf.argtypes = [C.c_float]; L.syo_atanf.restype = C.c_float
        L.syo_sigmoid.argtypes = [C.c_float]; L.syo_sigmoid.restype = C.c_float
        L.syo_pow6.argtypes = [C.c_float]; L.syo_pow6.restype = C.c_float
        L.syo_conv_forward.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int, C.c_int, vp, F32P]
        L.syo_conv_backward.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int, C.c_int, F32P, F32P, vp, vp]
        L.syo_grouped_conv_forward.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int, C.c_int, C.c_int, vp, F32P]
        L.syo_grouped_conv_backward.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int, C.c_int, C.c_int, F32P,
                                                F32P, vp, vp]
        L.syo_batchnorm_forward.argtypes = [F32P, C.c_int, C.c_int, F32P, F32P, F32P, F32P, C.c_float, C.c_float, C.c_int,
                                            F32P, F32P, F32P, vp, vp]
        L.syo_batchnorm_backward.argtypes = [F32P, F32P, F32P, F32P, C.c_int, C.c_int, F32P, F32P, F32P]
        L.syo_silu_forward.argtypes = [F32P, C.c_int, F32P, F32P]
        L.syo_silu_backward.argtypes = [F32P, F32P, F32P, C.c_int, F32P]
        L.syo_right_transposed.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int, C.c_int]
        L.syo_all_finite.argtypes = [F32P, C.c_long]; L.syo_all_finite.restype = C.c_int
        L.syo_sgd_update.argtypes = [F32P, F32P, F32P, C.c_long, C.c_float, C.c_float, C.c_float, C.c_int, C.c_int]
        L.syo_sgd_update.restype = C.c_int
        L.syo_adamw_update.argtypes = [F32P, F32P, F32P, F32P, C.c_long, C.c_float, C.c_float, C.c_float, C.c_float,
                                       C.c_float, C.c_int, C.c_int, C.c_int]
        L.syo_adamw_update.restype = C.c_int
        L.syo_progressive_weight.argtypes = [C.c_int, C.c_int]; L.syo_progressive_weight.restype = C.c_float
        L.syo_detection_loss.argtypes = [C.POINTER(vp), C.POINTER(vp), ip, ip, fp, C.c_int, C.c_int, C.c_int,
                                         C.POINTER(Box), C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                         C.POINTER(vp), C.POINTER(vp), C.POINTER(Loss), vp, vp]
        L.syo_detection_loss.restype = C.c_int
        L.syo_ciou.argtypes = [fp, fp, fp]; L.syo_ciou.restype = C.c_float
        L.syo_head_eval_image.argtypes = [C.POINTER(HeadDesc), F32P, F32P, C.POINTER(vp), C.POINTER(Box), C.c_int,
                                          C.POINTER(Loss)]
        L.syo_head_eval_image.restype = C.c_int
        L.syo_head_param_count.argtypes = [C.POINTER(HeadDesc)]; L.syo_head_param_count.restype = C.c_long
        L.syo_head_buffer_count.argtypes = [C.POINTER(HeadDesc)]; L.syo_head_buffer_count.restype = C.c_long
        L.syo_head_image.argtypes = [C.POINTER(HeadDesc), F32P, F32P, C.POINTER(vp), C.POINTER(Box), C.c_int, F32P,
                                     C.POINTER(Loss), C.c_int, ip]
        L.syo_head_image.restype = C.c_int
        L.syo_backbone_param_count.argtypes = [C.POINTER(BackboneDesc)]; L.syo_backbone_param_count.restype = C.c_long
        L.syo_backbone_feature_channels.argtypes = [C.POINTER(BackboneDesc), ip]
        L.syo_backbone_forward.argtypes = [C.POINTER(BackboneDesc), F32P, C.POINTER(C.c_uint8), F32P, F32P, F32P]
        L.syo_train_step.argtypes = [C.POINTER(BackboneDesc), F32P, C.POINTER(HeadDesc), F32P, F32P, F32P, F32P,
                                     C.POINTER(Optim), C.POINTER(vp), C.POINTER(Box), I32P, C.c_int, C.c_int, vp,
                                     C.POINTER(StepResult)]
        L.syo_head_eval_outputs.argtypes = [C.POINTER(HeadDesc), F32P, F32P, C.POINTER(vp), C.c_int,
                                            C.POINTER(vp), C.POINTER(vp)]
        L.syo_head_eval_outputs.restype = C.c_int
        L.syo_head_decode.argtypes = [F32P, F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                                      F32P, C.c_int, C.c_int]
        L.syo_end_to_end_topk.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, F32P]
        L.syo_end_to_end_topk.restype = C.c_int
        L.syo_decode_detections.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Letterbox),
                                            C.POINTER(DetectOptions), C.POINTER(Detection)]
        L.syo_decode_detections.restype = C.c_int
        L.syo_detection_iou.argtypes = [C.POINTER(Detection), C.POINTER(Detection)]
        L.syo_detection_iou.restype = C.c_float
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- operators (one image, NCHW)

def conv_forward(x, w, bias=None):
    x, w = _f32(x), _f32(w)
    ic, h, wd = x.shape
    oc, _, k, _ = w.shape
    y = np.zeros((oc, h, wd), np.float32)
    b = None if bias is None else _f32(bias)
    lib().syo_conv_forward(x, ic, h, wd, w, oc, k, _ptr(b), y)
    return y


def conv_backward(x, w, dy, with_bias=False, with_dx=True):
    x, w, dy = _f32(x), _f32(w), _f32(dy)
    ic, h, wd = x.shape
    oc, _, k, _ = w.shape
    dw = np.zeros_like(w)
    db = np.zeros(oc, np.float32) if with_bias else None
    dx = np.zeros_like(x) if with_dx else None
    lib().syo_conv_backward(x, ic, h, wd, w, oc, k, dy, dw, _ptr(db), _ptr(dx))
    return dw, db, dx


def grouped_conv_forward(x, w, groups, bias=None):
    x, w = _f32(x), _f32(w)
    ic, h, wd = x.shape
    oc, _, k, _ = w.shape
    y = np.zeros((oc, h, wd), np.float32)
    b = None if bias is None else _f32(bias)
    lib().syo_grouped_conv_forward(x, ic, h, wd, w, oc, k, groups, _ptr(b), y)
    return y


def grouped_conv_backward(x, w, groups, dy, with_bias=False, with_dx=True):
    x, w, dy = _f32(x), _f32(w), _f32(dy)
    ic, h, wd = x.shape
    oc, _, k, _ = w.shape
    dw = np.zeros_like(w)
    db = np.zeros(oc, np.float32) if with_bias else None
    dx = np.zeros_like(x) if with_dx else None
    lib().syo_grouped_conv_backward(x, ic, h, wd, w, oc, k, groups, dy, dw, _ptr(db), _ptr(dx))
    return dw, db, dx


def batchnorm_forward(x, gamma, beta, rmean, rvar, eps=1e-3, momentum=0.03, training=True):
    x = _f32(x)
    c = x.shape[0]
    sp = int(np.prod(x.shape[1:]))
    y, xhat, inv = np.zeros_like(x), np.zeros_like(x), np.zeros(c, np.float32)
    bm, bv = np.zeros(c, np.float32), np.zeros(c, np.float32)
    lib().syo_batchnorm_forward(x, c, sp, _f32(gamma), _f32(beta), rmean, rvar, eps, momentum, int(training), y, xhat,
                                inv, _ptr(bm), _ptr(bv))
    return y, xhat, inv, bm, bv


def batchnorm_backward(dy, xhat, inv, gamma):
    dy = _f32(dy)
    c = dy.shape[0]
    sp = int(np.prod(dy.shape[1:]))
    dg, dbt, dx = np.zeros(c, np.float32), np.zeros(c, np.float32), np.zeros_like(dy)
    lib().syo_batchnorm_backward(dy, _f32(xhat), _f32(inv), _f32(gamma), c, sp, dg, dbt, dx)
    return dg, dbt, dx


def silu_forward(x):
    x = _f32(x)
    y, s = np.zeros_like(x), np.zeros_like(x)
    lib().syo_silu_forward(x.ravel(), x.size, y.ravel(), s.ravel())
    return y, s


def silu_backward(x, sig, dy):
    x = _f32(x)
    dx = np.zeros_like(x)
    lib().syo_silu_backward(x.ravel(), _f32(sig).ravel(), _f32(dy).ravel(), x.size, dx.ravel())
    return dx


def right_transposed(a, b):
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    lib().syo_right_transposed(a, b, c, m, n, k)
    return c


def sgd_update(w, v, g, lr, momentum, wd, images, has_grad=True):
    """In place on float32 arrays; returns status (0 ok, 1 non-finite)."""
    return lib().syo_sgd_update(w, v, g, w.size, lr, momentum, wd, images, int(has_grad))


def boxes(truth):
    arr = (Box * max(1, len(truth)))()
    for i, (c, x1, y1, x2, y2) in enumerate(truth):
        arr[i] = Box(int(c), float(x1), float(y1), float(x2), float(y2))
    return arr


def detection_loss(box_levels, cls_levels, strides, truth, nc, bins=16, topk=10, topk2=10, grad_scale=1.0,
                   backward=True):
    """DetectionLoss.Compute for one image.  box_levels[l]: [4*bins, H, W]; cls_levels[l]: [nc, H, W].
    Returns (loss dict, dbox list, dcls list, assigned[A], scores[A])."""
    L = lib()
    n = len(box_levels)
    bl = [_f32(b) for b in box_levels]
    cl = [_f32(c) for c in cls_levels]
    hs = np.array([b.shape[1] for b in bl], np.int32)
    ws = np.array([b.shape[2] for b in bl], np.int32)
    st = np.array(strides, np.float32)
    db = [np.zeros_like(b) for b in bl]
    dc = [np.zeros_like(c) for c in cl]
    A = int((hs * ws).sum())
    assigned = np.zeros(A, np.int32)
    scores = np.zeros(A, np.float32)
    VP = C.c_void_p * n
    out = Loss()
    tb = boxes(truth)
    rc = L.syo_detection_loss(VP(*[_ptr(b) for b in bl]), VP(*[_ptr(c) for c in cl]),
                              hs.ctypes.data_as(C.POINTER(C.c_int32)), ws.ctypes.data_as(C.POINTER(C.c_int32)),
                              st.ctypes.data_as(C.POINTER(C.c_float)), n, nc, bins, tb, len(truth), topk, topk2,
                              grad_scale, int(backward), VP(*[_ptr(b) for b in db]), VP(*[_ptr(c) for c in dc]),
                              C.byref(out), _ptr(assigned), _ptr(scores))
    if rc != 0:
        raise ValueError("oracle detection_loss rejected its arguments")
    loss = dict(box=out.box, cls=out.cls, dfl=out.dfl, positives=out.positives, connected=out.connected)
    return loss, db, dc, assigned, scores


def ciou(p, t):
    p, t = _f32(p), _f32(t)
    g = np.zeros(4, np.float32)
    v = lib().syo_ciou(p.ctypes.data_as(C.POINTER(C.c_float)), t.ctypes.data_as(C.POINTER(C.c_float)),
                       g.ctypes.data_as(C.POINTER(C.c_float)))
    return v, g


# ---------------------------------------------------------------- detection post-processing

def head_decode(levels, bins, nc, xyxy=False):
    """CpuHead.DecodeInto over joined levels: levels = [(box [B][4*bins][h][w], cls [B][nc][h][w], stride)].
    Returns [B][nc + 4][anchors] float32."""
    batch = levels[0][0].shape[0]
    anchors = sum(b.shape[2] * b.shape[3] for b, _, _ in levels)
    out = np.zeros((batch, nc + 4, anchors), np.float32)
    start = 0
    for box, cls, stride in levels:
        box, cls = _f32(box), _f32(cls)
        h, w = box.shape[2], box.shape[3]
        lib().syo_head_decode(box, cls, batch, h, w, bins, nc, stride, int(xyxy), out, anchors, start)
        start += h * w
    return out


def end_to_end_topk(x, nc, maximum=300):
    """PtModel.EndToEndTopK: x [B][fields][anchors] -> [B][min(maximum, anchors)][6 + extra]."""
    x = _f32(x)
    batch, fields, anchors = x.shape
    k = min(maximum, anchors)
    out = np.zeros((batch, k, 6 + fields - nc - 4), np.float32)
    assert lib().syo_end_to_end_topk(x, batch, fields, anchors, nc, maximum, out) == k
    return out


def decode_detections(output, layout, class_count=0, letterbox=None, confidence=0.25, iou_threshold=0.45,
                      max_detections=300, max_candidates=30000, class_agnostic=False):
    """YoloDetector.DecodeIndexed on one image's output [dim1][dim2]; layout 1 channels-first, 2 channels-last,
    3 end-to-end.  Returns a list of (class_id, confidence, x, y, width, height) in output order."""
    output = _f32(output)
    dim1, dim2 = output.shape
    if letterbox is None:
        letterbox = Letterbox(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1.0, 1.0, 0, 0)
    opt = DetectOptions(confidence, iou_threshold, max_detections, max_candidates, int(class_agnostic))
    out = (Detection * max_detections)()
    n = lib().syo_decode_detections(output, dim1, dim2, layout, class_count, C.byref(letterbox), C.byref(opt), out)
    if n < 0:
        raise ValueError(f"syo_decode_detections: {n}")
    return [(d.class_id, d.confidence, d.x, d.y, d.width, d.height) for d in out[:n]]
