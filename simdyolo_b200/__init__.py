"""simdyolo_b200: B200-native detection-head fine-tuning step behind a C ABI.

The CUDA library (libsimdyolo_cuda.so, built from csrc/ for sm_100a) implements the hot path of
SimdYolo.Training (YoloTrainer's batch loop: frozen backbone forward, Detect head forward/backward,
DFL + CIoU + BCE loss with the task-aligned assigner, SGD-momentum / AdamW, NCCL all-reduce).
This module is the Python mirror of the reference's host API over that ABI (ctypes), used by the
tests and bench.py.  There is no CPU fallback: every compute call goes to the CUDA library.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsimdyolo_cuda.so")

SY_OK = 0
SY_ERR_INVALID_ARGUMENT = 1
SY_ERR_UNSUPPORTED_SHAPE = 2
SY_ERR_NONFINITE = 3
SY_ERR_COMM = 4
SY_ERR_DEVICE = 5
SY_ERR_OUT_OF_MEMORY = 6
SY_OPT_SGD = 0
SY_OPT_ADAMW = 1
SY_PRECISION_TF32 = 0
SY_PRECISION_3XTF32 = 1
SY_BACKBONE_NONE = 0
SY_BACKBONE_YOLOV8 = 1
SY_BACKBONE_YOLO11 = 2


class SyError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class InvalidArgument(SyError, ValueError):
    """ArgumentException in the reference."""


class UnsupportedShape(SyError, NotImplementedError):
    """NotSupportedException in the reference."""


class NonFinite(SyError, ArithmeticError):
    """ArithmeticException in the reference (YoloTrainer.cs:193,196; TrainingParameter.cs:40)."""


def _raise(status: int, message: str):
    cls = {SY_ERR_INVALID_ARGUMENT: InvalidArgument, SY_ERR_UNSUPPORTED_SHAPE: UnsupportedShape,
           SY_ERR_NONFINITE: NonFinite}.get(status, SyError)
    raise cls(status, message)


class Box(C.Structure):
    _fields_ = [("class_id", C.c_int32), ("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float)]


class Block(C.Structure):
    _fields_ = [("ic", C.c_int32), ("oc", C.c_int32), ("k", C.c_int32), ("groups", C.c_int32),
                ("has_bn", C.c_int32), ("has_bias", C.c_int32)]


class Config(C.Structure):
    _fields_ = [("struct_size", C.c_int32), ("device", C.c_int32), ("rank", C.c_int32), ("world_size", C.c_int32),
                ("nccl_id", C.c_uint8 * 128), ("image_size", C.c_int32), ("max_batch", C.c_int32),
                ("max_boxes", C.c_int32), ("num_classes", C.c_int32), ("reg_max", C.c_int32),
                ("backbone", C.c_int32), ("width_mult", C.c_float), ("depth_mult", C.c_float),
                ("max_channels", C.c_int32), ("feature_channels", C.c_int32 * 3), ("n_box_blocks", C.c_int32),
                ("n_cls_blocks", C.c_int32), ("box_blocks", (Block * 8) * 3), ("cls_blocks", (Block * 8) * 3),
                ("bn_eps", C.c_float), ("bn_momentum", C.c_float), ("optimizer", C.c_int32), ("lr", C.c_float),
                ("momentum", C.c_float), ("weight_decay", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("adam_eps", C.c_float), ("precision", C.c_int32), ("end_to_end", C.c_int32),
                ("schedule_epochs", C.c_int32), ("comm_timeout_ms", C.c_int32)]


class StepStats(C.Structure):
    _fields_ = [("box", C.c_double), ("cls", C.c_double), ("dfl", C.c_double), ("positives", C.c_int64),
                ("images", C.c_int32), ("box_has_grad", C.c_int32), ("grad_checksum", C.c_double),
                ("device_ms", C.c_double), ("near_ties", C.c_int64)]


class Detection(C.Structure):
    """Detection (YoloDetector.cs:139): class, confidence, top-left corner and size in source pixels."""
    _fields_ = [("class_id", C.c_int32), ("confidence", C.c_float), ("x", C.c_float), ("y", C.c_float),
                ("width", C.c_float), ("height", C.c_float)]


class Letterbox(C.Structure):
    """Letterbox (YoloDetector.cs:149): x_source = (x_model - pad_x) / scale_x, clamped to the source."""
    _fields_ = [("source_width", C.c_int32), ("source_height", C.c_int32), ("target_width", C.c_int32),
                ("target_height", C.c_int32), ("scale_x", C.c_float), ("scale_y", C.c_float), ("pad_x", C.c_int32),
                ("pad_y", C.c_int32)]


class DetectOptions(C.Structure):
    """DetectorOptions' decode fields (YoloDetector.cs:88-105)."""
    _fields_ = [("confidence", C.c_float), ("iou_threshold", C.c_float), ("max_detections", C.c_int32),
                ("max_candidates", C.c_int32), ("class_agnostic", C.c_int32)]


SY_LAYOUT_AUTO, SY_LAYOUT_CHANNELS_FIRST, SY_LAYOUT_CHANNELS_LAST, SY_LAYOUT_END_TO_END = 0, 1, 2, 3


def detect_options(confidence: float = 0.25, iou_threshold: float = 0.45, max_detections: int = 300,
                   max_candidates: int = 30000, class_agnostic: bool = False) -> DetectOptions:
    """DetectorOptions defaults (YoloDetector.cs:92-104)."""
    return DetectOptions(confidence, iou_threshold, max_detections, max_candidates, int(class_agnostic))


def evaluation_options() -> DetectOptions:
    """The detector settings of DetectionEvaluator.Evaluate (DetectionEvaluator.cs:50-51)."""
    return detect_options(0.001, 0.7, 300)


_DETECTION_DTYPE = np.dtype([("class_id", "<i4"), ("confidence", "<f4"), ("x", "<f4"), ("y", "<f4"),
                             ("width", "<f4"), ("height", "<f4")])


def _detections(out, counts, max_det):
    """Per image a list of (class_id, confidence, x, y, width, height) from the [images][max_det] records."""
    arr = np.frombuffer(out, _DETECTION_DTYPE).reshape(len(counts), max_det)
    return [arr[b, :int(n)].tolist() for b, n in enumerate(counts)]


class TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char * 96), ("kind", C.c_int32), ("rank", C.c_int32), ("shape", C.c_int32 * 4),
                ("numel", C.c_int64)]


_lib = None


def lib():
    """Load the CUDA library; fails loudly when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m simdyolo_b200.build`")
        L = C.CDLL(LIB_PATH)
        vp, fp, ip = C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int32)
        st = C.c_int32
        L.sy_cuda_last_error.restype = C.c_char_p
        L.sy_cuda_last_error.argtypes = [vp]
        L.sy_cuda_nccl_unique_id.argtypes = [C.POINTER(C.c_uint8)]
        L.sy_cuda_create.argtypes = [C.POINTER(Config), C.POINTER(vp)]
        L.sy_cuda_destroy.argtypes = [vp]
        L.sy_cuda_tensor_count.argtypes = [vp]
        L.sy_cuda_tensor_count.restype = C.c_int32
        L.sy_cuda_tensor_info.argtypes = [vp, C.c_int32, C.POINTER(TensorInfo)]
        for name in ("sy_cuda_set_tensor", "sy_cuda_get_tensor"):
            getattr(L, name).argtypes = [vp, C.c_int32, fp, C.c_int64]
        for name in ("sy_cuda_set_optimizer_state", "sy_cuda_get_optimizer_state"):
            getattr(L, name).argtypes = [vp, C.c_int32, C.c_int32, fp, C.c_int64]
        L.sy_cuda_backbone_param_count.argtypes = [vp]
        L.sy_cuda_backbone_param_count.restype = C.c_int64
        L.sy_cuda_set_backbone.argtypes = [vp, fp, C.c_int64]
        L.sy_cuda_step.argtypes = [vp, C.POINTER(C.c_uint8), C.POINTER(Box), ip, C.c_int32, C.POINTER(StepStats)]
        L.sy_cuda_eval_loss.argtypes = L.sy_cuda_step.argtypes
        L.sy_cuda_step_features.argtypes = [vp, C.POINTER(fp), C.POINTER(Box), ip, C.c_int32, C.POINTER(StepStats)]
        L.sy_cuda_eval_loss_features.argtypes = L.sy_cuda_step_features.argtypes
        L.sy_cuda_get_last_gradients.argtypes = [vp, fp, C.c_int64]
        L.sy_cuda_get_optimizer_steps.argtypes = [vp, ip]
        L.sy_cuda_set_optimizer_steps.argtypes = [vp, ip]
        L.sy_cuda_wait_limit_selftest.argtypes = [C.c_int32, C.c_int32, ip]
        L.sy_cuda_set_epoch.argtypes = [vp, C.c_int32]
        L.sy_cuda_get_last_features.argtypes = [vp, C.c_int32, fp, C.c_int64]
        L.sy_cuda_detection_loss.argtypes = [C.c_int32, C.c_int32, C.c_int32, ip, ip, fp, C.c_int32, C.c_int32,
                                             C.POINTER(fp), C.POINTER(fp), C.POINTER(Box), ip, fp, ip, ip, fp,
                                             C.POINTER(fp), C.POINTER(fp)]
        L.sy_cuda_detection_loss_ex.argtypes = [C.c_int32, C.c_int32, C.c_int32, ip, ip, fp, C.c_int32, C.c_int32,
                                                C.POINTER(fp), C.POINTER(fp), C.POINTER(Box), ip, C.c_int32, C.c_int32,
                                                C.c_float, fp, ip, ip, fp, C.POINTER(fp), C.POINTER(fp)]
        L.sy_cuda_conv2d_forward.argtypes = [C.c_int32, fp, C.c_int32, C.c_int32, C.c_int32, C.c_int32, fp, C.c_int32,
                                             C.c_int32, fp, fp]
        L.sy_cuda_conv2d_backward_data.argtypes = [C.c_int32, fp, C.c_int32, C.c_int32, C.c_int32, C.c_int32, fp,
                                                   C.c_int32, C.c_int32, fp]
        L.sy_cuda_conv2d_backward_filter.argtypes = [C.c_int32, fp, fp, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                     C.c_int32, C.c_int32, fp]
        L.sy_cuda_matmul.argtypes = [C.c_int32, fp, fp, fp, C.c_int32, C.c_int32, C.c_int32]
        L.sy_cuda_sgd_update.argtypes = [C.c_int32, fp, fp, fp, C.c_int64, C.c_float, C.c_float, C.c_float, C.c_int32,
                                         C.c_int32]
        L.sy_cuda_conv2d_backward_filter_static.argtypes = [C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32,
                                                            C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                                            C.c_void_p]
        L.sy_cuda_step_device.argtypes = [vp, C.c_void_p, C.POINTER(Box), ip, C.c_int32, C.POINTER(StepStats)]
        L.sy_cuda_prefetch_images.argtypes = [vp, C.POINTER(C.c_uint8), C.c_int32]
        L.sy_cuda_launch_count.argtypes = []
        L.sy_cuda_launch_count.restype = C.c_int64
        L.sy_cuda_bench_conv.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                         C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_double)]
        L.sy_cuda_conv_profile.argtypes = [vp, st, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                           C.POINTER(C.c_int64)]
        L.sy_cuda_conv_profile_launches.argtypes = [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), ip, st,
                                                    C.POINTER(C.c_int32)]
        dp, lp, op = C.POINTER(Detection), C.POINTER(Letterbox), C.POINTER(DetectOptions)
        dbl = C.POINTER(C.c_double)
        L.sy_cuda_detect.argtypes = [vp, C.POINTER(C.c_uint8), C.c_int32, lp, op, dp, ip, dbl]
        L.sy_cuda_detect_features.argtypes = [vp, C.POINTER(fp), C.c_int32, lp, op, dp, ip, dbl]
        L.sy_cuda_get_last_head_outputs.argtypes = [vp, C.c_int32, C.c_int32, fp, C.c_int64, fp, C.c_int64]
        L.sy_cuda_head_decode.argtypes = [C.c_int32, C.c_int32, C.c_int32, ip, ip, fp, C.c_int32, C.c_int32,
                                          C.c_int32, C.POINTER(fp), C.POINTER(fp), fp]
        L.sy_cuda_end_to_end_topk.argtypes = [C.c_int32, fp, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                              fp]
        L.sy_cuda_decode_detections.argtypes = [C.c_int32, fp, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                C.c_int32, lp, op, dp, ip]
        _lib = L
    return _lib


EXPORTED = ["sy_cuda_nccl_unique_id", "sy_cuda_create", "sy_cuda_destroy", "sy_cuda_last_error",
            "sy_cuda_tensor_count", "sy_cuda_tensor_info", "sy_cuda_set_tensor", "sy_cuda_get_tensor",
            "sy_cuda_set_optimizer_state", "sy_cuda_get_optimizer_state", "sy_cuda_backbone_param_count",
            "sy_cuda_set_backbone", "sy_cuda_step", "sy_cuda_step_features", "sy_cuda_get_last_gradients",
            "sy_cuda_get_last_features", "sy_cuda_detection_loss", "sy_cuda_conv2d_forward",
            "sy_cuda_conv2d_backward_data", "sy_cuda_conv2d_backward_filter", "sy_cuda_matmul", "sy_cuda_sgd_update",
            "sy_cuda_step_device", "sy_cuda_launch_count", "sy_cuda_bench_conv",
            "sy_cuda_conv2d_backward_filter_static", "sy_cuda_conv_profile", "sy_cuda_eval_loss",
            "sy_cuda_eval_loss_features", "sy_cuda_detection_loss_ex", "sy_cuda_set_epoch",
            "sy_cuda_conv_profile_launches", "sy_cuda_get_optimizer_steps", "sy_cuda_set_optimizer_steps",
            "sy_cuda_wait_limit_selftest", "sy_cuda_detect", "sy_cuda_detect_features",
            "sy_cuda_get_last_head_outputs", "sy_cuda_head_decode", "sy_cuda_end_to_end_topk",
            "sy_cuda_decode_detections", "sy_cuda_prefetch_images"]


def _check(status: int, session=None):
    if status != SY_OK:
        msg = lib().sy_cuda_last_error(session)
        _raise(status, msg.decode() if msg else "")


def _fp(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _ip(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


# ------------------------------------------------------------------ model description

def _make_div8(x: float) -> int:
    return int(np.ceil(np.float32(x) / np.float32(8.0))) * 8


def yolov8_channels(width: float, max_channels: int):
    ch = lambda c: _make_div8(np.float32(min(c, max_channels)) * np.float32(width))
    return ch(256), ch(512), ch(1024)


def yolov8_backbone_convs(width: float, depth: float, max_channels: int):
    """(oc, ic, k) of every conv of the YOLOv8 trunk in parameter order (weights then bias)."""
    ch = lambda c: _make_div8(np.float32(min(c, max_channels)) * np.float32(width))
    dep = lambda n: max(int(np.floor(n * depth + 0.5)), 1)
    c64, c128, c256, c512, c1024 = ch(64), ch(128), ch(256), ch(512), ch(1024)
    n3, n6 = dep(3), dep(6)
    convs = []

    def conv(ic, oc, k):
        convs.append((oc, ic, k))

    def c2f(c1, c2, n):
        c = c2 // 2
        conv(c1, 2 * c, 1)
        for _ in range(n):
            conv(c, c, 3)
            conv(c, c, 3)
        conv((2 + n) * c, c2, 1)

    conv(3, c64, 3)
    conv(c64, c128, 3)
    c2f(c128, c128, n3)
    conv(c128, c256, 3)
    c2f(c256, c256, n6)
    conv(c256, c512, 3)
    c2f(c512, c512, n6)
    conv(c512, c1024, 3)
    c2f(c1024, c1024, n3)
    conv(c1024, c1024 // 2, 1)
    conv(c1024 // 2 * 4, c1024, 1)
    c2f(c1024 + c512, c512, n3)
    c2f(c512 + c256, c256, n3)
    conv(c256, c256, 3)
    c2f(c256 + c512, c512, n3)
    conv(c512, c512, 3)
    c2f(c512 + c1024, c1024, n3)
    return convs


def yolo11_backbone_convs(width: float, depth: float, max_channels: int):
    """(oc, ic per group, k) of every conv of the YOLO11 trunk in parameter order (weights then bias),
    the order in which the trunk builders take them: C3k2 = cv1, modules, cv2; C3k = cv1, bottlenecks,
    cv2, cv3; Bottleneck = cv1, cv2; C2PSA = cv1, PSABlocks, cv2; PSABlock = attention (qkv, depthwise
    pe, proj), ffn (two 1x1)."""
    ch = lambda c: _make_div8(np.float32(min(c, max_channels)) * np.float32(width))
    n2 = max(int(np.floor(2 * depth + 0.5)), 1)
    c64, c128, c256, c512, c1024 = ch(64), ch(128), ch(256), ch(512), ch(1024)
    convs = []

    def conv(ic, oc, k):
        convs.append((oc, ic, k))

    def bottleneck(c1, c2, e):
        c_ = int(c2 * e)
        conv(c1, c_, 3)
        conv(c_, c2, 3)

    def c3k(c1, c2, n):
        c_ = int(c2 * 0.5)
        conv(c1, c_, 1)
        for _ in range(n):
            bottleneck(c_, c_, 1.0)
        conv(c1, c_, 1)
        conv(2 * c_, c2, 1)

    def c3k2(c1, c2, use_c3k, e):
        c = int(c2 * e)
        conv(c1, 2 * c, 1)
        for _ in range(n2):
            if use_c3k:
                c3k(c, c, 2)
            else:
                bottleneck(c, c, 0.5)
        conv((2 + n2) * c, c2, 1)

    def c2psa(c1):
        c = int(c1 * 0.5)
        heads = max(c // 64, 1)
        hd = c // heads
        kd = int(hd * 0.5)
        conv(c1, 2 * c, 1)
        for _ in range(n2):
            conv(c, c + 2 * kd * heads, 1)   # qkv
            convs.append((c, 1, 3))          # depthwise positional conv
            conv(c, c, 1)                    # proj
            conv(c, 2 * c, 1)                # ffn
            conv(2 * c, c, 1)
        conv(2 * c, c1, 1)

    conv(3, c64, 3)
    conv(c64, c128, 3)
    c3k2(c128, c256, False, 0.25)
    conv(c256, c256, 3)
    c3k2(c256, c512, False, 0.25)
    conv(c512, c512, 3)
    c3k2(c512, c512, True, 0.5)
    conv(c512, c1024, 3)
    c3k2(c1024, c1024, True, 0.5)
    conv(c1024, c1024 // 2, 1)   # SPPF
    conv(c1024 // 2 * 4, c1024, 1)
    c2psa(c1024)
    c3k2(c1024 + c512, c512, False, 0.5)
    c3k2(c512 + c512, c256, False, 0.5)
    conv(c256, c256, 3)
    c3k2(c256 + c512, c512, False, 0.5)
    conv(c512, c512, 3)
    c3k2(c512 + c1024, c1024, True, 0.5)
    return convs


def detect_head_blocks(feature_channels, nc: int, reg_max: int = 16, dw_cls: bool = False):
    """Ultralytics Detect head: cv2 = Conv(c,c2,3), Conv(c2,c2,3), Conv2d(c2,4*reg_max,1) with
    c2 = max(16, ch0/4, 4*reg_max), c3 = max(ch0, min(nc, 100)); cv3 = Conv(c,c3,3), Conv(c3,c3,3),
    Conv2d(c3,nc,1) (YOLOv8), or for YOLO11 (dw_cls) the nested [DWConv(c,c,3), Conv(c,c3,1)],
    [DWConv(c3,c3,3), Conv(c3,c3,1)], Conv2d(c3,nc,1), flattened to five blocks as the reference's
    training schema does (DetectionHead.cs:31-36).  Blocks: (ic, oc, k, groups, has_bn, has_bias)."""
    ch0 = feature_channels[0]
    c2 = max(16, ch0 // 4, 4 * reg_max)
    c3 = max(ch0, min(nc, 100))
    box, cls = [], []
    for c in feature_channels:
        box.append([(c, c2, 3, 1, 1, 0), (c2, c2, 3, 1, 1, 0), (c2, 4 * reg_max, 1, 1, 0, 1)])
        if dw_cls:
            cls.append([(c, c, 3, c, 1, 0), (c, c3, 1, 1, 1, 0), (c3, c3, 3, c3, 1, 0), (c3, c3, 1, 1, 1, 0),
                        (c3, nc, 1, 1, 0, 1)])
        else:
            cls.append([(c, c3, 3, 1, 1, 0), (c3, c3, 3, 1, 1, 0), (c3, nc, 1, 1, 0, 1)])
    return box, cls


MODELS = {
    # name: (width, depth, max_channels)
    "yolov8n": (0.25, 0.33, 1024),
    "yolov8s": (0.50, 0.33, 1024),
    "yolov8l": (1.00, 1.00, 512),
    "yolo11s": (0.50, 0.50, 1024),
}


def tensor_group(name: str) -> int:
    """Optimizer group of a head tensor: 0 class branches (always receive a gradient), 1 cv2, 2
    one2one_cv2 (a box branch receives one only when its loss assigned a positive)."""
    return 1 if name.startswith("cv2.") else 2 if name.startswith("one2one_cv2.") else 0


def model_family(model: str) -> str:
    """'yolo11' (C3k2 / C2PSA trunk, depthwise class branch) or 'yolov8'."""
    return "yolo11" if model.startswith("yolo11") else "yolov8"


def make_config(model: str = "yolov8n", image_size: int = 640, max_batch: int = 8, max_boxes: int = 8,
                num_classes: int = 80, device: int = 0, rank: int = 0, world_size: int = 1, nccl_id: bytes = b"",
                backbone: bool = True, optimizer: int = SY_OPT_SGD, lr: float = 0.01, momentum: float = 0.937,
                weight_decay: float = 5e-4, beta1: float = 0.9, beta2: float = 0.999, adam_eps: float = 1e-8,
                bn_eps: float = 1e-3, bn_momentum: float = 0.03, precision: int = SY_PRECISION_TF32,
                end_to_end: bool = False, reg_max: int = 16, schedule_epochs: int = 100,
                comm_timeout_ms: int = 0) -> Config:
    """Session description for `model`'s trunk and Detect head.  end_to_end adds the one2one_cv2 /
    one2one_cv3 branches (YOLOv10 v10Detect with reg_max 16; YOLO26-style progressive loss with
    reg_max 1, TrainingHeadSchema.cs:17-21); schedule_epochs is the progressive schedule length.
    comm_timeout_ms bounds a data-parallel step's wait for its collectives (0: 300 s)."""
    width, depth, max_ch = MODELS[model]
    feats = yolov8_channels(width, max_ch)
    cfg = Config()
    cfg.struct_size = C.sizeof(Config)
    cfg.device, cfg.rank, cfg.world_size = device, rank, world_size
    for i, b in enumerate(nccl_id[:128]):
        cfg.nccl_id[i] = b
    cfg.image_size, cfg.max_batch, cfg.max_boxes = image_size, max_batch, max_boxes
    cfg.num_classes, cfg.reg_max = num_classes, reg_max
    family = model_family(model)
    cfg.backbone = (SY_BACKBONE_YOLO11 if family == "yolo11" else SY_BACKBONE_YOLOV8) if backbone else SY_BACKBONE_NONE
    cfg.width_mult, cfg.depth_mult, cfg.max_channels = width, depth, max_ch
    for i in range(3):
        cfg.feature_channels[i] = feats[i]
    box, cls = detect_head_blocks(feats, num_classes, reg_max, dw_cls=model_family(model) == "yolo11")
    cfg.n_box_blocks, cfg.n_cls_blocks = len(box[0]), len(cls[0])
    for lvl in range(3):
        for i, b in enumerate(box[lvl]):
            cfg.box_blocks[lvl][i] = Block(*b)
        for i, b in enumerate(cls[lvl]):
            cfg.cls_blocks[lvl][i] = Block(*b)
    cfg.bn_eps, cfg.bn_momentum = bn_eps, bn_momentum
    cfg.optimizer, cfg.lr, cfg.momentum, cfg.weight_decay = optimizer, lr, momentum, weight_decay
    cfg.beta1, cfg.beta2, cfg.adam_eps = beta1, beta2, adam_eps
    cfg.precision = precision
    cfg.end_to_end, cfg.schedule_epochs = int(bool(end_to_end)), schedule_epochs
    cfg.comm_timeout_ms = comm_timeout_ms
    return cfg


# ------------------------------------------------------------------ ground truth

BOX_DTYPE = np.dtype([("class_id", "<i4"), ("x1", "<f4"), ("y1", "<f4"), ("x2", "<f4"), ("y2", "<f4")])


class PackedBoxes:
    """The ground truth of one batch in the C layout (sy_box records, per-image counts), packed once."""

    def __init__(self, records: np.ndarray, counts: np.ndarray):
        self.records = np.ascontiguousarray(records, BOX_DTYPE)
        self.counts = np.ascontiguousarray(counts, np.int32)
        self.pointer = self.records.ctypes.data_as(C.POINTER(Box))


def pack_boxes(boxes_per_image) -> PackedBoxes:
    """Per-image lists of (cls, x1, y1, x2, y2) -> PackedBoxes (TrainingBox records, YoloTrainer's labels)."""
    counts = np.array([len(b) for b in boxes_per_image], np.int32)
    n = int(counts.sum())
    rec = np.zeros(max(1, n), BOX_DTYPE)
    if n:
        flat = np.array([bx for b in boxes_per_image for bx in b], np.float64).reshape(n, 5)
        rec["class_id"][:n] = flat[:, 0].astype(np.int32)
        for k, f in enumerate(("x1", "y1", "x2", "y2")):
            rec[f][:n] = flat[:, k + 1]
    return PackedBoxes(rec, counts)


# ------------------------------------------------------------------ session

class Session:
    """One data-parallel rank of the fine-tuning step (YoloTrainer's batch loop on the GPU)."""

    def __init__(self, config: Config):
        self.config = config
        h = C.c_void_p()
        _check(lib().sy_cuda_create(C.byref(config), C.byref(h)))
        self._h = h
        n = lib().sy_cuda_tensor_count(h)
        self.tensors = []
        for i in range(n):
            info = TensorInfo()
            _check(lib().sy_cuda_tensor_info(h, i, C.byref(info)), h)
            self.tensors.append(dict(index=i, name=info.name.decode(), kind=info.kind,
                                     shape=tuple(info.shape[:info.rank]), numel=int(info.numel)))

    def close(self):
        if getattr(self, "_h", None):
            lib().sy_cuda_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def params(self):
        return [t for t in self.tensors if t["kind"] == 0]

    def set_tensor(self, index: int, values: np.ndarray):
        v = np.ascontiguousarray(values, np.float32).ravel()
        _check(lib().sy_cuda_set_tensor(self._h, index, _fp(v), v.size), self._h)

    def get_tensor(self, index: int) -> np.ndarray:
        t = self.tensors[index]
        out = np.zeros(t["numel"], np.float32)
        _check(lib().sy_cuda_get_tensor(self._h, index, _fp(out), out.size), self._h)
        return out.reshape(t["shape"]) if t["shape"] else out

    def set_optimizer_state(self, index: int, moment: int, values: np.ndarray):
        v = np.ascontiguousarray(values, np.float32).ravel()
        _check(lib().sy_cuda_set_optimizer_state(self._h, index, moment, _fp(v), v.size), self._h)

    def get_optimizer_state(self, index: int, moment: int = 0) -> np.ndarray:
        t = self.tensors[index]
        out = np.zeros(t["numel"], np.float32)
        _check(lib().sy_cuda_get_optimizer_state(self._h, index, moment, _fp(out), out.size), self._h)
        return out

    def backbone_param_count(self) -> int:
        return int(lib().sy_cuda_backbone_param_count(self._h))

    def set_backbone(self, values: np.ndarray):
        v = np.ascontiguousarray(values, np.float32).ravel()
        _check(lib().sy_cuda_set_backbone(self._h, _fp(v), v.size), self._h)

    def flat_params(self) -> np.ndarray:
        return np.concatenate([self.get_tensor(t["index"]).ravel() for t in self.params])

    def flat_buffers(self) -> np.ndarray:
        return np.concatenate([self.get_tensor(t["index"]).ravel() for t in self.tensors if t["kind"] == 1])

    def set_flat_params(self, flat: np.ndarray):
        off = 0
        for t in self.params:
            self.set_tensor(t["index"], flat[off:off + t["numel"]])
            off += t["numel"]

    def set_flat_buffers(self, flat: np.ndarray):
        off = 0
        for t in self.tensors:
            if t["kind"] == 1:
                self.set_tensor(t["index"], flat[off:off + t["numel"]])
                off += t["numel"]

    def flat_velocity(self, moment: int = 0) -> np.ndarray:
        return np.concatenate([self.get_optimizer_state(t["index"], moment) for t in self.params])

    @staticmethod
    def _boxes(boxes_per_image):
        """(Box array pointer, counts) from per-image lists of (cls, x1, y1, x2, y2), or from the PackedBoxes
        that pack_boxes made (then no per-box Python work is left for the call)."""
        if isinstance(boxes_per_image, PackedBoxes):
            return boxes_per_image.pointer, boxes_per_image.counts
        packed = pack_boxes(boxes_per_image)
        return packed.pointer, packed.counts

    def prefetch_images(self, images: np.ndarray):
        """Starts the host-to-device copy of uint8 [B, S, S, 3] images (sy_cuda_prefetch_images); a later
        step / eval_loss / detect given this same array uses the copy.  The array must stay unchanged (and
        alive: the session keeps a reference to the two most recent ones) until then."""
        if images.dtype != np.uint8 or not images.flags["C_CONTIGUOUS"]:
            raise ValueError("prefetch_images wants a C-contiguous uint8 array (the pointer identifies the batch)")
        _check(lib().sy_cuda_prefetch_images(self._h, images.ctypes.data_as(C.POINTER(C.c_uint8)), images.shape[0]),
               self._h)
        self._prefetched = ([images] + getattr(self, "_prefetched", []))[:2]

    def step(self, images: np.ndarray, boxes_per_image) -> StepStats:
        """images: uint8 [B, S, S, 3] RGB (letterboxed); boxes_per_image: list of (cls, x1, y1, x2, y2)."""
        img = np.ascontiguousarray(images, np.uint8)
        arr, counts = self._boxes(boxes_per_image)
        stats = StepStats()
        _check(lib().sy_cuda_step(self._h, img.ctypes.data_as(C.POINTER(C.c_uint8)), arr, _ip(counts), img.shape[0],
                                  C.byref(stats)), self._h)
        return stats

    def step_device(self, images_device_ptr: int, batch: int, boxes_per_image) -> StepStats:
        """Step with the uint8 [B, S, S, 3] images already in this GPU's memory (device pointer)."""
        arr, counts = self._boxes(boxes_per_image)
        stats = StepStats()
        _check(lib().sy_cuda_step_device(self._h, C.c_void_p(images_device_ptr), arr, _ip(counts), batch,
                                         C.byref(stats)), self._h)
        return stats

    def step_features(self, features, boxes_per_image) -> StepStats:
        feats = [np.ascontiguousarray(f, np.float32) for f in features]
        arr, counts = self._boxes(boxes_per_image)
        ptrs = (C.POINTER(C.c_float) * 3)(*[_fp(f) for f in feats])
        stats = StepStats()
        _check(lib().sy_cuda_step_features(self._h, ptrs, arr, _ip(counts), feats[0].shape[0], C.byref(stats)),
               self._h)
        return stats

    def eval_loss(self, images: np.ndarray, boxes_per_image) -> StepStats:
        """YoloTrainer.EvaluateLoss on a batch: BatchNorm with running statistics, no update."""
        img = np.ascontiguousarray(images, np.uint8)
        arr, counts = self._boxes(boxes_per_image)
        stats = StepStats()
        _check(lib().sy_cuda_eval_loss(self._h, img.ctypes.data_as(C.POINTER(C.c_uint8)), arr, _ip(counts),
                                       img.shape[0], C.byref(stats)), self._h)
        return stats

    def eval_loss_features(self, features, boxes_per_image) -> StepStats:
        feats = [np.ascontiguousarray(f, np.float32) for f in features]
        arr, counts = self._boxes(boxes_per_image)
        ptrs = (C.POINTER(C.c_float) * 3)(*[_fp(f) for f in feats])
        stats = StepStats()
        _check(lib().sy_cuda_eval_loss_features(self._h, ptrs, arr, _ip(counts), feats[0].shape[0],
                                                C.byref(stats)), self._h)
        return stats

    def set_epoch(self, epoch: int):
        """Completed epochs, fed to the progressive end-to-end loss weight (DetectionHead.ProgressiveWeight)."""
        _check(lib().sy_cuda_set_epoch(self._h, epoch), self._h)

    def optimizer_steps(self) -> list:
        """AdamW steps taken per optimizer group (class branches, cv2, one2one_cv2)."""
        out = np.zeros(3, np.int32)
        _check(lib().sy_cuda_get_optimizer_steps(self._h, _ip(out)), self._h)
        return [int(v) for v in out]

    def set_optimizer_steps(self, steps):
        v = np.ascontiguousarray(steps, np.int32)
        _check(lib().sy_cuda_set_optimizer_steps(self._h, _ip(v)), self._h)

    def last_gradients(self) -> np.ndarray:
        n = sum(t["numel"] for t in self.params)
        out = np.zeros(n, np.float32)
        _check(lib().sy_cuda_get_last_gradients(self._h, _fp(out), n), self._h)
        return out

    def conv_profile(self, enable: bool):
        """Totals (device ms, GFLOP, launches) of the tensor-core conv launches since the previous call;
        `enable` switches CUDA-event timing of those launches on or off for the following steps."""
        ms, gf, n = C.c_double(), C.c_double(), C.c_int64()
        _check(lib().sy_cuda_conv_profile(self._h, int(bool(enable)), C.byref(ms), C.byref(gf), C.byref(n)), self._h)
        return ms.value, gf.value, n.value

    def conv_profile_launches(self):
        """[(ms, GFLOP, (pass, ic, oc, taps, h, w))] of every tensor-core conv launch of the most recent
        profiled step; pass 0 trunk stride 1, 1 trunk stride 2, 2 head forward, 3 head data gradient."""
        n = C.c_int32()
        _check(lib().sy_cuda_conv_profile_launches(self._h, None, None, None, 0, C.byref(n)), self._h)
        m = max(1, n.value)
        ms, gf, sh = (C.c_double * m)(), (C.c_double * m)(), (C.c_int32 * (6 * m))()
        _check(lib().sy_cuda_conv_profile_launches(self._h, ms, gf, sh, n.value, C.byref(n)), self._h)
        return [(ms[i], gf[i], tuple(sh[6 * i:6 * i + 6])) for i in range(n.value)]

    def last_features(self, level: int, shape) -> np.ndarray:
        out = np.zeros(int(np.prod(shape)), np.float32)
        _check(lib().sy_cuda_get_last_features(self._h, level, _fp(out), out.size), self._h)
        return out.reshape(shape)

    def last_head_outputs(self, level: int, images: int, set: int = 0):
        """Raw (box, class) logits of the latest head forward (over `images` images) at `level`, NCHW."""
        c = self.config
        h = c.image_size >> (3 + level)
        box = np.zeros((images, 4 * c.reg_max, h, h), np.float32)
        cls = np.zeros((images, c.num_classes, h, h), np.float32)
        _check(lib().sy_cuda_get_last_head_outputs(self._h, set, level, _fp(box), box.size, _fp(cls), cls.size),
               self._h)
        return box, cls

    def _detect(self, fn, source, images, options, transforms, as_array):
        o = options if options is not None else detect_options()
        tf = None
        if transforms is not None:
            tf = (Letterbox * images)(*transforms)
        out = np.zeros((images, o.max_detections), _DETECTION_DTYPE)
        counts = np.zeros(images, np.int32)
        timing = (C.c_double * 2)()
        _check(fn(self._h, source, images, tf, C.byref(o), out.ctypes.data_as(C.POINTER(Detection)), _ip(counts),
                  timing), self._h)
        self.last_detect_ms = (timing[0], timing[1])
        if as_array:
            return out, counts
        return [out[b, :int(n)].tolist() for b, n in enumerate(counts)]

    def detect(self, images: np.ndarray, options: DetectOptions = None, transforms=None, as_array: bool = False):
        """YoloDetector.Detect on letterboxed uint8 [B, S, S, 3] images: per image a list of
        (class_id, confidence, x, y, width, height) in source pixels (transforms: one Letterbox per image);
        with as_array, the [B, max_detections] records and the per-image counts as numpy arrays."""
        img = np.ascontiguousarray(images, np.uint8)
        return self._detect(lib().sy_cuda_detect, img.ctypes.data_as(C.POINTER(C.c_uint8)), img.shape[0], options,
                            transforms, as_array)

    def detect_features(self, features, options: DetectOptions = None, transforms=None, as_array: bool = False):
        feats = [np.ascontiguousarray(f, np.float32) for f in features]
        ptrs = (C.POINTER(C.c_float) * 3)(*[_fp(f) for f in feats])
        return self._detect(lib().sy_cuda_detect_features, ptrs, feats[0].shape[0], options, transforms, as_array)


def wait_limit_selftest(spins: int, device: int = 0) -> int:
    """Runs the bounded-wait check kernel (sy_cuda_wait_limit_selftest): returns the error code the wait
    reported; raises SyError for anything but the expected SY_ERR_DEVICE from a timed-out wait."""
    code = np.zeros(1, np.int32)
    status = lib().sy_cuda_wait_limit_selftest(device, spins, _ip(code))
    if status not in (SY_OK, SY_ERR_DEVICE):
        _check(status)
    return int(code[0])


def launch_count() -> int:
    """Kernels launched by the CUDA library in this process so far."""
    return int(lib().sy_cuda_launch_count())


def bench_conv(kind: int, n: int, ic: int, oc: int, h: int, w: int, k: int, iters: int = 10, device: int = 0) -> float:
    """Device ms per launch of one conv pass (0 forward, 1 data gradient, 2 weight gradient)."""
    ms = C.c_double()
    _check(lib().sy_cuda_bench_conv(device, kind, n, ic, oc, h, w, k, iters, C.byref(ms)))
    return ms.value


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _check(lib().sy_cuda_nccl_unique_id(buf))
    return bytes(buf)


# ------------------------------------------------------------------ standalone operators

def head_decode(levels, bins: int, nc: int, xyxy: bool = False, device: int = 0) -> np.ndarray:
    """CpuHead.DecodeInto over joined levels on the GPU: levels = [(box [B, 4*bins, h, w], cls [B, nc, h, w],
    stride)].  Returns [B, 4 + nc, anchors]."""
    bl = [np.ascontiguousarray(b, np.float32) for b, _, _ in levels]
    cl = [np.ascontiguousarray(c, np.float32) for _, c, _ in levels]
    B = bl[0].shape[0]
    hs = np.array([b.shape[2] for b in bl], np.int32)
    ws = np.array([b.shape[3] for b in bl], np.int32)
    st = np.array([s for _, _, s in levels], np.float32)
    out = np.zeros((B, nc + 4, int((hs * ws).sum())), np.float32)
    P = C.POINTER(C.c_float) * len(bl)
    _check(lib().sy_cuda_head_decode(device, B, len(bl), _ip(hs), _ip(ws), _fp(st), bins, nc, int(xyxy),
                                     P(*map(_fp, bl)), P(*map(_fp, cl)), _fp(out)))
    return out


def end_to_end_topk(x, nc: int, maximum: int = 300, device: int = 0) -> np.ndarray:
    """PtModel.EndToEndTopK on the GPU: x [B, fields, anchors] -> [B, min(maximum, anchors), 6 + extra]."""
    x = np.ascontiguousarray(x, np.float32)
    B, fields, anchors = x.shape
    out = np.zeros((B, min(maximum, anchors), 6 + fields - nc - 4), np.float32)
    _check(lib().sy_cuda_end_to_end_topk(device, _fp(x), B, fields, anchors, nc, maximum, _fp(out)))
    return out


def decode_detections(output, layout: int = SY_LAYOUT_AUTO, class_count: int = 0, transforms=None,
                      options: DetectOptions = None, device: int = 0):
    """YoloDetector.DecodeIndexed on the GPU for output [B, dim1, dim2]: per image a list of
    (class_id, confidence, x, y, width, height)."""
    x = np.ascontiguousarray(output, np.float32)
    if x.ndim == 2:
        x = x[None]
    B, d1, d2 = x.shape
    o = options if options is not None else detect_options()
    tf = (Letterbox * B)(*transforms) if transforms is not None else None
    out = (Detection * (B * o.max_detections))()
    counts = np.zeros(B, np.int32)
    _check(lib().sy_cuda_decode_detections(device, _fp(x), B, d1, d2, layout, class_count, tf, C.byref(o), out,
                                           _ip(counts)))
    return _detections(out, counts, o.max_detections)


def detection_loss(boxes, classes, strides, truth, nc, device=0, with_grad=True, reg_max=16, topk=10, topk2=10,
                   grad_scale=1.0):
    """DetectionLoss.Compute on the GPU for a batch.  boxes[l]: [B, 4 * reg_max, H, W]; classes[l]:
    [B, nc, H, W]; truth: list (per image) of (cls, x1, y1, x2, y2).  Returns (loss[B,3], positives[B],
    assigned[B,A], scores[B,A], dbox list, dcls list)."""
    bl = [np.ascontiguousarray(b, np.float32) for b in boxes]
    cl = [np.ascontiguousarray(c, np.float32) for c in classes]
    B = bl[0].shape[0]
    hs = np.array([b.shape[2] for b in bl], np.int32)
    ws = np.array([b.shape[3] for b in bl], np.int32)
    st = np.array(strides, np.float32)
    A = int((hs * ws).sum())
    arr, counts = Session._boxes(truth)
    loss = np.zeros((B, 3), np.float32)
    pos = np.zeros(B, np.int32)
    assigned = np.zeros((B, A), np.int32)
    scores = np.zeros((B, A), np.float32)
    db = [np.zeros_like(b) for b in bl] if with_grad else None
    dc = [np.zeros_like(c) for c in cl] if with_grad else None
    P = C.POINTER(C.c_float) * len(bl)
    _check(lib().sy_cuda_detection_loss_ex(device, B, len(bl), _ip(hs), _ip(ws), _fp(st), nc, reg_max,
                                           P(*map(_fp, bl)), P(*map(_fp, cl)), arr, _ip(counts), topk, topk2,
                                           grad_scale, _fp(loss), _ip(pos), _ip(assigned), _fp(scores),
                                           P(*map(_fp, db)) if with_grad else None,
                                           P(*map(_fp, dc)) if with_grad else None))
    return loss, pos, assigned, scores, db, dc


def conv2d_forward(x, w, bias=None, device=0):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n, ic, h, wd = x.shape
    oc, _, k, _ = w.shape
    y = np.zeros((n, oc, h, wd), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    _check(lib().sy_cuda_conv2d_forward(device, _fp(x), n, ic, h, wd, _fp(w), oc, k, None if b is None else _fp(b),
                                        _fp(y)))
    return y


def conv2d_backward_data(dy, w, device=0):
    dy = np.ascontiguousarray(dy, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n, oc, h, wd = dy.shape
    _, ic, k, _ = w.shape
    dx = np.zeros((n, ic, h, wd), np.float32)
    _check(lib().sy_cuda_conv2d_backward_data(device, _fp(dy), n, oc, h, wd, _fp(w), ic, k, _fp(dx)))
    return dx


def conv2d_backward_filter(x, dy, k, device=0):
    x = np.ascontiguousarray(x, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    n, ic, h, wd = x.shape
    oc = dy.shape[1]
    dw = np.zeros((oc, ic, k, k), np.float32)
    _check(lib().sy_cuda_conv2d_backward_filter(device, _fp(x), _fp(dy), n, ic, oc, h, wd, k, _fp(dw)))
    return dw


def padded_rows(h: int, w: int) -> int:
    """Rows per image of the library's padded channels-last layout (one-pixel zero halo, 128-row tiles)."""
    return ((h + 2) * (w + 2) + 127) // 128 * 128


def conv2d_backward_filter_static(x_padded_ptr: int, dy_padded_ptr: int, n: int, ic: int, oc: int, h: int, w: int,
                                  k: int, dw_ptr: int, stream_ptr: int = 0, device: int = 0):
    """Weight gradient for callers that cannot allocate: device pointers only, scratch in a static
    device array (see include/simdyolo_cuda.h)."""
    status = lib().sy_cuda_conv2d_backward_filter_static(device, C.c_void_p(x_padded_ptr), C.c_void_p(dy_padded_ptr),
                                                         n, ic, oc, h, w, k, C.c_void_p(dw_ptr),
                                                         C.c_void_p(stream_ptr) if stream_ptr else None)
    _check(status)


def matmul(a, b, device=0):
    """IComputeBackend.MatMul (Compute.cs:11-25): C = A @ B, row-major."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32)
    _check(lib().sy_cuda_matmul(device, _fp(a), _fp(b), _fp(c), m, n, k))
    return c


def sgd_update(w, v, g, lr, momentum, wd, images, has_grad=True, device=0):
    """TrainingParameter.Update on float32 arrays in place; raises NonFinite like the reference."""
    _check(lib().sy_cuda_sgd_update(device, _fp(w), _fp(v), _fp(g), w.size, lr, momentum, wd, images, int(has_grad)))
