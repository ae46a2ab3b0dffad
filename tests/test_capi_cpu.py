"""CPU-side checks of the C ABI library and of the host-side model description (no GPU calls)."""
import ctypes as C
import os
import re

import numpy as np

import simdyolo_b200 as sy
from oracle import oracle as O
from tests.helpers import backbone_desc, head_desc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "simdyolo_cuda.h")).read()
    return sorted(set(re.findall(r"^SY_API [^\n(]*?\b(sy_cuda_\w+)\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    L = sy.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(L, name), name
    assert sorted(sy.EXPORTED) == names


def test_config_struct_size_matches_header_layout():
    # offsetof checks against the C layout: nccl_id follows 4 int32, blocks are 6 int32 each
    assert sy.Config.nccl_id.offset == 16
    assert C.sizeof(sy.Block) == 24
    assert sy.Config.box_blocks.offset + 3 * 8 * 24 == sy.Config.cls_blocks.offset


def test_status_to_exception_mapping():
    for status, cls in [(sy.SY_ERR_INVALID_ARGUMENT, ValueError), (sy.SY_ERR_UNSUPPORTED_SHAPE, NotImplementedError),
                        (sy.SY_ERR_NONFINITE, ArithmeticError)]:
        try:
            sy._raise(status, "x")
        except cls as e:
            assert e.status == status
        else:
            raise AssertionError("not raised")


def test_calls_without_gpu_fail_cleanly():
    # no CUDA device here: the standalone ops must return an error status, not crash
    import torch
    if torch.cuda.is_available():
        return
    a = np.ones((2, 2), np.float32)
    try:
        sy.matmul(a, a)
    except sy.SyError as e:
        assert e.status in (sy.SY_ERR_INVALID_ARGUMENT, sy.SY_ERR_DEVICE)
    else:
        raise AssertionError("matmul without a GPU did not fail")


def test_backbone_description_matches_oracle():
    for model in ("yolov8n", "yolov8s", "yolov8l"):
        cfg = sy.make_config(model, image_size=640)
        convs = sy.yolov8_backbone_convs(cfg.width_mult, cfg.depth_mult, cfg.max_channels)
        count = sum(oc * ic * k * k + oc for oc, ic, k in convs)
        bd = backbone_desc(cfg)
        assert O.lib().syo_backbone_param_count(C.byref(bd)) == count
        ch = np.zeros(3, np.int32)
        O.lib().syo_backbone_feature_channels(C.byref(bd), ch.ctypes.data_as(C.POINTER(C.c_int32)))
        assert tuple(ch) == tuple(cfg.feature_channels)


def test_yolov8n_head_sizes():
    """v8n head at 80 classes: 897,648 parameters (conv + BN), channels 64 / 80 (survey figure)."""
    cfg = sy.make_config("yolov8n")
    assert tuple(cfg.feature_channels) == (64, 128, 256)
    d = head_desc(cfg)
    assert O.lib().syo_head_param_count(C.byref(d)) == 897_648
    assert cfg.box_blocks[0][0].oc == 64 and cfg.cls_blocks[0][0].oc == 80
