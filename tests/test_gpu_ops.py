"""GPU parity of the standalone operators against the CPU oracle, through the C ABI.

Tolerances: TF32 tensor-core convolutions must match the FP32 oracle within 2e-3 relative L2 (the
bound the path is specified with for TF32); the assigner's output (assigned gt per anchor, target
scores) must be bit-identical; loss values and their gradients within 1e-5.
"""
import numpy as np
import pytest

import simdyolo_b200 as sy
from oracle import oracle as O
from tests.helpers import rel_l2

TF32_TOL = 2e-3

pytestmark = pytest.mark.gpu


def oracle_conv(x, w, bias=None):
    return np.stack([O.conv_forward(xi, w, bias) for xi in x])


@pytest.mark.parametrize("n,ic,oc,h,w,k", [
    (1, 32, 16, 8, 8, 3),
    (2, 64, 64, 20, 20, 3),
    (2, 64, 80, 40, 40, 3),
    (2, 80, 80, 20, 20, 3),
    (2, 64, 144, 20, 20, 3),
    (2, 16, 48, 12, 20, 3),
    (2, 64, 64, 20, 20, 1),
    (2, 80, 80, 40, 40, 1),
    (1, 256, 64, 20, 20, 3),
])
def test_conv_forward(n, ic, oc, h, w, k):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((n, ic, h, w)).astype(np.float32)
    wt = (rng.standard_normal((oc, ic, k, k)) / np.sqrt(ic * k * k)).astype(np.float32)
    b = rng.standard_normal(oc).astype(np.float32)
    y = sy.conv2d_forward(x, wt, b)
    ref = oracle_conv(x, wt, b)
    assert rel_l2(y, ref) < TF32_TOL


@pytest.mark.parametrize("n,ic,oc,h,w,k", [
    (2, 64, 64, 20, 20, 3),
    (2, 80, 80, 40, 40, 3),
    (2, 64, 80, 20, 20, 1),
    (2, 144, 64, 20, 20, 3),
])
def test_conv_backward_data(n, ic, oc, h, w, k):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((n, ic, h, w)).astype(np.float32)
    wt = (rng.standard_normal((oc, ic, k, k)) / np.sqrt(ic * k * k)).astype(np.float32)
    dy = rng.standard_normal((n, oc, h, w)).astype(np.float32)
    dx = sy.conv2d_backward_data(dy, wt)
    ref = np.stack([O.conv_backward(x[i], wt, dy[i])[2] for i in range(n)])
    assert rel_l2(dx, ref) < TF32_TOL


@pytest.mark.parametrize("n,ic,oc,h,w,k", [
    (2, 64, 64, 20, 20, 3),
    (2, 80, 80, 20, 20, 3),
    (3, 64, 144, 40, 40, 3),
    (2, 256, 64, 20, 20, 3),
    (2, 64, 80, 20, 20, 1),
    (1, 32, 16, 8, 8, 3),
    (2, 64, 20, 16, 16, 1),    # output channels not a multiple of the MMA width (20-class head)
    (2, 48, 20, 12, 12, 3),
])
def test_conv_backward_filter(n, ic, oc, h, w, k):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((n, ic, h, w)).astype(np.float32)
    wt = np.zeros((oc, ic, k, k), np.float32)
    dy = rng.standard_normal((n, oc, h, w)).astype(np.float32)
    dw = sy.conv2d_backward_filter(x, dy, k)
    ref = np.zeros_like(wt)
    for i in range(n):
        ref += O.conv_backward(x[i], wt, dy[i], with_dx=False)[0]
    assert rel_l2(dw, ref) < TF32_TOL


@pytest.mark.parametrize("m,n,k", [(5, 9, 67), (4, 8, 64), (1, 3, 5), (7, 17, 129), (300, 200, 100)])
def test_matmul_seam(m, n, k):
    """IComputeBackend.MatMul semantics (Compute.cs:11-25); shapes of Program.cs:44-53 plus one large."""
    a = np.sin(np.arange(m * k, dtype=np.float32) * np.float32(.13)).reshape(m, k).astype(np.float32)
    b = np.cos(np.arange(k * n, dtype=np.float32) * np.float32(.17)).reshape(k, n).astype(np.float32)
    c = sy.matmul(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    # TF32 keeps 10 mantissa bits of each operand: |error| <= 2^-9 * sum_k |a_ik b_kj| (+ fp32 accumulation)
    bound = 2.0 ** -9 * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)) + 1e-6
    assert np.all(np.abs(c - ref) <= bound)


def test_sgd_known_answer_on_gpu():
    """Program.cs:128-134 through the C ABI."""
    w = np.array([2], np.float32)
    v = np.zeros(1, np.float32)
    sy.sgd_update(w, v, np.array([4], np.float32), .1, .9, .01, 2)
    assert abs(w[0] - 1.798) <= 1e-6 * (1 + 1.798) and abs(v[0] - 2.02) <= 1e-6 * (1 + 2.02)
    sy.sgd_update(w, v, np.array([2], np.float32), .1, .9, .01, 1)
    assert abs(w[0] - 1.414402) <= 1e-6 * (1 + 1.414402)
    w0, v0 = w.copy(), v.copy()
    sy.sgd_update(w, v, np.zeros(1, np.float32), .1, .9, .01, 1, has_grad=False)
    assert w.tobytes() == w0.tobytes() and v.tobytes() == v0.tobytes()


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_sgd_rejects_nonfinite_on_gpu(bad):
    """Program.cs:54-63"""
    for length in (3, 8, 19):
        for idx in (0, length - 1):
            g = np.ones(length, np.float32)
            g[idx] = bad
            with pytest.raises(ArithmeticError):
                sy.sgd_update(np.zeros(length, np.float32), np.zeros(length, np.float32), g, .01, .9, 0.0, 1)


def test_empty_labels_bce_on_gpu():
    """Program.cs:135-139 through the C ABI."""
    loss, pos, assigned, scores, db, dc = sy.detection_loss([np.zeros((1, 64, 2, 2), np.float32)],
                                                            [np.zeros((1, 1, 2, 2), np.float32)], [8.0], [[]], 1)
    assert abs(loss[0, 1] - 2 * np.log(2)) <= 1e-6 * (1 + 2 * np.log(2))
    assert abs(dc[0].ravel()[0] - .25) <= 1e-6 * 1.25
    assert pos[0] == 0 and loss[0, 0] == 0 and loss[0, 2] == 0 and np.all(assigned == -1)


def random_head_outputs(rng, batch, size, nc, nboxes, scale=1.5, cls_shift=-2.0):
    hs = [size // 8, size // 16, size // 32]
    boxes = [(rng.standard_normal((batch, 64, h, h)) * scale).astype(np.float32) for h in hs]
    classes = [(rng.standard_normal((batch, nc, h, h)) + cls_shift).astype(np.float32) for h in hs]
    truth = []
    for _ in range(batch):
        per = []
        for _ in range(nboxes):
            w, h = np.exp(rng.uniform(np.log(8), np.log(size / 2), 2))
            cx, cy = rng.uniform(0, size, 2)
            per.append((int(rng.integers(nc)), float(np.float32(max(0, cx - w / 2))), float(np.float32(max(0, cy - h / 2))),
                        float(np.float32(min(size, cx + w / 2))), float(np.float32(min(size, cy + h / 2)))))
        truth.append(per)
    return boxes, classes, truth


@pytest.mark.parametrize("seed,size,nc,nboxes", [(0, 640, 80, 8), (1, 320, 3, 5), (2, 256, 20, 30), (3, 640, 80, 1)])
def test_assigner_and_loss_match_oracle(seed, size, nc, nboxes):
    rng = np.random.default_rng(seed)
    batch = 3
    boxes, classes, truth = random_head_outputs(rng, batch, size, nc, nboxes)
    truth[-1] = truth[-1][:0] if seed == 3 else truth[-1]   # one empty image
    loss, pos, assigned, scores, db, dc = sy.detection_loss(boxes, classes, [8.0, 16.0, 32.0], truth, nc)
    for b in range(batch):
        ol, odb, odc, oa, os_ = O.detection_loss([x[b] for x in boxes], [x[b] for x in classes], [8.0, 16.0, 32.0],
                                                 truth[b], nc)
        assert np.array_equal(assigned[b], oa), f"image {b}: assignment differs"
        assert np.array_equal(scores[b], os_), f"image {b}: target scores differ"
        assert pos[b] == ol["positives"]
        # the reference (and the oracle) accumulate the 672k BCE terms in float, the GPU in double:
        # float summation alone moves the sum by ~1e-5 relative
        for got, want in zip(loss[b], (ol["box"], ol["cls"], ol["dfl"])):
            assert abs(got - want) <= 1e-4 * max(1.0, abs(want))
        for l in range(3):
            assert rel_l2(dc[l][b], odc[l]) < 1e-5
            if ol["positives"]:
                assert rel_l2(db[l][b], odb[l]) < 1e-4 or np.abs(odb[l]).max() == 0
            else:
                assert np.all(db[l][b] == 0)


def test_assigner_ties_resolve_to_lowest_anchor():
    """Equal metrics (constant logits) must keep the lowest anchor indices, like the bounded
    PriorityQueue of (metric, -anchor) in DetectionLoss.cs:65."""
    size, nc = 256, 2
    hs = [size // 8, size // 16, size // 32]
    boxes = [np.zeros((1, 64, h, h), np.float32) for h in hs]
    classes = [np.zeros((1, nc, h, h), np.float32) for h in hs]
    truth = [[(1, 40.0, 40.0, 200.0, 180.0), (0, 100.0, 60.0, 140.0, 230.0)]]
    _, pos, assigned, scores, _, _ = sy.detection_loss(boxes, classes, [8.0, 16.0, 32.0], truth, nc)
    _, _, _, oa, os_ = O.detection_loss([b[0] for b in boxes], [c[0] for c in classes], [8.0, 16.0, 32.0], truth[0], nc)
    assert np.array_equal(assigned[0], oa) and np.array_equal(scores[0], os_)
    assert pos[0] > 0


@pytest.mark.parametrize("reg_max,topk,topk2,scale,seed", [
    (16, 7, 1, 0.3, 4),    # YOLO26 one-to-one branch early in the progressive schedule
    (16, 1, 1, 1.0, 5),    # YOLOv10 one-to-one branch
    (1, 10, 10, 0.8, 6),   # reg_max 1: L1 box loss instead of DFL
    (1, 7, 1, 0.2, 7),
])
def test_end_to_end_loss_variants_match_oracle(reg_max, topk, topk2, scale, seed):
    """DetectionLoss.Compute with the end-to-end heads' arguments (DetectionLoss.cs:48-91, :123-131):
    the second top-k after the conflicts, reg_max 1 and the gradient scale; assignment bit-exact."""
    rng = np.random.default_rng(seed)
    batch, size, nc = 3, 320, 20
    boxes, classes, truth = random_head_outputs(rng, batch, size, nc, 12)
    if reg_max == 1:
        # raw distances (grid units) instead of DFL logits
        boxes = [np.abs(b[:, :4]) * 2.0 + 0.5 for b in boxes]
    loss, pos, assigned, scores, db, dc = sy.detection_loss(boxes, classes, [8.0, 16.0, 32.0], truth, nc,
                                                            reg_max=reg_max, topk=topk, topk2=topk2, grad_scale=scale)
    for b in range(batch):
        ol, odb, odc, oa, os_ = O.detection_loss([x[b] for x in boxes], [x[b] for x in classes], [8.0, 16.0, 32.0],
                                                 truth[b], nc, bins=reg_max, topk=topk, topk2=topk2, grad_scale=scale)
        assert np.array_equal(assigned[b], oa), f"image {b}: assignment differs"
        assert np.array_equal(scores[b], os_), f"image {b}: target scores differ"
        assert pos[b] == ol["positives"]
        for got, want in zip(loss[b], (ol["box"], ol["cls"], ol["dfl"])):
            assert abs(got - want) <= 1e-4 * max(1.0, abs(want))
        for l in range(3):
            assert rel_l2(dc[l][b], odc[l]) < 1e-5
            if ol["positives"]:
                assert rel_l2(db[l][b], odb[l]) < 1e-4 or np.abs(odb[l]).max() == 0
