"""Pins the CPU oracle to the reference's own known-answer and finite-difference tests.

Each test restates one case of tests/SimdYolo.Training.Tests/Program.cs (reference project) with the
same inputs, tolerances and the same ``Near`` rule |a - e| <= tol * (1 + |e|) (Program.cs:260).
"""
import math

import numpy as np
import pytest

from oracle import oracle as O


def near(actual, expected, tol):
    actual = float(actual)
    expected = float(expected)
    assert math.isfinite(actual) and abs(actual - expected) <= tol * (1 + abs(expected)), (actual, expected, tol)


def f32seq(n, fn):
    return np.array([fn(np.float32(i)) for i in range(n)], np.float32)


@pytest.mark.parametrize("m,n,k", [(5, 9, 67), (4, 8, 64), (1, 3, 5), (7, 17, 129)])
def test_right_transposed_vs_double(m, n, k):
    """Program.cs:44-53"""
    a = np.sin(np.arange(m * k, dtype=np.float32) * np.float32(.13)).astype(np.float32).reshape(m, k)
    b = np.cos(np.arange(n * k, dtype=np.float32) * np.float32(.17)).astype(np.float32).reshape(n, k)
    c = O.right_transposed(a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    for i in range(m):
        for j in range(n):
            near(c[i, j], np.float32(ref[i, j]), 3e-5)


@pytest.mark.parametrize("length", [3, 8, 19])
@pytest.mark.parametrize("where", ["first", "last"])
@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_sgd_rejects_nonfinite(length, where, bad):
    """Program.cs:54-63 (default TrainingOptions: lr .01, momentum .9, wd .0005; decay off)"""
    data = np.ones(length, np.float32)
    data[0 if where == "first" else length - 1] = bad
    assert O.lib().syo_all_finite(data, length) == 0
    w = np.zeros(length, np.float32)
    v = np.zeros(length, np.float32)
    assert O.sgd_update(w, v, data.copy(), .01, .9, 0.0, 1, True) == 1


def test_conv_gradient_accumulates_and_forward_is_kept():
    """Program.cs:64-77: three backward passes accumulate step * once; forward output unchanged."""
    x = np.sin(np.arange(128, dtype=np.float32) * np.float32(.2)).astype(np.float32).reshape(2, 8, 8)
    w = (np.cos(np.arange(36, dtype=np.float32)) * np.float32(.1)).astype(np.float32).reshape(2, 2, 3, 3)
    acc = np.zeros_like(w)
    once = out0 = None
    for step in range(3):
        y = O.conv_forward(x, w)
        dw, _, _ = O.conv_backward(x, w, np.ones_like(y), with_dx=False)
        acc += dw
        if step == 0:
            once, out0 = acc.copy(), y.copy()
        for i in range(w.size):
            near(acc.ravel()[i], once.ravel()[i] * (step + 1), 2e-4)
        assert np.array_equal(y, out0)


def _objective(x, w, up, bias=None, groups=1):
    if groups == 1:
        y = O.conv_forward(x, w, bias)
    else:
        y = O.grouped_conv_forward(x, w, groups, bias)
    return float(np.sum(y.astype(np.float64) * up.astype(np.float64)))


def test_conv_finite_differences():
    """Program.cs:78-89: input 1x2x4x5, W 3x2x3x3, eps .002, tol .002"""
    x = np.sin(np.arange(40, dtype=np.float32) * np.float32(.31)).astype(np.float32).reshape(2, 4, 5)
    w = (np.cos(np.arange(54, dtype=np.float32) * np.float32(.23)) * np.float32(.1)).astype(np.float32).reshape(3, 2, 3, 3)
    up = np.sin(np.arange(60, dtype=np.float32) * np.float32(.17)).astype(np.float32).reshape(3, 4, 5)
    dw, _, dx = O.conv_backward(x, w, up)
    e = np.float32(.002)
    for idx in (0, 13, 53):
        wp, wm = w.copy(), w.copy()
        wp.ravel()[idx] += e
        wm.ravel()[idx] -= e
        near(dw.ravel()[idx], (_objective(x, wp, up) - _objective(x, wm, up)) / (2 * e), .002)
    for idx in (0, 17, 39):
        xp, xm = x.copy(), x.copy()
        xp.ravel()[idx] += e
        xm.ravel()[idx] -= e
        near(dx.ravel()[idx], (_objective(xp, w, up) - _objective(xm, w, up)) / (2 * e), .002)


@pytest.mark.parametrize("ic,oc,groups", [(4, 6, 2), (3, 3, 3), (2, 4, 2)])
def test_grouped_conv_finite_differences(ic, oc, groups):
    """Program.cs:90-105: 5x9 input, weight/bias/input central differences, tol .002"""
    x = np.sin(np.arange(ic * 45, dtype=np.float32) * np.float32(.31)).astype(np.float32).reshape(ic, 5, 9)
    count = oc * (ic // groups) * 9
    w = (np.cos(np.arange(count, dtype=np.float32) * np.float32(.23)) * np.float32(.1)).astype(np.float32)
    w = w.reshape(oc, ic // groups, 3, 3)
    b = np.zeros(oc, np.float32)
    up = np.sin(np.arange(oc * 45, dtype=np.float32) * np.float32(.17)).astype(np.float32).reshape(oc, 5, 9)
    dw, db, dx = O.grouped_conv_backward(x, w, groups, up, with_bias=True)

    def fd(arr, idx, which):
        p, m = arr.copy(), arr.copy()
        p.ravel()[idx] += np.float32(.002)
        m.ravel()[idx] -= np.float32(.002)
        args_p = dict(x=x, w=w, bias=b)
        args_m = dict(x=x, w=w, bias=b)
        args_p[which] = p
        args_m[which] = m
        return (_objective(args_p["x"], args_p["w"], up, args_p["bias"], groups) -
                _objective(args_m["x"], args_m["w"], up, args_m["bias"], groups)) / .004

    for idx in (0, count // 2, count - 1):
        near(dw.ravel()[idx], fd(w, idx, "w"), .002)
    for idx in (0, 44, x.size - 1):
        near(dx.ravel()[idx], fd(x, idx, "x"), .002)
    for idx in (0, oc - 1):
        near(db[idx], fd(b, idx, "bias"), .002)


def test_progressive_weight():
    """Program.cs:106-110"""
    L = O.lib()
    near(L.syo_progressive_weight(0, 5), .8, 1e-7)
    near(L.syo_progressive_weight(2, 5), .45, 1e-7)
    near(L.syo_progressive_weight(4, 5), .1, 1e-7)
    near(L.syo_progressive_weight(9, 5), .1, 1e-7)


def test_silu_finite_differences():
    """Program.cs:111-115"""
    data = np.array([-30, -2, -.3, 0, .7, 5, 30], np.float32)
    _, sig = O.silu_forward(data)
    dx = O.silu_backward(data, sig, np.ones_like(data))
    sigm = O.lib().syo_sigmoid
    for i, v in enumerate(data):
        a, b = np.float32(v + np.float32(.002)), np.float32(v - np.float32(.002))
        near(dx[i], (a * sigm(a) - b * sigm(b)) / .004, .002)


def test_batchnorm_backward_and_running_variance():
    """Program.cs:116-127"""
    data = np.sin(np.arange(24, dtype=np.float32) * np.float32(.7)).astype(np.float32).reshape(2, 3, 4)
    gamma = np.array([1.2, .8], np.float32)
    beta = np.array([.1, -.2], np.float32)
    mean = np.zeros(2, np.float32)
    var = np.ones(2, np.float32)
    y, xhat, inv, _, _ = O.batchnorm_forward(data, gamma, beta, mean, var, .001, .03, True)
    dy = np.cos(np.arange(24, dtype=np.float32) * np.float32(.2)).astype(np.float32).reshape(2, 3, 4)
    dg, dbt, dx = O.batchnorm_backward(dy, xhat, inv, gamma)

    def objective(d):
        yy, *_ = O.batchnorm_forward(d, gamma, beta, np.zeros(2, np.float32), np.ones(2, np.float32), .001, .03, True)
        return float(np.sum(yy.astype(np.float64) * dy))

    for idx in (0, 13, 23):
        p, m = data.copy(), data.copy()
        p.ravel()[idx] += np.float32(.002)
        m.ravel()[idx] -= np.float32(.002)
        near(dx.ravel()[idx], (objective(p) - objective(m)) / .004, .002)
    for c in range(2):
        near(dbt[c], dy[c].sum(dtype=np.float32), 1e-5)
    assert np.all(np.isfinite(var)) and np.all(var > 0)


def test_sgd_known_answer():
    """Program.cs:128-134: w=2, g=4, lr .1, m .9, wd .01, images 2 -> w 1.798, v 2.02; g=2 -> 1.414402"""
    w = np.array([2], np.float32)
    v = np.zeros(1, np.float32)
    assert O.sgd_update(w, v, np.array([4], np.float32), .1, .9, .01, 2, True) == 0
    near(w[0], 1.798, 1e-6)
    near(v[0], 2.02, 1e-6)
    assert O.sgd_update(w, v, np.array([2], np.float32), .1, .9, .01, 1, True) == 0
    near(w[0], 1.414402, 1e-6)
    w0, v0 = w.copy(), v.copy()
    assert O.sgd_update(w, v, np.zeros(1, np.float32), .1, .9, .01, 1, False) == 0
    assert w.tobytes() == w0.tobytes() and v.tobytes() == v0.tobytes()


def test_empty_labels_bce():
    """Program.cs:135-139: 1 level 2x2, nc 1, zero logits, no truth -> cls 2 ln 2, grad[0] .25"""
    loss, db, dc, assigned, _ = O.detection_loss([np.zeros((64, 2, 2), np.float32)], [np.zeros((1, 2, 2), np.float32)],
                                                 [8.0], [], 1)
    near(loss["cls"], math.log(2) * 2, 1e-6)
    near(dc[0].ravel()[0], .25, 1e-6)
    assert loss["positives"] == 0 and loss["box"] == 0 and loss["dfl"] == 0
    assert not loss["connected"] and np.all(assigned == -1)


def test_invalid_class_rejected():
    """DetectionLoss.cs:51: class id outside [0, nc) is an argument error."""
    with pytest.raises(ValueError):
        O.detection_loss([np.zeros((64, 2, 2), np.float32)], [np.zeros((1, 2, 2), np.float32)], [8.0],
                         [(3, 0, 0, 8, 8)], 1)


def test_deterministic_math_is_correctly_rounded():
    """The assigner's exp/atan agree with the double-precision libm rounded once to float."""
    L = O.lib()
    rng = np.random.default_rng(7)
    xs = np.concatenate([rng.uniform(-100, 88, 4000), rng.normal(0, 3, 4000)]).astype(np.float32)
    for x in xs:
        assert L.syo_expf(float(x)) == np.float32(math.exp(float(x)))
    ys = np.concatenate([rng.uniform(-50, 50, 4000), rng.normal(0, 1, 4000)]).astype(np.float32)
    for y in ys:
        assert L.syo_atanf(float(y)) == np.float32(math.atan(float(y)))
