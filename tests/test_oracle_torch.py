"""Cross-checks the CPU oracle against PyTorch (CPU) autograd.

The reference's external oracle is Ultralytics' official loss, which is not installed here; these tests
check gradient consistency instead: the hand-written backward of the restated operators and loss
(HeadOperations.cs, DetectionLoss.cs) against torch autograd of the same forward definitions.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("ic,oc,k,h,w", [(8, 16, 3, 9, 11), (16, 8, 1, 7, 5), (5, 7, 3, 4, 4)])
def test_conv_matches_torch(ic, oc, k, h, w):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((ic, h, w)).astype(np.float32)
    wt = (rng.standard_normal((oc, ic, k, k)) * .2).astype(np.float32)
    b = rng.standard_normal(oc).astype(np.float32)
    dy = rng.standard_normal((oc, h, w)).astype(np.float32)
    y = O.conv_forward(x, wt, b)
    dw, db, dx = O.conv_backward(x, wt, dy, with_bias=True)
    tx = torch.tensor(x[None], requires_grad=True)
    tw = torch.tensor(wt, requires_grad=True)
    tb = torch.tensor(b, requires_grad=True)
    ty = F.conv2d(tx, tw, tb, padding=k // 2)
    ty.backward(torch.tensor(dy[None]))
    assert rel_l2(y, ty.detach()[0]) < 1e-6
    assert rel_l2(dw, tw.grad) < 1e-6
    assert rel_l2(db, tb.grad) < 1e-6
    assert rel_l2(dx, tx.grad[0]) < 1e-6


def test_depthwise_conv_matches_torch():
    rng = np.random.default_rng(2)
    c, h, w = 6, 7, 9
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c, 1, 3, 3)) * .3).astype(np.float32)
    dy = rng.standard_normal((c, h, w)).astype(np.float32)
    y = O.grouped_conv_forward(x, wt, c)
    dw, _, dx = O.grouped_conv_backward(x, wt, c, dy)
    tx = torch.tensor(x[None], requires_grad=True)
    tw = torch.tensor(wt, requires_grad=True)
    ty = F.conv2d(tx, tw, None, padding=1, groups=c)
    ty.backward(torch.tensor(dy[None]))
    assert rel_l2(y, ty.detach()[0]) < 1e-6
    assert rel_l2(dw, tw.grad) < 1e-6
    assert rel_l2(dx, tx.grad[0]) < 1e-6


def test_batchnorm_train_matches_torch():
    rng = np.random.default_rng(3)
    c, h, w = 5, 6, 7
    x = (rng.standard_normal((c, h, w)) * 3 + 1).astype(np.float32)
    g = rng.uniform(.5, 1.5, c).astype(np.float32)
    be = rng.standard_normal(c).astype(np.float32)
    rm = rng.standard_normal(c).astype(np.float32)
    rv = rng.uniform(.5, 2, c).astype(np.float32)
    dy = rng.standard_normal((c, h, w)).astype(np.float32)
    trm, trv = torch.tensor(rm), torch.tensor(rv)
    y, xhat, inv, _, _ = O.batchnorm_forward(x, g, be, rm, rv, 1e-3, .03, True)
    dg, dbt, dx = O.batchnorm_backward(dy, xhat, inv, g)
    tx = torch.tensor(x[None], requires_grad=True)
    tg = torch.tensor(g, requires_grad=True)
    tbe = torch.tensor(be, requires_grad=True)
    ty = F.batch_norm(tx, trm, trv, tg, tbe, training=True, momentum=.03, eps=1e-3)
    ty.backward(torch.tensor(dy[None]))
    assert rel_l2(y, ty.detach()[0]) < 1e-5
    assert rel_l2(dx, tx.grad[0]) < 1e-5
    assert rel_l2(dg, tg.grad) < 1e-5
    assert rel_l2(dbt, tbe.grad) < 1e-5
    assert rel_l2(rm, trm) < 1e-6 and rel_l2(rv, trv) < 1e-6


def torch_ciou(p, t):
    """DetectionLoss.cs:171-183 in torch; alpha detached (the reference's stop-gradient)."""
    eps = 1e-7
    x1, y1, x2, y2 = p.unbind(-1)
    a1, b1, a2, b2 = t.unbind(-1)
    w1, h1 = x2 - x1, y2 - y1 + eps
    w2, h2 = a2 - a1, b2 - b1 + eps
    inter = (torch.minimum(x2, a2) - torch.maximum(x1, a1)).clamp(min=0) * \
            (torch.minimum(y2, b2) - torch.maximum(y1, b1)).clamp(min=0)
    iou = inter / (w1 * h1 + w2 * h2 - inter + eps)
    cw = torch.maximum(x2, a2) - torch.minimum(x1, a1)
    ch = torch.maximum(y2, b2) - torch.minimum(y1, b1)
    rho = ((a1 + a2 - x1 - x2) ** 2 + (b1 + b2 - y1 - y2) ** 2) / 4
    v = 4 / (np.pi ** 2) * (torch.atan(w2 / h2) - torch.atan(w1 / h1)) ** 2
    with torch.no_grad():
        alpha = v / (v - iou + 1 + eps)
    return iou - rho / (cw ** 2 + ch ** 2 + eps) - v * alpha


def make_case(seed, hs=(8, 4, 2), nc=3, ngt=3, image=64):
    rng = np.random.default_rng(seed)
    boxes = [(rng.standard_normal((64, h, h)) * 1.5).astype(np.float32) for h in hs]
    classes = [(rng.standard_normal((nc, h, h)) - 2).astype(np.float32) for h in hs]
    truth = []
    for _ in range(ngt):
        w, h = rng.uniform(8, 40, 2)
        cx, cy = rng.uniform(w / 2, image - w / 2), rng.uniform(h / 2, image - h / 2)
        truth.append((int(rng.integers(nc)), cx - w / 2, cy - h / 2, cx + w / 2, cy + h / 2))
    return boxes, classes, truth


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_loss_gradients_match_autograd(seed):
    strides = [8.0, 16.0, 32.0]
    boxes, classes, truth = make_case(seed)
    nc = classes[0].shape[0]
    loss, db, dc, assigned, scores = O.detection_loss(boxes, classes, strides, truth, nc)
    assert loss["positives"] > 0
    tb = [torch.tensor(b, requires_grad=True) for b in boxes]
    tc = [torch.tensor(c, requires_grad=True) for c in classes]
    # anchors, level-major, pixel row-major
    logits = torch.cat([c.reshape(nc, -1) for c in tc], 1).T
    dist = torch.cat([b.reshape(4, 16, -1) for b in tb], 2).permute(2, 0, 1)    # [A,4,16]
    ctr, st = [], []
    for h, s in zip([b.shape[1] for b in boxes], strides):
        ys, xs = np.meshgrid(np.arange(h), np.arange(h), indexing="ij")
        ctr.append(np.stack([(xs.ravel() + .5) * s, (ys.ravel() + .5) * s], 1))
        st.append(np.full(h * h, s))
    ctr = torch.tensor(np.concatenate(ctr), dtype=torch.float32)
    st = torch.tensor(np.concatenate(st), dtype=torch.float32)
    prob = dist.softmax(-1)
    expect = (prob * torch.arange(16, dtype=torch.float32)).sum(-1)       # [A,4]
    dec = torch.stack([ctr[:, 0] - expect[:, 0] * st, ctr[:, 1] - expect[:, 1] * st,
                       ctr[:, 0] + expect[:, 2] * st, ctr[:, 1] + expect[:, 3] * st], 1)
    sc = torch.tensor(scores)
    ss = max(1.0, float(scores.sum(dtype=np.float32)))
    target = torch.zeros_like(logits)
    tru = np.array([t[1:] for t in truth], np.float32)
    cls = np.array([t[0] for t in truth])
    pos = np.nonzero(assigned >= 0)[0]
    for a in pos:
        target[a, cls[assigned[a]]] = sc[a]
    bce = (logits.clamp(min=0) - logits * target + torch.log1p(torch.exp(-logits.abs()))).sum() * (.5 / ss)
    pa = torch.tensor(pos)
    tg = torch.tensor(tru[assigned[pos]])
    ci = torch_ciou(dec[pa] / st[pa, None], tg / st[pa, None])
    box = ((1 - ci) * sc[pa] * 7.5 / ss).sum()
    d = torch.stack([(ctr[pa, 0] - tg[:, 0]), (ctr[pa, 1] - tg[:, 1]), (tg[:, 2] - ctr[pa, 0]),
                     (tg[:, 3] - ctr[pa, 1])], 1) / st[pa, None]
    d = d.clamp(0, 14.99)
    left = d.long()
    rw = d - left
    lp = torch.log_softmax(dist[pa], -1)
    ce = -(lp.gather(-1, left[..., None])[..., 0] * (1 - rw) + lp.gather(-1, (left + 1)[..., None])[..., 0] * rw)
    dfl = (ce * (1.5 * sc[pa] / (4 * ss))[:, None]).sum()
    (bce + box + dfl).backward()
    assert abs(float(bce) - loss["cls"]) <= 1e-4 * max(1, abs(loss["cls"]))
    assert abs(float(box) - loss["box"]) <= 1e-4 * max(1, abs(loss["box"]))
    assert abs(float(dfl) - loss["dfl"]) <= 1e-4 * max(1, abs(loss["dfl"]))
    for ours, ref in zip(dc, tc):
        assert rel_l2(ours, ref.grad) < 1e-4
    for ours, ref in zip(db, tb):
        assert rel_l2(ours, ref.grad) < 1e-3


def test_adamw_matches_torch_over_steps():
    """Config 3's optimizer (the reference has no AdamW): the oracle's update against
    torch.optim.AdamW on gradients already divided by the image count, with the step skipped for a
    group without gradient (TrainingParameter.cs:24 semantics)."""
    rng = np.random.default_rng(8)
    n, images, lr, wd, b1, b2, eps = 257, 4, 1e-3, 0.05, 0.9, 0.999, 1e-8
    w0 = rng.standard_normal(n).astype(np.float32)
    w, m, v = w0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    tw = torch.tensor(w0, requires_grad=True)
    opt = torch.optim.AdamW([tw], lr=lr, betas=(b1, b2), eps=eps, weight_decay=wd)
    for step in range(1, 6):
        g = (rng.standard_normal(n) * images).astype(np.float32)
        gc = g.copy()
        assert O.lib().syo_adamw_update(w, m, v, gc, n, lr, b1, b2, eps, wd, step, images, 1) == 0
        assert not gc.any()   # gradients are cleared after the update
        opt.zero_grad()
        tw.grad = torch.tensor(g / np.float32(images))
        opt.step()
        np.testing.assert_allclose(w, tw.detach().numpy(), rtol=2e-6, atol=1e-7)
    # no gradient: nothing moves
    before = w.copy()
    assert O.lib().syo_adamw_update(w, m, v, np.ones(n, np.float32), n, lr, b1, b2, eps, wd, 6, images, 0) == 0
    assert np.array_equal(w, before)


def test_batchnorm_evaluation_mode_matches_torch():
    """HeadOperations.BatchNorm with training = false (EvaluateLoss): running statistics, no update."""
    rng = np.random.default_rng(12)
    c, h, w = 6, 5, 7
    x = rng.standard_normal((c, h, w)).astype(np.float32) * 2 + 0.5
    gamma = rng.uniform(0.5, 1.5, c).astype(np.float32)
    beta = rng.standard_normal(c).astype(np.float32)
    rmean = rng.standard_normal(c).astype(np.float32)
    rvar = rng.uniform(0.5, 2.0, c).astype(np.float32)
    rm0, rv0 = rmean.copy(), rvar.copy()
    y = O.batchnorm_forward(x, gamma, beta, rmean, rvar, eps=1e-3, momentum=0.03, training=False)[0]
    ref = F.batch_norm(torch.tensor(x)[None], torch.tensor(rm0), torch.tensor(rv0), torch.tensor(gamma),
                       torch.tensor(beta), training=False, eps=1e-3)[0]
    np.testing.assert_allclose(y.reshape(c, h, w), ref.numpy(), rtol=1e-5, atol=1e-6)
    assert np.array_equal(rmean, rm0) and np.array_equal(rvar, rv0)
