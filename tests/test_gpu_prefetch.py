"""sy_cuda_prefetch_images: a batch's host-to-device copy started on the session's copy stream before the
call that uses it.  The results must not change: a loop that prefetches batch k + 1 before stepping batch k
ends bit-identical to the same loop without prefetches (parameters, buffers, velocities, every step's
losses), a prefetch that the next call does not use is ignored, pageable memory works through the staging
buffer, and evaluation and detection take prefetched batches too."""
import numpy as np
import pytest

import simdyolo_b200 as sy
from simdyolo_b200 import data

pytestmark = pytest.mark.gpu
IMAGE, BATCH = 256, 4


def new_session():
    cfg = sy.make_config("yolov8n", image_size=IMAGE, max_batch=BATCH, max_boxes=8)
    s = sy.Session(cfg)
    params, buffers = data.head_params(s, seed=3, image_size=IMAGE)
    s.set_flat_params(params)
    s.set_flat_buffers(buffers)
    s.set_backbone(data.backbone_params("yolov8n", seed=3))
    return s


def batches(n):
    rng = np.random.default_rng(17)
    return [data.synthetic_batch(rng, BATCH, IMAGE, 80, boxes=(1, 6), wh=(8.0, 96.0)) for _ in range(n)]


def stats_tuple(st):
    return (st.box, st.cls, st.dfl, st.positives, st.box_has_grad, st.grad_checksum)


@pytest.mark.parametrize("pinned", [True, False], ids=["pinned", "pageable"])
def test_prefetched_loop_matches_plain_loop(pinned):
    import torch
    work = batches(3)
    if pinned:
        host = [torch.from_numpy(b[0]).pin_memory().numpy() for b in work]
    else:
        host = [np.ascontiguousarray(b[0]) for b in work]
    order = [0, 1, 2, 0, 1, 2, 2]
    plain, fetched = new_session(), new_session()
    a = [stats_tuple(plain.step(host[k], work[k][1])) for k in order]
    b = []
    fetched.prefetch_images(host[order[0]])
    for i, k in enumerate(order):
        if i + 1 < len(order):
            fetched.prefetch_images(host[order[i + 1]])
        b.append(stats_tuple(fetched.step(host[k], work[k][1])))
    assert a == b
    assert plain.flat_params().tobytes() == fetched.flat_params().tobytes()
    assert plain.flat_buffers().tobytes() == fetched.flat_buffers().tobytes()
    assert plain.flat_velocity().tobytes() == fetched.flat_velocity().tobytes()
    plain.close()
    fetched.close()


def test_unused_prefetch_is_ignored_and_eval_detect_take_prefetches():
    work = batches(3)
    host = [np.ascontiguousarray(b[0]) for b in work]
    s1, s2 = new_session(), new_session()
    # a prefetch of another batch (or another image count) does not stand in for the one stepped
    s1.prefetch_images(host[1])
    s1.prefetch_images(host[2][:2].copy())
    assert stats_tuple(s1.step(host[0], work[0][1])) == stats_tuple(s2.step(host[0], work[0][1]))
    # evaluation and detection from prefetched batches
    s1.prefetch_images(host[1])
    e1 = s1.eval_loss(host[1], work[1][1])
    e2 = s2.eval_loss(host[1], work[1][1])
    assert (e1.box, e1.cls, e1.dfl, e1.positives) == (e2.box, e2.cls, e2.dfl, e2.positives)
    o = sy.detect_options(0.0, 0.5, 50)
    s1.prefetch_images(host[2])
    d1 = s1.detect(host[2], o)
    d2 = s2.detect(host[2], o)
    assert d1 == d2
    with pytest.raises(sy.InvalidArgument):
        s1.prefetch_images(np.zeros((BATCH + 1, IMAGE, IMAGE, 3), np.uint8))
    s1.close()
    s2.close()
