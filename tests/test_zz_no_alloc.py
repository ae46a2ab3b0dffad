"""The allocation-free weight-gradient entry point (sy_cuda_conv2d_backward_filter_static).

It exists for hosts that cannot let a library call cudaMalloc (an embedding runtime or caching allocator
that has reserved all device memory for its own pool, or a serving loop that must not take the driver's
allocation locks mid-request): they pass their own device buffers and the split-K scratch is a static
device array.  Its output must equal the ordinary entry point's (which allocates its scratch) within the
TF32 tolerance the other GPU tests use, on consecutive calls that reuse the static scratch.  This file is
collected last so a failure here never hides the other tests.
"""
import numpy as np
import pytest
import torch

import simdyolo_b200 as sy
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu
TF32_TOL = 2e-3


def to_padded(arr: np.ndarray) -> torch.Tensor:
    """NCHW host array -> the library's padded channels-last layout on cuda:0."""
    n, c, h, w = arr.shape
    rows, pitch = sy.padded_rows(h, w), (c + 3) // 4 * 4
    buf = torch.zeros(n, rows, pitch, dtype=torch.float32)
    grid = buf[:, :(h + 2) * (w + 2), :].view(n, h + 2, w + 2, pitch)
    grid[:, 1:h + 1, 1:w + 1, :c] = torch.from_numpy(arr).permute(0, 2, 3, 1)
    return buf.reshape(n * rows, pitch).to("cuda:0").contiguous()


def static_wgrad(x: np.ndarray, dy: np.ndarray, k: int) -> np.ndarray:
    n, ic, h, w = x.shape
    oc = dy.shape[1]
    xp, dyp = to_padded(x), to_padded(dy)
    dw = torch.full((oc, ic, k, k), float("nan"), dtype=torch.float32, device="cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    sy.conv2d_backward_filter_static(xp.data_ptr(), dyp.data_ptr(), n, ic, oc, h, w, k, dw.data_ptr(), stream)
    return dw.cpu().numpy()


@pytest.mark.parametrize("cases", [[(2, 64, 64, 20, 20, 3, 0), (3, 80, 80, 20, 20, 3, 1)],
                                   [(2, 64, 80, 16, 24, 1, 2), (2, 64, 80, 16, 24, 1, 3)]])
def test_static_scratch_matches_allocating_entry_on_consecutive_calls(cases):
    for n, ic, oc, h, w, k, seed in cases:
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((n, ic, h, w)).astype(np.float32)
        dy = rng.standard_normal((n, oc, h, w)).astype(np.float32)
        got = static_wgrad(x, dy, k)
        want = sy.conv2d_backward_filter(x, dy, k)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, want) < TF32_TOL


def test_static_scratch_writes_only_the_callers_weight_gradient():
    """Output channels that are not a multiple of the MMA width (20 classes): the entry point writes
    exactly oc * ic * k * k floats into the caller's buffer and leaves the memory after it untouched."""
    n, ic, oc, h, w, k = 2, 64, 20, 16, 16, 1
    rng = np.random.default_rng(4)
    x = rng.standard_normal((n, ic, h, w)).astype(np.float32)
    dy = rng.standard_normal((n, oc, h, w)).astype(np.float32)
    xp, dyp = to_padded(x), to_padded(dy)
    size = oc * ic * k * k
    buf = torch.full((size + 4096,), 7.0, dtype=torch.float32, device="cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    sy.conv2d_backward_filter_static(xp.data_ptr(), dyp.data_ptr(), n, ic, oc, h, w, k, buf.data_ptr(), stream)
    out = buf.cpu().numpy()
    assert np.all(out[size:] == 7.0)
    assert rel_l2(out[:size].reshape(oc, ic, k, k), sy.conv2d_backward_filter(x, dy, k)) < TF32_TOL


def test_static_scratch_rejects_oversized_problems():
    tiny = torch.zeros(16, device="cuda:0")
    with pytest.raises(NotImplementedError, match="scratch"):
        # P3-sized batch of 64: its split-K partial sums exceed the 16 MiB static scratch
        sy.conv2d_backward_filter_static(tiny.data_ptr(), tiny.data_ptr(), 64, 64, 144, 80, 80, 3, tiny.data_ptr())
    with pytest.raises(NotImplementedError, match="input channels"):
        sy.conv2d_backward_filter_static(tiny.data_ptr(), tiny.data_ptr(), 1, 5000, 16, 8, 8, 1, tiny.data_ptr())
    with pytest.raises(NotImplementedError, match="output channels"):
        sy.conv2d_backward_filter_static(tiny.data_ptr(), tiny.data_ptr(), 1, 16, 300, 8, 8, 1, tiny.data_ptr())
