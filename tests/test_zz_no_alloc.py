"""The allocation-free greedy lm_head entry point (fiber_gemv_argmax_noalloc).

It serves callers that cannot allocate device memory where they run the step
(a host whose own pool owns all device memory, or a latency-critical loop that
cannot take cudaMalloc's implicit synchronization); its cross-CTA scratch is a
static device array. This file is named to be collected last so that a run
stopping at the first failure has run every other test before it.

The check: two calls in a row through the C-ABI give the same logits as the
existing fiber_gemv entry point and as the CPU oracle's GEMV (within the GEMV
tolerance used elsewhere), and the first index of their maximum.
"""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb

pytestmark = pytest.mark.gpu

REL_RMS = 1e-5  # same GEMV tolerance as tests/test_gpu_kernels.py


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a.astype(np.float64) - b) ** 2)) / (np.sqrt(np.mean(b.astype(np.float64) ** 2)) + 1e-30))


@pytest.mark.parametrize("t,rows,cols", [(fb.GGML_Q6_K, 32000, 2048), (fb.GGML_Q4_K, 5000, 768)])
def test_noalloc_matches_existing_gemv_twice(t, rows, cols):
    import torch

    blocks = fb.random_blocks(t, rows, cols, seed=rows + 3)
    x = fb.randn(cols, seed=11)
    dw = torch.from_numpy(blocks).cuda()
    dx = torch.from_numpy(x).cuda()
    y_ref = torch.empty(rows, dtype=torch.float32, device="cuda")
    fb.gemv(t, dw.data_ptr(), dx.data_ptr(), y_ref.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    from oracle import oracle as orc

    want = orc.gemv(t, blocks, x, rows, cols)  # the oracle: dequant.h weights, fp32 dot products
    for call in range(2):
        y = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        fb.gemv_argmax_noalloc(t, dw.data_ptr(), dx.data_ptr(), y.data_ptr(), am.data_ptr(), rows, cols)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert _rel_rms(got, ref) < REL_RMS, call
        assert np.abs(got - ref).max() < 1e-4 * (np.abs(ref).max() + 1), call
        assert int(am.item()) == int(np.argmax(got)), call
        assert int(am.item()) == int(np.argmax(ref)), call
        assert _rel_rms(got, want) < REL_RMS, call
        assert int(am.item()) == int(np.argmax(want)), call


def test_noalloc_rejects_rows_beyond_limit():
    import torch

    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(fb.FiberError, match="static scratch limit"):
        fb.gemv_argmax_noalloc(fb.GGML_Q4_K, w.data_ptr(), w.data_ptr(), w.data_ptr(), w.data_ptr(),
                               262144 + 16, 256)
