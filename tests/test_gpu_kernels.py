"""Kernel-level parity on the GPU through the C-ABI (fiber_gemv, fiber_dequant)
against the CPU oracle: bit-exact decoded weights, GEMV within tolerance."""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

# GEMV tolerance vs the fp32 oracle: same fp16 weights, fp32 accumulation in a
# different order -> relative RMS error ~1e-7; we allow 1e-5 relative RMS and
# 1e-4 * scale absolute.
REL_RMS = 1e-5


def _dev(a: np.ndarray):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _rel_rms(a, b):
    return float(np.sqrt(np.mean((a.astype(np.float64) - b) ** 2)) / (np.sqrt(np.mean(b.astype(np.float64) ** 2)) + 1e-30))


@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q5_K, fb.GGML_Q6_K])
@pytest.mark.parametrize("rows,cols", [(48, 1024), (37, 2048), (5, 256)])
def test_dequant_bit_exact(t, rows, cols):
    import torch

    blocks = fb.random_blocks(t, rows, cols, seed=rows * 7 + cols)
    dw = _dev(blocks)
    if t == fb.GGML_Q5_K:
        out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        fb.dequant(t, dw.data_ptr(), out.data_ptr(), rows, cols)
        torch.cuda.synchronize()
        want = orc.dequant_f32(t, blocks, rows, cols)
        assert np.array_equal(out.cpu().numpy().reshape(rows, cols).view(np.uint32), want.view(np.uint32))
    else:
        out = torch.empty(rows * cols, dtype=torch.int16, device="cuda")
        fb.dequant(t, dw.data_ptr(), out.data_ptr(), rows, cols)
        torch.cuda.synchronize()
        want = orc.dequant_f16(t, blocks, rows, cols).view(np.uint16)
        assert np.array_equal(out.cpu().numpy().view(np.uint16).reshape(rows, cols), want)


@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q5_K, fb.GGML_Q6_K])
def test_gemv_one_hot_reads_back_exact_weights(t):
    """With x = e_k the GEMV returns column k of the decoded weights exactly,
    so the fused decode inside the GEMV is bit-exact too."""
    import torch

    rows, cols = 64, 512
    blocks = fb.random_blocks(t, rows, cols, seed=99)
    want = orc.dequant_f32(t, blocks, rows, cols)
    dw = _dev(blocks)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    for k in [0, 1, 31, 32, 63, 64, 100, 127, 128, 200, 255, 256, 300, 511]:
        x = np.zeros(cols, np.float32)
        x[k] = 1.0
        dx = _dev(x)
        fb.gemv(t, dw.data_ptr(), dx.data_ptr(), y.data_ptr(), rows, cols)
        torch.cuda.synchronize()
        # exact equality (a -0.0 weight times 1.0 plus +0.0 terms reads back as +0.0)
        assert np.array_equal(y.cpu().numpy(), want[:, k]), k


@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q5_K, fb.GGML_Q6_K])
@pytest.mark.parametrize("rows,cols", [(5632, 2048), (2048, 5632), (100, 256), (33, 11008)])
def test_gemv_matches_oracle(t, rows, cols):
    import torch

    blocks = fb.random_blocks(t, rows, cols, seed=rows + cols + t)
    x = fb.randn(cols, seed=cols)
    want = orc.gemv(t, blocks, x, rows, cols)
    dw, dx = _dev(blocks), _dev(x)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    fb.gemv(t, dw.data_ptr(), dx.data_ptr(), y.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert _rel_rms(got, want) < REL_RMS
    assert np.abs(got - want).max() < 1e-4 * (np.abs(want).max() + 1)


def test_gemv_config1_workload_and_host_entry():
    """The single-GEMV workload: 5632x2048 Q4_K random super-blocks, x ~ N(0,1)
    fp32; through the host-buffer entry point as a caller would use it."""
    import torch

    rows, cols = 5632, 2048
    blocks = fb.random_blocks(fb.GGML_Q4_K, rows, cols, seed=2024)
    x = fb.randn(cols, seed=7)
    want = orc.gemv(fb.GGML_Q4_K, blocks, x, rows, cols)
    dw = _dev(blocks)
    dx = torch.empty(cols, dtype=torch.float32, device="cuda")
    dy = torch.empty(rows, dtype=torch.float32, device="cuda")
    y = np.empty(rows, np.float32)
    fb.gemv_host(fb.GGML_Q4_K, dw.data_ptr(), x, y, rows, cols, dx.data_ptr(), dy.data_ptr())
    assert _rel_rms(y, want) < REL_RMS


def test_gemv_rejects_bad_shapes():
    import torch

    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(fb.FiberError):
        fb.gemv(fb.GGML_Q4_K, w.data_ptr(), w.data_ptr(), w.data_ptr(), 4, 200)
    with pytest.raises(fb.FiberError):
        fb.gemv(7, w.data_ptr(), w.data_ptr(), w.data_ptr(), 4, 256)
