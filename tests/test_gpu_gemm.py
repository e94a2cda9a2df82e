"""Tensor-core dequant-GEMM (fiber_gemm, tcgen05) against a float64 product of the
exactly decoded weights: the same fp16 weights the GEMV uses, inputs split into fp16
hi + lo parts, fp32 accumulation -> relative RMS error ~1e-7; the bar is 1e-5 relative
RMS and 1e-4 of the output scale max-abs. Covers partial row and token tiles, the
RMSNorm fold-in and the accumulate (residual) form."""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

REL_RMS = 1e-5


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _weights(t, rows, cols, seed):
    """(device blocks, float64 decoded weights [rows][cols])"""
    if t == fb.GGML_F16:
        w = (np.random.default_rng(seed).standard_normal((rows, cols)) * 0.05).astype(np.float16)
        return _dev(w.view(np.uint8).reshape(-1)), w.astype(np.float64)
    blocks = fb.random_blocks(t, rows, cols, seed=seed)
    if t == fb.GGML_Q5_K:  # fp32 weights (the Metal kernel's arithmetic)
        w = orc.dequant_f32(t, blocks, rows, cols).astype(np.float64)
    else:
        w = orc.dequant_f16(t, blocks, rows, cols).astype(np.float64)
    # Q6_K rows are read through 16-byte-aligned spans: keep 14+ readable bytes after
    padded = np.concatenate([np.asarray(blocks, dtype=np.uint8).reshape(-1), np.zeros(256, np.uint8)])
    return _dev(padded), w


@pytest.mark.parametrize("t", [fb.GGML_Q4_K, fb.GGML_Q5_K, fb.GGML_Q6_K, fb.GGML_F16])
@pytest.mark.parametrize("rows,cols,ntok", [(300, 512, 70), (128, 256, 1), (256, 2048, 64), (130, 768, 129)])
def test_gemm_matches_decoded_product(t, rows, cols, ntok):
    import torch

    dw, w = _weights(t, rows, cols, seed=rows + cols + ntok)
    rng = np.random.default_rng(ntok)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    y = torch.full((ntok, rows), float("nan"), dtype=torch.float32, device="cuda")
    dx = _dev(x)
    fb.gemm(t, dw.data_ptr(), rows, cols, dx.data_ptr(), ntok, y.data_ptr(), rows)
    got = y.cpu().numpy()
    want = x.astype(np.float64) @ w.T
    assert np.isfinite(got).all()
    err = np.sqrt(np.mean((got - want) ** 2) / np.mean(want ** 2))
    assert err < REL_RMS, err
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max()


def test_gemm_norm_and_accumulate():
    import torch

    t, rows, cols, ntok = fb.GGML_Q4_K, 384, 1024, 40
    dw, w = _weights(t, rows, cols, seed=5)
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((ntok, cols)) * 3).astype(np.float32)
    rr = (1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(1) + 1e-5)).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    base = rng.standard_normal((ntok, rows + 16)).astype(np.float32)
    y = _dev(base.copy())
    dx, drr, dnw = _dev(x), _dev(rr), _dev(nw)
    fb.gemm(t, dw.data_ptr(), rows, cols, dx.data_ptr(), ntok, y.data_ptr(), rows + 16, out_off=16,
            d_rrms=drr.data_ptr(), d_nw=dnw.data_ptr(), accumulate=True)
    got = y.cpu().numpy()
    xn = (x * rr[:, None]).astype(np.float32) * nw[None, :]
    want = base.astype(np.float64).copy()
    want[:, 16:] += xn.astype(np.float64) @ w.T
    assert np.array_equal(got[:, :16], base[:, :16])  # outside the output window: untouched
    err = np.sqrt(np.mean((got - want) ** 2) / np.mean(want ** 2))
    assert err < REL_RMS, err


def test_gemm_rejects_bad_shapes():
    with pytest.raises(fb.FiberError):
        fb.gemm(fb.GGML_Q4_K, 1, 128, 200, 1, 4, 1, 128)  # cols not a multiple of 256
    with pytest.raises(fb.FiberError):
        fb.gemm(fb.GGML_F32, 16, 128, 256, 16, 4, 16, 128)  # type not covered
