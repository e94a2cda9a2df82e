"""Device sampler (fiber_sample, fiber_decode_sample) against the host sampler, which is the
reference sampler's procedure (src/sampler.c:48-112): the same token for every draw of a
seeded sequence, over temperatures, top-k (1, 40, 1024, the whole vocabulary), top-p and
logits with ties; and a sampling decode loop on the device equal to a host-driven loop."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import fiber_b200 as fb

pytestmark = pytest.mark.gpu


def _host_draws(logits_rows, temperature, top_k, top_p):
    st = fb.Sampler()
    fb.host().sampler_init(C.byref(st), logits_rows.shape[1], temperature, top_k, top_p)
    return [int(fb.host().sampler_sample(C.byref(st), np.ascontiguousarray(r))) for r in logits_rows]


def _ref_draws(logits_rows, temperature, top_k, top_p):
    """The reference's own sampler_sample (src/sampler.c, compiled into oracle/_ref)."""
    from oracle import oracle as orc

    st = fb.Sampler()  # same layout as the reference's sampler_t (src/sampler.h)
    orc.ref().sampler_init(C.addressof(st), logits_rows.shape[1], temperature, top_k, top_p)
    return [int(orc.ref().sampler_sample(C.addressof(st), np.ascontiguousarray(r))) for r in logits_rows]


def _device_draws(logits_rows, temperature, top_k, top_p):
    """Row i drawn with the state left by rows 0..i-1 (one row at a time, one state)."""
    import torch

    n, V = logits_rows.shape
    d_lg = torch.from_numpy(np.ascontiguousarray(logits_rows)).cuda()
    d_rng = torch.tensor([42], dtype=torch.int64, device="cuda")
    d_out = torch.zeros(n, dtype=torch.int32, device="cuda")
    for i in range(n):
        fb.sample_device(d_lg[i].data_ptr(), 1, V, V, temperature, top_k, top_p, d_rng.data_ptr(),
                         d_out[i].data_ptr())
    return d_out.cpu().numpy().tolist()


@pytest.mark.parametrize("V", [1000, 32000])
@pytest.mark.parametrize("temperature,top_k,top_p", [(0.7, 40, 0.9), (1.0, 1, 1.0), (0.5, 1024, 0.95),
                                                     (1.3, 0, 1.0), (0.9, 40, 0.3), (0.0, 40, 0.9)])
def test_device_draws_equal_host_draws(V, temperature, top_k, top_p):
    if top_k == 0 and V > 49152:
        pytest.skip("unsorted case limited to 49152 entries")
    rng = np.random.default_rng(V + top_k)
    rows = (rng.standard_normal((40, V)) * 2.5).astype(np.float32)
    rows[:, 7] = rows[:, 3]  # ties: equal values keep index order
    rows[::3, 11] = rows[::3].max(axis=1)  # a tie at the top in some rows
    got = _device_draws(rows, temperature, top_k, top_p)
    assert got == _host_draws(rows, temperature, top_k, top_p)
    from oracle import oracle as orc

    if orc.ref_available():  # and the reference's own compiled sampler.c
        assert got == _ref_draws(rows, temperature, top_k, top_p)


def test_batched_rows_and_limits():
    import torch

    V = 5000
    rows = (np.random.default_rng(2).standard_normal((8, V)) * 2).astype(np.float32)
    d_lg = torch.from_numpy(rows).cuda()
    d_rng = torch.full((8,), 42, dtype=torch.int64, device="cuda")
    d_out = torch.zeros(8, dtype=torch.int32, device="cuda")
    fb.sample_device(d_lg.data_ptr(), 8, V, V, 0.8, 40, 0.9, d_rng.data_ptr(), d_out.data_ptr())
    want = [_host_draws(rows[i:i + 1], 0.8, 40, 0.9)[0] for i in range(8)]  # every row from state 42
    assert d_out.cpu().numpy().tolist() == want
    with pytest.raises(fb.FiberError):  # top_k above the device limit, below the vocabulary
        fb.sample_device(d_lg.data_ptr(), 8, V, V, 0.8, 2000, 0.9, d_rng.data_ptr(), d_out.data_ptr())


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_sampling_decode_loop_equals_host_loop(tiny_model, mode):
    hm = fb.HostModel(tiny_model("q4km"))
    ctx = fb.Context(hm, max_seq=256)
    try:
        ctx.set_mode(mode)
    except fb.FiberError:
        pytest.skip(f"decode mode {mode} does not cover this model")
    kv = ctx.kv(256)
    prompt = np.random.default_rng(5).integers(1, hm.params.vocab_size, 12).astype(np.int32)
    first = ctx.prefill(kv, prompt)
    dev, _, st = ctx.decode_sample(kv, first, len(prompt), 30, 0.8, 40, 0.9)
    # host loop: logits of each step from the GPU, token from the host sampler
    kv2 = ctx.kv(256)
    ctx.prefill(kv2, prompt)
    s = fb.Sampler()
    fb.host().sampler_init(C.byref(s), hm.params.vocab_size, 0.8, 40, 0.9)
    tok, want = first, []
    for i in range(30):
        _, lg = ctx.forward(kv2, tok, len(prompt) + i)
        tok = int(fb.host().sampler_sample(C.byref(s), lg))
        want.append(tok)
    assert dev.tolist() == want
    assert st == s.rng_state
