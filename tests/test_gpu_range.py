"""Activation range of the one-kernel decode step (decode mode 2).

The MMA inputs are fp16 hi/lo fragments of the staged input; each 256-element chunk
is scaled by its own power of two before the split, so the step has no fixed
activation limit. This model grows its residual stream past 1e5 (the ffn_norm
weights are 3000, the attention norms 1, so q/k/v and the fp16 KV cache stay in
range): after the first layer |x| is about 2e5 and |x * ffn_norm| about 6e8, far
beyond fp16. The step must decode it like the oracle, greedy token for token, with
logits within the usual tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def big_residual_model(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("range") / "big_residual.gguf")
    cfg = fb.synth_cfg(None, dim=256, n_layers=3, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=1000,
                       recipe="Q4_K_M", seed=21, context_length=512, ffn_norm_value=3000.0)
    return fb.write_model(path, cfg)


def test_residual_above_1e5_decodes_like_oracle(big_residual_model):
    hm = fb.HostModel(big_residual_model)
    ctx = fb.Context(hm, max_seq=128)
    ctx.set_mode(2)
    ctx.set_prefill_mode(1)  # the prompt through the same step kernel (one step per token)
    kv = ctx.kv(128)
    prompt = np.array([5, 17, 300, 42, 7, 999, 123, 64], np.int32)
    first = ctx.prefill(kv, prompt)
    n_gen = 40
    dev, _ = ctx.decode_greedy(kv, first, len(prompt), n_gen)

    om = orc.Model(big_residual_model)
    st = om.state(128, kv_fp16=True)
    want = st.generate(prompt, n_gen)
    assert first == want[0]
    assert dev.tolist() == want[1:].tolist()

    # logits of one more step, against the oracle's (relative RMS and max-abs tolerance)
    pos = len(prompt) + n_gen
    tok = int(dev[-1])
    _, got = ctx.forward(kv, tok, pos, want_logits=True)
    ref = st.forward(tok, pos)
    got = np.asarray(got, np.float32)
    rel = float(np.sqrt(np.mean((got - ref) ** 2) / np.mean(ref ** 2)))
    assert rel < 1e-3, rel
    assert float(np.abs(got - ref).max()) < 2e-2
