"""A karpathy / llama2.c checkpoint runs through the decode path once converted: the
greedy tokens of the GPU (token-by-token and batched prefill, device loop) equal the
oracle's on the converted model."""
from __future__ import annotations

import numpy as np
import pytest

import fiber_b200 as fb
from oracle import oracle as orc
from test_karpathy import write_bin

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shared", [True, False])
def test_converted_checkpoint_decodes_like_the_oracle(tmp_path, shared):
    b, g = str(tmp_path / "k.bin"), str(tmp_path / "k.gguf")
    write_bin(b, shared=shared, seq=256, seed=9)
    fb.karpathy_to_gguf(b, g)
    hm = fb.HostModel(g)
    prompt = np.random.default_rng(4).integers(1, hm.params.vocab_size, 20).astype(np.int32)
    want = orc.Model(g).state(256, kv_fp16=True).generate(prompt, 30)
    ctx = fb.Context(hm, max_seq=256)
    for mode in (0, 1):  # batched prefill, then token by token
        ctx.set_prefill_mode(mode)
        kv = ctx.kv(256)
        first = ctx.prefill(kv, prompt)
        dev, _ = ctx.decode_greedy(kv, first, len(prompt), 30)
        assert first == want[0]
        assert dev.tolist() == want[1:].tolist()
