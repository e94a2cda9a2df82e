"""Write the committed golden fixtures from the reference's own C.

Run from the repository root after `make -C oracle` (needs oracle/_ref, i.e. the
reference tree at build time):  python tests/golden/make_golden.py
* dequant.json -- fp16 bits of src/dequant.h on seeded random Q4_K / Q6_K blocks
* forward.json -- selected logits (bit patterns) and argmax of the reference's
  cpu_forward_token (src/fiber_proof.m:56-154) on the seeded tiny model "q4km"
"""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fiber-inference_b200"), os.path.join(ROOT, "tests")]

import fiber_b200 as fb  # noqa: E402
from conftest import TINY_MODELS  # noqa: E402
from oracle import oracle as orc  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    cases = []
    for t, seed in [(fb.GGML_Q4_K, 101), (fb.GGML_Q6_K, 102)]:
        rows, cols = 2, 512
        blocks = fb.random_blocks(t, rows, cols, seed)
        bits = orc.ref_dequant_f16(t, blocks, rows, cols).view(np.uint16).reshape(-1)
        cases.append({"type": t, "rows": rows, "cols": cols, "seed": seed, "blocks": blocks.tobytes().hex(),
                      "f16_bits": bits.tolist()})
    with open(os.path.join(HERE, "dequant.json"), "w") as f:
        json.dump({"source": "reference src/dequant.h via oracle/_ref", "cases": cases}, f)

    path = "/tmp/golden_q4km.gguf"
    fb.write_model(path, fb.synth_cfg(**TINY_MODELS["q4km"]))
    rm = orc.RefModel(path)
    kv = rm.kv(64)
    steps = []
    rng = np.random.default_rng(0)
    idx = sorted(rng.choice(rm.vocab, 16, replace=False).tolist())
    for pos, tok in enumerate([1, 17, 300, 42, 7, 99]):
        lg = kv.forward(tok, pos)
        steps.append({"pos": pos, "token": tok, "idx": idx, "bits": lg[idx].view(np.uint32).tolist(),
                      "argmax": int(np.argmax(lg))})
    with open(os.path.join(HERE, "forward.json"), "w") as f:
        json.dump({"source": "reference cpu_forward_token via oracle/_ref", "model": "q4km", "steps": steps}, f)


if __name__ == "__main__":
    main()
