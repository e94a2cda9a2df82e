"""Write the full-shape parity fixtures: greedy token sequences, per-step top-2 margins and
teacher-forced logits of the oracle on the benchmark workloads at their real shapes.

Run from the repository root after `make -C oracle` (oracle/_ref adds the reference's own
cpu_forward_token run with fp32 K/V):

    python tests/golden/make_fullshape.py [name ...]      # names: see WORKLOADS

For each workload it writes tests/golden/fullshape_<name>.json (+ .npz with the logits):

* ``sha256`` of the seeded GGUF file (fiber_synth_write_gguf), so a test on another
  machine can check it rebuilt the very same model;
* ``tokens``: the prompt's greedy next token followed by the greedy decode, from the
  oracle with fp16 K/V storage (kv_fp16, the device's cache precision);
* ``margin``: per generated token, logit(top-1) - logit(top-2) of the oracle;
* ``logits`` (npz, fp16): teacher-forced logits at a few positions;
* ``ref``: when oracle/_ref exists, the reference's own cpu_forward_token (fp32 K/V, as
  src/fiber_proof.m:82-83 keeps it) run greedily on the same prompt: its first divergence
  from ``tokens`` (or null) and the oracle's margin at that step.

Workloads (seeded like bench.py):
* tinyllama: 1.1B Q4_K_M, 128-token prompt, 512 greedy steps;
* stories: fp16 stories shape, 32-token prompt, 256 steps;
* q5long: 1.1B Q5_K_M, K/V pre-filled with seeded N(0,1) fp16 values for 2048 positions,
  64 steps from token 5 (slot 0) and from tokens (5 + 7 s) % vocab for slots s = 0..7;
* llama7b: 7B Q4_K_M, 512-token prompt, 32 greedy steps.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fiber-inference_b200")]

import fiber_b200 as fb  # noqa: E402
from oracle import oracle as orc  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
SEED = 1234

# name -> (preset, prompt length, decode steps, logits positions as decode-step indices)
WORKLOADS = {
    "tinyllama": ("tinyllama", 128, 512, [0, 1, 100, 255, 511]),
    "stories": ("stories", 32, 256, [0, 1, 128, 255]),
    "q5long": ("tinyllama-q5", 2048, 64, [0, 63]),
    "llama7b": ("llama7b", 512, 32, [0, 31]),
}
Q5_SLOTS = 8


def prompt_ids(vocab: int, n: int) -> np.ndarray:
    """The benchmark's seeded prompt (bench.py: prompt_ids)."""
    return np.random.default_rng(SEED).integers(1, vocab, n).astype(np.int32)


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def model_path(name: str) -> str:
    preset = WORKLOADS[name][0]
    path = f"/tmp/fiber_fullshape_{name}.gguf"
    if not os.path.exists(path):
        fb.write_model(path + ".tmp", fb.synth_cfg(preset, seed=SEED))
        os.replace(path + ".tmp", path)
    return path


def q5_kv(layer: int, P: int, kvd: int):
    """Seeded N(0,1) K/V rows of the long-context workload, rounded to fp16 (bench.py)."""
    k = fb.randn(P * kvd, seed=100 + layer).reshape(P, kvd).astype(np.float16).astype(np.float32)
    v = fb.randn(P * kvd, seed=200 + layer).reshape(P, kvd).astype(np.float16).astype(np.float32)
    return k, v


def top2(lg: np.ndarray):
    i = int(np.argmax(lg))
    rest = lg.copy()
    rest[i] = -np.inf
    return i, float(lg[i] - rest.max())


def greedy(forward, first_pos: int, first_token: int, steps: int, want: set):
    """Greedy decode from (first_token at first_pos); returns tokens, margins, logits at want."""
    toks, margins, logits = [], [], {}
    tok, pos = first_token, first_pos
    for s in range(steps):
        lg = forward(tok, pos)
        i, m = top2(lg)
        if s in want:
            logits[s] = lg.astype(np.float16)
        toks.append(i)
        margins.append(m)
        tok, pos = i, pos + 1
    return toks, margins, logits


def run_prompted(name: str, out: dict, arrays: dict):
    preset, P, D, want = WORKLOADS[name]
    path = model_path(name)
    out["sha256"] = sha256(path)
    om = orc.Model(path)
    prompt = prompt_ids(om.vocab, P)
    st = om.state(P + D + 1, kv_fp16=True)
    t0 = time.time()
    for p in range(P - 1):
        st.forward(int(prompt[p]), p)
    # step 0 consumes the last prompt token; its argmax is the first generated token
    toks, margins, logits = greedy(st.forward, P - 1, int(prompt[P - 1]), D + 1, {w for w in want})
    out.update(prompt_len=P, decode_steps=D, tokens=toks, margin=margins,
               logits_steps=sorted(logits), oracle_s=time.time() - t0)
    for s, lg in logits.items():
        arrays[f"logits_{s}"] = lg
    st.close()
    om.close()
    # the reference's own cpu_forward_token runs single-threaded here: hours at 7B, so it
    # is run on the 1.1B-and-smaller workloads only
    if orc.ref_available() and name not in ("q5long", "llama7b"):
        rm = orc.RefModel(path)
        kv = rm.kv(P + D + 1)
        for p in range(P - 1):
            kv.forward(int(prompt[p]), p)
        rtoks, _, _ = greedy(kv.forward, P - 1, int(prompt[P - 1]), D + 1, set())
        div = next((i for i, (a, b) in enumerate(zip(toks, rtoks)) if a != b), None)
        out["ref"] = {"what": "reference cpu_forward_token (src/fiber_proof.m:56-154), fp32 K/V",
                      "first_divergence": div, "margin_at_divergence": None if div is None else margins[div],
                      "tokens": rtoks}
        kv.close()
        rm.close()


def run_q5long(out: dict, arrays: dict):
    preset, P, D, want = WORKLOADS["q5long"]
    path = model_path("q5long")
    out["sha256"] = sha256(path)
    om = orc.Model(path)
    kvd = om.n_kv_heads * om.head_dim
    kvs = [q5_kv(layer, P, kvd) for layer in range(om.n_layers)]
    t0 = time.time()
    slots = []
    for s in range(Q5_SLOTS):
        st = om.state(P + D + 1, kv_fp16=True)
        for layer, (k, v) in enumerate(kvs):
            for p in range(P):
                st.set_kv(layer, p, k[p], v[p])
        first = (5 + 7 * s) % om.vocab
        toks, margins, logits = greedy(st.forward, P, first, D, set(want) if s == 0 else set())
        slots.append({"first": first, "tokens": toks, "margin": margins})
        for st_i, lg in logits.items():
            arrays[f"logits_{st_i}"] = lg
        st.close()
    out.update(context=P, decode_steps=D, slots=slots, logits_steps=sorted(want), oracle_s=time.time() - t0)
    om.close()


def main(names):
    for name in names:
        out, arrays = {"workload": name, "preset": WORKLOADS[name][0], "seed": SEED,
                       "source": "oracle/oracle.c (kv_fp16) restating src/fiber_proof.m:23-154"}, {}
        t0 = time.time()
        if name == "q5long":
            run_q5long(out, arrays)
        else:
            run_prompted(name, out, arrays)
        out["wall_s"] = time.time() - t0
        with open(os.path.join(HERE, f"fullshape_{name}.json"), "w") as f:
            json.dump(out, f)
        np.savez_compressed(os.path.join(HERE, f"fullshape_{name}.npz"), **arrays)
        mm = min(out["margin"]) if "margin" in out else min(min(s["margin"]) for s in out["slots"])
        print(f"{name}: done in {out['wall_s']:.0f} s, min margin {mm:.3g}, ref {out.get('ref', {}).get('first_divergence')}",
              flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or list(WORKLOADS))
