"""The fiber-inference command-line driver (the reference's main.m flags).

CPU: --help, a missing --model and --list-tensors (no GPU needed before the model
is listed). GPU: a greedy run (--temperature 0) prints the same tokens the oracle
generates from the prompt ids the CLI reports (--ids), and the reference's
"--- Stats ---" block with Prefill / Decode throughput (src/main.m:553-603).
"""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "fiber-inference_b200", "bin", "fiber-inference")


def _exe():
    if not os.path.exists(EXE):
        subprocess.run(["make", "-C", os.path.join(ROOT, "fiber-inference_b200"), "cli"], check=True,
                       capture_output=True)
    return EXE


def test_help_and_missing_model():
    r = subprocess.run([_exe(), "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0
    for flag in ("--model", "--prompt", "--tokens", "--ctx-len", "--temperature", "--top-k", "--top-p"):
        assert flag in r.stderr
    r = subprocess.run([_exe(), "--prompt", "x"], capture_output=True, text=True, timeout=60)
    assert r.returncode != 0 and "--model is required" in r.stderr


def test_list_tensors(tiny_model):
    r = subprocess.run([_exe(), "--model", tiny_model("q4km"), "--list-tensors"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert "token_embd.weight" in r.stdout and "blk.1.ffn_down.weight" in r.stdout


def _ids(text, label):
    m = re.search(rf"^{label}:((?: \d+)*)$", text, re.M)
    assert m, text
    return [int(v) for v in m.group(1).split()]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q4km", "gqa8"])
def test_greedy_run_matches_oracle(tiny_model, name):
    path = tiny_model(name)
    n = 32
    r = subprocess.run([_exe(), "--model", path, "--prompt", "Hello world, this is a test", "--tokens", str(n),
                        "--temperature", "0", "--ids"], capture_output=True, text=True, errors="replace",
                       timeout=600)
    assert r.returncode == 0, r.stderr
    assert "--- Stats ---" in r.stdout and "Prefill:" in r.stdout and "Decode:" in r.stdout
    prompt = _ids(r.stderr, "prompt ids")
    got = _ids(r.stderr, "generated ids")
    assert len(prompt) > 1 and len(got) >= 1
    om = orc.Model(path)
    want = om.state(len(prompt) + n + 1, kv_fp16=True).generate(np.array(prompt, np.int32), n)
    assert got == want.tolist()[: len(got)]
