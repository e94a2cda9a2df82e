"""Shared test setup: markers, import paths, build-on-demand of the libraries,
and small seeded synthetic models written once per session."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fiber-inference_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size workloads")


def _ensure_built():
    libs = [os.path.join(PKG, "lib", "libfiber_host.so"), os.path.join(PKG, "lib", "libfiber_cuda.so"),
            os.path.join(ROOT, "oracle", "liboracle.so")]
    if all(os.path.exists(p) for p in libs):
        return
    subprocess.run(["make", "-C", PKG, "host", "cuda"], check=True, capture_output=True)
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True, capture_output=True)


_ensure_built()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


# name -> synthetic config overrides (small shapes the oracle runs in milliseconds)
TINY_MODELS = {
    "q4km": dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, vocab=1000, recipe="Q4_K_M", seed=11,
                 context_length=512),
    "q5km": dict(dim=512, n_layers=2, n_heads=8, n_kv_heads=1, ffn_dim=768, vocab=800, recipe="Q5_K_M", seed=12,
                 context_length=512),
    "f16": dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=512, vocab=700, recipe="F16", seed=13,
                context_length=512, tied=1),
    "q6k": dict(dim=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn_dim=256, vocab=600, recipe="Q6_K", seed=14,
                context_length=512),
    "gqa8": dict(dim=512, n_layers=3, n_heads=8, n_kv_heads=1, ffn_dim=1024, vocab=1200, recipe="Q4_K_M",
                 seed=15, context_length=1024),
    "hd128": dict(dim=512, n_layers=2, n_heads=4, n_kv_heads=4, ffn_dim=768, vocab=900, recipe="Q4_K_M", seed=16,
                  context_length=512),
    # splits over 2 ranks: 4 query / 2 KV heads and 2 of 4 FFN super-blocks each; Q4_K_M puts
    # Q6_K on attn_v / ffn_down of layer 0, so both shard paths (144- and 210-byte blocks) run
    "tp": dict(dim=512, n_layers=3, n_heads=8, n_kv_heads=4, ffn_dim=1024, vocab=1100, recipe="Q4_K_M", seed=17,
               context_length=512),
    # splits over 4 ranks: 4 query / 1 KV head each, 11 FFN super-blocks as 2/3/3/3 (uneven,
    # like the 7B FFN's 43 blocks over 4 ranks)
    "tp4": dict(dim=1024, n_layers=2, n_heads=16, n_kv_heads=4, ffn_dim=2816, vocab=1100, recipe="Q4_K_M",
                seed=18, context_length=512),
}


@pytest.fixture(scope="session")
def tiny_model(model_dir):
    import fiber_b200 as fb

    cache = {}

    def get(name: str) -> str:
        if name not in cache:
            path = str(model_dir / f"{name}.gguf")
            fb.write_model(path, fb.synth_cfg(**TINY_MODELS[name]))
            cache[name] = path
        return cache[name]

    return get
