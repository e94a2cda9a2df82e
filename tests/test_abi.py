"""The C-ABI libraries load without a GPU and export every function the public
headers declare."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re

import fiber_b200 as fb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", re.M)


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"typedef[^;]*;", "", text)  # types (function-pointer typedefs included)
        for m in DECL.finditer(text):
            name = m.group(1)
            if name in {"if", "sizeof", "defined"}:
                continue
            names.add(name)
    return names


def test_headers_declare_expected_entry_points():
    names = declared_functions()
    for must in ["gpu_init", "gpu_forward_token", "gpu_get_logits", "kv_cache_init", "fiber_forward_token",
                 "fiber_gemv", "gguf_open", "model_open", "tokenizer_encode", "sampler_sample"]:
        assert must in names


def test_every_declared_function_is_exported():
    host = C.CDLL(fb.HOST_SO)
    cuda = C.CDLL(fb.CUDA_SO)
    missing = []
    for name in sorted(declared_functions()):
        if not (hasattr(host, name) or hasattr(cuda, name)):
            missing.append(name)
    assert not missing, missing


def test_cuda_library_reports_errors_without_gpu_work():
    L = fb.cuda_lib()
    # argument validation happens before any device call
    rc = L.fiber_gemv(99, None, None, None, 1, 256, None)
    assert rc == -1
    assert b"not supported" in L.fiber_last_error()
    rc = L.fiber_gemv(fb.GGML_Q4_K, None, None, None, 16, 100, None)
    assert rc == -1
    assert L.fiber_cuda_init(None, 0, 1, 16) is None
