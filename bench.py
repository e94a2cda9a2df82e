"""Benchmark: batch-1 greedy decode of the 1.1B (TinyLlama-shape) Q4_K_M model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fiber|reference]

Workload (seeded synthetic model, random init, weights N(0, 0.02) quantized with
the Q4_K_M recipe): dim 2048, 22 layers, 32 query / 4 KV heads, head_dim 64,
SwiGLU 5632, vocab 32000. A 128-token seeded prompt is prefilled once; one
*step* is 512 greedy decode tokens at positions 128..639 (each step restarts at
position 128 and overwrites the same KV rows). ``value`` is decode tokens/s with
all inputs resident in HBM, timed with CUDA events on the decode stream (the
weights, 633 MB per token, exceed the 126 MB L2, so no flush is needed).
``e2e`` is the same loop through the public C call fiber_forward_token with
host buffers: every token copies its inputs in and its argmax out.
With --gpus N (torchrun) every rank decodes its own replica (weak scaling:
the model fits one GPU and the decode loop has no data-parallel exchange).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "fiber-inference_b200")]

METRIC = "decode tok/s (1.1B Q4_K_M, bs=1); dequant-GEMV HBM GB/s vs B200 peak"
PROMPT_LEN, DECODE_LEN, SEED = 128, 512, 1234
MODEL_PATH = "/tmp/fiber_bench_tinyllama_q4km.gguf"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, device: int):
        self.device, self.samples, self.proc = device, [], None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([s.strip() for s in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx = float(s[2])
                for n, v in zip(names, s[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# DRAM traffic of one decode_persistent_kernel launch from an ncu capture (decode step at
# position 13): dram__bytes_read.sum + dram__bytes_write.sum, and that launch's algorithmic bytes.
# dram__bytes_read.sum + dram__bytes_write.sum of one step-kernel launch under ncu (profiles/),
# with the algorithmic bytes of that launch's KV position
PK_CAPTURE = {"dram_bytes": 635_233_536 + 6_902_784, "algorithmic_bytes": 633_700_000, "position": 13}
FL_CAPTURE = {"dram_bytes": 639_928_832 + 7_345_152, "algorithmic_bytes": 639_348_864, "position": 132}


def traffic_of(mode: int, roof: dict) -> dict:
    """Per-launch DRAM traffic of the dominant kernel, scaled from the ncu capture by the
    algorithmic bytes of the timed launches (traffic tracks the bytes streamed)."""
    cap = {0: PK_CAPTURE, 2: FL_CAPTURE}.get(mode)
    if cap is None:
        return {"traffic": None}
    ratio = cap["dram_bytes"] / cap["algorithmic_bytes"]
    return {"traffic": roof["algorithmic_bytes_per_launch"] * ratio,
            "traffic_source": f"ncu capture at position {cap['position']}: traffic/algorithmic = {ratio:.3f}, "
                              "scaled to the timed launches' algorithmic bytes"}


def make_model(path: str):
    import fiber_b200 as fb

    if not os.path.exists(path):
        tmp = path + f".{os.getpid()}.tmp"
        fb.write_model(tmp, fb.synth_cfg("tinyllama", seed=SEED))
        os.replace(tmp, path)
    return path


def prompt_ids(vocab: int) -> np.ndarray:
    return np.random.default_rng(SEED).integers(1, vocab, PROMPT_LEN).astype(np.int32)


def gemv_bandwidth(device: int, n_launch: int = 400, reps: int = 5):
    """Single Q4_K GEMV 5632x2048 (random super-blocks), 40 rotating weight
    copies (260 MB > L2). The launches are captured once in a CUDA graph so the
    timing (CUDA events on the capturing stream) sees the GPU, not the Python
    launch loop."""
    import torch

    import fiber_b200 as fb

    rows, cols, copies = 5632, 2048, 40
    blocks = fb.random_blocks(fb.GGML_Q4_K, rows, cols, seed=2024)
    w = torch.from_numpy(np.tile(blocks, copies)).to(f"cuda:{device}")
    nb = blocks.size
    x = torch.from_numpy(fb.randn(cols, seed=7)).to(f"cuda:{device}")
    y = torch.empty(rows, dtype=torch.float32, device=f"cuda:{device}")
    base = w.data_ptr()
    st = torch.cuda.Stream(device)
    with torch.cuda.stream(st):
        for i in range(copies):
            fb.gemv(fb.GGML_Q4_K, base + i * nb, x.data_ptr(), y.data_ptr(), rows, cols, st)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(n_launch):
                fb.gemv(fb.GGML_Q4_K, base + (i % copies) * nb, x.data_ptr(), y.data_ptr(), rows, cols, st)
        g.replay()
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
        e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (n_launch * reps)
    algo = rows * cols // 256 * 144 + cols * 4 + rows * 4
    return {"workload": "Q4_K GEMV 5632x2048, x fp32, 40 rotating weight copies, graph of back-to-back launches",
            "us_per_launch": us, "algorithmic_bytes": algo, "gbs": algo / us / 1e3}


def omp_threads(n: int):
    """Thread count of the OpenMP runtime the CPU checker libraries use."""
    import ctypes

    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except OSError:
        pass


class CpuReference:
    """The reference's own C path on the host cores: fiber_model_t built by gguf.c +
    dequant.h, cpu_forward_token with an OpenMP cblas_sgemv stand-in (oracle/_ref);
    the restated oracle when _ref is absent. Starts like the GPU arm: the seeded
    128-token prompt prefilled token by token (the reference's own prefill loop), so
    decode tokens are timed from position 128 on."""

    def __init__(self, path: str, prefill: bool = True):
        from oracle import oracle as orc

        if orc.ref_available():
            self.m, self.kind = orc.RefModel(path), "reference"
            self.kv = self.m.kv(PROMPT_LEN + DECODE_LEN)
            self.fwd = self.kv.forward
        else:
            self.m, self.kind = orc.Model(path), "port"
            self.kv = self.m.state(PROMPT_LEN + DECODE_LEN, kv_fp16=False)
            self.fwd = self.kv.forward
        self.pos, self.tok = 0, 1
        if prefill:
            prompt = prompt_ids(32000)
            for t in prompt:
                lg = self.fwd(int(t), self.pos)
                self.pos += 1
            self.tok = int(np.argmax(lg))

    def decode(self, n: int) -> float:
        """n greedy tokens from the current position; returns seconds."""
        t0 = time.perf_counter()
        for _ in range(n):
            lg = self.fwd(self.tok, self.pos)
            self.tok = int(np.argmax(lg))
            self.pos += 1
        return time.perf_counter() - t0


def cpu_reference_decode(path: str, budget_s: float, n_tokens_max: int):
    """Bounded CPU baseline sample for the GPU arm's line: greedy tokens at positions
    0.. (no prompt, to keep the leg within seconds) on all host threads, then a few on
    one thread."""
    cores = os.cpu_count()
    omp_threads(cores)
    ref = CpuReference(path, prefill=False)
    n, t = 0, 0.0
    while n < n_tokens_max and (n < 2 or t < budget_s):
        t += ref.decode(1)
        n += 1
    omp_threads(1)
    n1, t1 = 0, 0.0
    while n1 < 2 or (t1 < budget_s / 2 and n1 < 8):
        t1 += ref.decode(1)
        n1 += 1
    omp_threads(cores)
    return {"value": n / t, "unit": "tok/s", "cores": cores, "kind": ref.kind,
            "single_thread": {"value": n1 / t1, "unit": "tok/s", "cores": 1,
                              "sample": f"{n1} greedy decode tokens after the {n} above"},
            "sample": f"{n} greedy decode tokens at positions 0..{n - 1} of the same model, fp32 weights "
                      f"(4.4 GB) via OpenMP sgemv on {cores} threads"}


def run_reference(args, rank: int, world: int):
    """The reference arm: the reference's own CPU decode on this workload (seeded 128-token
    prompt prefilled token by token, then greedy decode from position 128, as the GPU arm
    decodes positions 128..639), every step a bounded sample of 4 decode tokens."""
    if rank != 0:
        return
    path = make_model(MODEL_PATH)
    per_step = 4
    cores = os.cpu_count()
    omp_threads(cores)
    t0 = time.perf_counter()
    ref = CpuReference(path, prefill=True)
    prefill_s = time.perf_counter() - t0
    for _ in range(args.warmup):
        ref.decode(per_step)
    secs = sum(ref.decode(per_step) for _ in range(args.steps))
    value = per_step * args.steps / secs
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random init)",
            "impl": "reference",
            "config": {"workload": "1.1B Q4_K_M (TinyLlama shape) batch-1 greedy decode",
                       "model": "dim 2048, 22 layers, 32/4 heads, hd 64, ffn 5632, vocab 32000, Q4_K_M",
                       "prompt": PROMPT_LEN, "global_batch": 1, "parallelism": "replicas x1",
                       "step": f"{per_step} decode tokens", "positions": f"{PROMPT_LEN}..{ref.pos - 1}",
                       "prefill_s": prefill_s},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": ref.kind,
                             "sample": f"{per_step * (args.warmup + args.steps)} greedy decode tokens at positions "
                                       f"{PROMPT_LEN}..{ref.pos - 1} after the seeded {PROMPT_LEN}-token prompt, "
                                       f"fp32 weights (4.4 GB) via OpenMP sgemv on {cores} threads"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


MODEL_7B = "/tmp/fiber_bench_llama7b_q4km.gguf"
# Q4_K_M 7B: 32 layers x (Q4_K 113,836,032 B or Q6_K-recipe 129,785,856 B) + Q6_K output 107,520,000 B
WEIGHTS_7B = 16 * 113_836_032 + 16 * 129_785_856 + 107_520_000 + 32 * 2 * 16_384 + 16_384 + 2_304


def step_phase_times(ctx, kv, first: int, pos: int) -> dict:
    """Critical-path time of each phase kind of the one-kernel step at KV position pos, from
    the step's own per-phase timeline (fiber_trace_step): for phase k, the latest CTA end of
    phase k minus the latest CTA end of phase k - 1, averaged over the layers (microseconds)."""
    tr = None
    for _ in range(3):  # the last of three (warm) traced steps
        tr = ctx.trace_step(kv, first, pos)
    if ctx.mode == 2:
        end = tr[:, :, ctx.FLOW_TRACE_FIELDS.index("t_end_ns")].astype(np.int64)
        start = tr[:, :, ctx.FLOW_TRACE_FIELDS.index("t_start_ns")].astype(np.int64)
    else:
        end = tr[:, :, ctx.TRACE_FIELDS.index("t_release_ns")].astype(np.int64)
        start = end
    n = tr.shape[0]
    ends = np.array([end[k][end[k] > 0].max() for k in range(n)], dtype=np.float64)
    names = ["qkv", "attention", "wo", "gate_up", "down"]
    out = {k: [] for k in names}
    for k in range(1, n - 1):
        out[names[k % 5]].append((ends[k] - ends[k - 1]) / 1e3)
    res = {k: float(np.mean(v)) for k, v in out.items() if v}
    res["lm_head"] = float((ends[n - 1] - ends[n - 2]) / 1e3)
    s0 = start[0][start[0] > 0].min()
    res["step_us"] = float((ends[n - 1] - s0) / 1e3)
    res["position"] = pos
    return res


def measure_7b_tp(fb, torch, dist, rank, world, local, P: int, D: int, steps: int, warmup: int) -> dict:
    """7B Q4_K_M batch-1 greedy decode, tensor-parallel over the N ranks (one process per
    GPU; the Wo and W_down partial sums all-reduced inside each step). Every rank returns
    the same dict: decode tok/s from CUDA events (max over ranks), the collective used and
    whether all ranks produced the same tokens."""
    if rank == 0 and not os.path.exists(MODEL_7B):
        fb.write_model(MODEL_7B + ".tmp", fb.synth_cfg("llama7b"))
        os.replace(MODEL_7B + ".tmp", MODEL_7B)
    box = [fb.tp_unique_id() if rank == 0 else None]
    if dist is not None:
        dist.barrier()
        dist.broadcast_object_list(box, src=0)
    hm = fb.HostModel(MODEL_7B)
    ctx = fb.Context(hm, device=local, max_seq=P + D, tp=(rank, world, box[0]))
    kv = ctx.kv(P + D)
    prompt = prompt_ids(hm.params.vocab_size)[:P]
    t0 = time.perf_counter()
    first = ctx.prefill(kv, prompt)
    prefill_tps = P / (time.perf_counter() - t0)
    for _ in range(warmup):
        ctx.decode_greedy(kv, first, P, D)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(local)
    ms_total, toks0 = 0.0, None
    with Clocks(local) as clk:
        for _ in range(steps):
            toks, ms = ctx.decode_greedy(kv, first, P, D)
            ms_total += ms
            toks0 = toks if toks0 is None else toks0
    if dist is not None:
        t = torch.tensor([ms_total], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        h = torch.tensor([int(np.sum(toks0.astype(np.int64) * np.arange(1, D + 1)))], device=f"cuda:{local}")
        hs = [torch.zeros_like(h) for _ in range(world)]
        dist.all_gather(hs, h)
        same = all(int(x.item()) == int(h.item()) for x in hs)
    else:
        same = True
    value = steps * D / (ms_total / 1e3)
    peak, peak_kind = peaks()
    kv_bytes = 524_288 * (P + D / 2)  # mean KV read per token over the decode positions
    bytes_tok = WEIGHTS_7B + kv_bytes
    out = {"value": value, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
           "ms_per_step": ms_total / steps, "prompt": P, "decode_tokens_per_step": D, "parallelism": f"tp{world}",
           "collective": {0: "none (one GPU)", 1: "NCCL all-reduce", 2: "one-shot peer-memory all-reduce",
                          3: "fused into the step: peer stores of the Wo / W_down partial sums, summed by "
                             "the next phase"}[ctx.tp_collective],
           "step_mode": STEP_MODES[ctx.mode] + (", exchange after Wo and W_down" if world > 1 else ""),
           "tokens_identical_on_all_ranks": same, "prefill_tok_s": prefill_tps,
           "roofline": {"bound": "hbm", "achieved": bytes_tok * value / world / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": bytes_tok * value / world / 1e9 / peak, "peak_source": peak_kind,
                        "algorithmic_bytes_per_token": bytes_tok,
                        "note": "per GPU: weights and KV of the whole model divided over the ranks"},
           "gpu_launches": ctx.step_launches() * D * steps, "clocks": clk.summary()}
    ctx.close()
    if dist is not None:
        dist.barrier()
    return out


def run_7b_tp(args, fb, torch, dist, rank, world, local):
    """Config 5: 7B Q4_K_M (dim 4096, 32 layers, 32 heads, hd 128, ffn 11008) batch-1 greedy
    decode, tensor-parallel over the N ranks (one process per GPU; all-reduce after Wo
    and W_down inside each step). Total work is fixed: scaling is strong."""
    # config 5: 512-token prompt, 256 decode steps (shorter only when asked for)
    P = 512 if args.prompt_len == PROMPT_LEN else args.prompt_len
    D = 256 if args.decode_len == DECODE_LEN else args.decode_len
    r = measure_7b_tp(fb, torch, dist, rank, world, local, P, D, args.steps, args.warmup)
    if rank == 0:
        line = {"metric": "decode tok/s (7B Q4_K_M, bs=1, tensor-parallel)", "value": r["value"], "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init weights, seeded prompt ids)",
                "config": {"workload": "7B Q4_K_M (Llama-2-7B shape) batch-1 greedy decode, tensor-parallel",
                           "model": "dim 4096, 32 layers, 32/32 heads, hd 128, ffn 11008, vocab 32000, Q4_K_M",
                           "prompt": P, "decode_tokens_per_step": D, "global_batch": 1,
                           "parallelism": f"tp{world}", "step_mode": r["step_mode"] + " (" + r["collective"] + ")",
                           "tokens_identical_on_all_ranks": r["tokens_identical_on_all_ranks"],
                           "prefill_tok_s": r["prefill_tok_s"]},
                "roofline": dict(r["roofline"], traffic=None),
                "gpu_launches": r["gpu_launches"], "clocks": r["clocks"]}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


CONFIG_NAMES = {"stories": "stories fp16 (dim 768, 12 layers, 12 heads, ffn 2048, vocab 32000, tied)",
                "q5km-long": "1.1B Q5_K_M (TinyLlama shape), KV pre-filled to 2048 positions"}
STEP_MODES = {0: "persistent kernel per token", 1: "one kernel per phase", 2: "dataflow kernel per token"}


def measure_config(fb, torch, dist, rank, world, local, workload: str, D: int, steps: int, warmup: int) -> dict:
    """Configs 2 and 4 at batch 1 (one replica per rank): the fp16 stories-shaped model with a
    32-token prompt, or the 1.1B Q5_K_M model decoding after its KV cache was pre-filled with
    seeded N(0,1) fp16 keys/values for 2048 positions. Returns the measurement as a dict."""
    if workload == "stories":
        path, preset, P = "/tmp/fiber_bench_stories_f16.gguf", "stories", 32
    else:
        path, preset, P = "/tmp/fiber_bench_tinyllama_q5km.gguf", "tinyllama-q5", 2048
    if not os.path.exists(path):
        tmp = path + f".{os.getpid()}.tmp"
        fb.write_model(tmp, fb.synth_cfg(preset, seed=SEED))
        os.replace(tmp, path)
    hm = fb.HostModel(path)
    p = hm.params
    ctx = fb.Context(hm, device=local, max_seq=P + D)
    kv = ctx.kv(P + D)
    kvd = p.n_kv_heads * p.head_dim
    if workload == "stories":
        first = ctx.prefill(kv, prompt_ids(p.vocab_size)[:P])
    else:
        for layer in range(p.n_layers):
            kv.write(layer, 0, fb.randn(P * kvd, seed=100 + layer).reshape(P, kvd),
                     fb.randn(P * kvd, seed=200 + layer).reshape(P, kvd))
        first = 5
    for _ in range(warmup):
        ctx.decode_greedy(kv, first, P, D)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(local)
    ms_total = 0.0
    with Clocks(local) as clk:
        for _ in range(steps):
            _, ms = ctx.decode_greedy(kv, first, P, D)
            ms_total += ms
    if dist is not None:
        t = torch.tensor([ms_total], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    value = world * steps * D / (ms_total / 1e3)
    mid = P + D // 2
    step_bytes = 0.0
    for kind in range(7):
        _, b = ctx.time_kernel(kv, kind, mid, reps=2)
        step_bytes += b * (1 if kind >= 5 else p.n_layers)
    peak, peak_kind = peaks()
    out = {"value": value, "unit": "tok/s", "ms_per_step": ms_total / steps, "steps": steps, "warmup": warmup,
           "workload": CONFIG_NAMES[workload], "context": P, "decode_tokens_per_step": D,
           "dtype": "f32" if workload != "stories" else "f16 weights, f32 activations",
           "step_mode": STEP_MODES[ctx.mode],
           "roofline": {"bound": "hbm", "achieved": step_bytes * value / world / 1e9, "peak": peak,
                        "unit": "GB/s", "frac": step_bytes * value / world / 1e9 / peak,
                        "peak_source": peak_kind, "traffic": None,
                        "algorithmic_bytes_per_token": step_bytes, "kv_position": mid},
           "gpu_launches": ctx.step_launches() * D * steps, "clocks": clk.summary()}
    ctx.close()
    return out


def run_config(args, fb, torch, dist, rank, world, local):
    """Configs 2 and 4 at batch 1 as their own bench line (256 decode steps)."""
    D = 256 if args.decode_len == DECODE_LEN else args.decode_len
    r = measure_config(fb, torch, dist, rank, world, local, args.workload, D, args.steps, args.warmup)
    if rank == 0:
        line = {"metric": f"decode tok/s ({args.workload}, bs=1)", "value": r["value"], "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": r["dtype"],
                "data": "synthetic (seeded random-init weights; seeded prompt ids or seeded N(0,1) KV)",
                "config": {"workload": r["workload"], "context": r["context"], "decode_tokens_per_step": D,
                           "global_batch": 1, "parallelism": f"replicas x{world}", "step_mode": r["step_mode"]},
                "roofline": r["roofline"], "gpu_launches": r["gpu_launches"], "clocks": r["clocks"]}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_prefill(args, fb, torch, dist, rank, world, local):
    """Batched prefill of a 512-token prompt (1.1B Q4_K_M): tokens/s through fiber_prefill and the
    tensor-core GEMM throughput it implies (2 x params FLOPs per token; the kernels run twice the
    columns for the hi/lo split of x, reported separately)."""
    P = 512 if args.prompt_len == PROMPT_LEN else args.prompt_len
    path = MODEL_PATH if world == 1 else MODEL_PATH.replace(".gguf", f".r{rank}.gguf")
    make_model(path)
    hm = fb.HostModel(path)
    p = hm.params
    ctx = fb.Context(hm, device=local, max_seq=P + 8)
    kv = ctx.kv(P + 8)
    prompt = np.resize(prompt_ids(p.vocab_size), P).astype(np.int32)
    for _ in range(args.warmup):
        ctx.prefill(kv, prompt)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(local)
    times = []
    with Clocks(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            ctx.prefill(kv, prompt)  # synchronizes the context stream before returning
            times.append(time.perf_counter() - t0)
    sec = sum(times)
    if dist is not None:
        t = torch.tensor([sec], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t.item())
    value = world * args.steps * P / sec
    n_params = p.n_layers * (2 * p.dim * p.dim + 2 * p.dim * p.n_kv_heads * p.head_dim + 3 * p.dim * p.ffn_dim)
    flops_tok = 2.0 * n_params
    peak_tf, peak_src = 1590.0, "fallback bf16"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak_tf, peak_src = float(json.load(f)["bf16_tflops"]), "measured bf16 burst"
    except (OSError, KeyError, ValueError):
        pass
    if rank == 0:
        ach = flops_tok * value / world / 1e12
        line = {"metric": "prefill tok/s (1.1B Q4_K_M, 512-token prompt)", "value": value, "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 x f16 -> f32",
                "data": "synthetic (seeded random-init weights, seeded prompt ids)",
                "config": {"workload": "1.1B Q4_K_M batched prefill (tcgen05 dequant-GEMMs)", "prompt": P,
                           "chunk": fb.PREFILL_CHUNK, "parallelism": f"replicas x{world}",
                           "timing": "host clock around fiber_prefill (it synchronizes its stream)"},
                "roofline": {"bound": "tensor", "achieved": ach, "peak": peak_tf, "unit": "TFLOP/s",
                             "frac": ach / peak_tf, "peak_source": peak_src,
                             "algorithmic_flops_per_token": flops_tok,
                             "issued_tensor_tflops": 2 * ach, "note": "issued = x split into fp16 hi and lo columns"},
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_batch(args, fb, torch, dist, rank, world, local):
    """Batched greedy decode (config 4 at batch 8 / 32, config 5 at batch 64): B sequences per
    step on KV slots 0..B-1 through the tensor-core layer pass, one captured graph per step.
    Config 4: the 1.1B Q5_K_M model, every slot's KV pre-filled with seeded N(0,1) fp16 keys /
    values for 2048 positions, 256 steps; one replica per rank (weak scaling). Config 5: the 7B
    Q4_K_M model, every slot prefilled with its own 512-token prompt, 256 steps, tensor-parallel
    over the ranks (strong scaling: the same B sequences whatever N)."""
    B = args.batch
    if args.workload == "7b-tp":
        path, P, D = MODEL_7B, 512, 256
        if rank == 0 and not os.path.exists(path):
            fb.write_model(path + ".tmp", fb.synth_cfg("llama7b"))
            os.replace(path + ".tmp", path)
        if dist is not None:
            dist.barrier()
    else:
        path, P, D = "/tmp/fiber_bench_tinyllama_q5km.gguf", 2048, 256
        if not os.path.exists(path):
            tmp = path + f".{os.getpid()}.tmp"
            fb.write_model(tmp, fb.synth_cfg("tinyllama-q5", seed=SEED))
            os.replace(tmp, path)
    if args.decode_len != DECODE_LEN:
        D = args.decode_len
    hm = fb.HostModel(path)
    p = hm.params
    tp = args.workload == "7b-tp" and world > 1
    if tp:
        box = [fb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ctx = fb.Context(hm, device=local, max_seq=P + D, tp=(rank, world, box[0]), max_batch=B)
    else:
        ctx = fb.Context(hm, device=local, max_seq=P + D, max_batch=B)
    kv = ctx.kv(P + D, max_batch=B)
    kvd = p.n_kv_heads * p.head_dim
    t_fill = time.perf_counter()
    if args.workload == "7b-tp":
        base = prompt_ids(p.vocab_size)[:P]
        firsts = [ctx.prefill(kv, np.roll(base, s), slot=s) for s in range(B)]
    else:
        for layer in range(p.n_layers):
            k = fb.randn(P * kvd, seed=100 + layer).reshape(P, kvd)
            v = fb.randn(P * kvd, seed=200 + layer).reshape(P, kvd)
            for s in range(B):
                kv.write(layer, 0, k, v, slot=s)
        firsts = [(5 + 7 * s) % p.vocab_size for s in range(B)]
    t_fill = time.perf_counter() - t_fill
    starts = [P] * B
    for _ in range(args.warmup):
        ctx.decode_greedy_batch(kv, firsts, starts, D)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(local)
    ms_total, wall = 0.0, 0.0
    with Clocks(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            toks, ms = ctx.decode_greedy_batch(kv, firsts, starts, D)  # host in -> device loop -> host out
            wall += time.perf_counter() - t0
            ms_total += ms
    if dist is not None:
        t = torch.tensor([ms_total, wall * 1e3], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total, wall = float(t[0].item()), float(t[1].item()) / 1e3
    reps = 1 if tp else world  # tensor parallel: the ranks share one batch
    value = reps * args.steps * D * B / (ms_total / 1e3)
    e2e = reps * args.steps * D * B / wall
    mid = P + D // 2
    if args.workload == "7b-tp":
        weights, kv_seq = WEIGHTS_7B, 524_288 * mid
    else:
        weights, kv_seq = 0.0, 0.0
        for kind in range(7):
            _, b = ctx.time_kernel(kv, kind, mid, reps=2)
            if kind == 1:
                kv_seq = b * p.n_layers  # attention reads: this sequence's K/V (+ q / out)
            else:
                weights += b * (1 if kind >= 5 else p.n_layers)
    step_bytes = weights + B * kv_seq
    peak, peak_kind = peaks()
    if rank == 0:
        ach = step_bytes * (value / B / reps) / (world if tp else 1) / 1e9
        name = {"7b-tp": "7B Q4_K_M (Llama-2-7B shape), each slot prefilled with a 512-token prompt",
                "q5km-long": "1.1B Q5_K_M (TinyLlama shape), every slot's KV pre-filled to 2048 positions"}[args.workload]
        line = {"metric": f"decode tok/s ({args.workload}, bs={B})", "value": value, "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_total / args.steps,
                "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
                "dtype": "f16 x f16 -> f32",
                "data": "synthetic (seeded random-init weights; seeded prompt ids or seeded N(0,1) KV)",
                "config": {"workload": name, "context": P, "decode_tokens_per_step": D, "global_batch": B * reps,
                           "parallelism": f"tp{world}" if tp else f"replicas x{world}",
                           "step_mode": "batched layer pass (tcgen05 GEMMs), one captured graph per step",
                           "fill_seconds": t_fill},
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * B / D, "d2h_bytes_per_step": 4 * B},
                "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                             "peak_source": peak_kind, "traffic": None, "algorithmic_bytes_per_step": step_bytes,
                             "weight_bytes": weights, "kv_bytes_per_sequence": kv_seq, "kv_position": mid},
                "gpu_launches": (5 + 14 * p.n_layers) * D * args.steps, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fiber", choices=["fiber", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--prompt-len", type=int, default=PROMPT_LEN, help="shorter runs for profiling only")
    ap.add_argument("--decode-len", type=int, default=DECODE_LEN, help="shorter runs for profiling only")
    ap.add_argument("--skip-extras", action="store_true", help="no single-GEMV, e2e or CPU legs (profiling)")
    ap.add_argument("--step-mode", type=int, default=None, choices=[0, 1, 2],
                    help="0: grid-barrier persistent kernel per token; 1: one kernel per phase; "
                         "2: dataflow kernel per token")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences per step for q5km-long / 7b-tp (>1: batched decode, one replica per rank)")
    ap.add_argument("--workload", default="1.1b", choices=["1.1b", "7b-tp", "stories", "q5km-long", "prefill"],
                    help="1.1b: the headline 1.1B Q4_K_M decode (replicas for N>1); "
                         "7b-tp: 7B Q4_K_M decode tensor-parallel over the N GPUs; "
                         "stories: fp16 stories-shaped model (dim 768, 12 layers), 32-token prompt, 256 steps; "
                         "q5km-long: 1.1B Q5_K_M with the KV cache pre-filled to 2048 positions, 256 steps; "
                         "prefill: 1.1B Q4_K_M batched prefill of a 512-token prompt")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch

    import fiber_b200 as fb

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    if args.batch > 1 and args.workload in ("7b-tp", "q5km-long"):
        return run_batch(args, fb, torch, dist, rank, world, local)
    if args.workload == "7b-tp":
        return run_7b_tp(args, fb, torch, dist, rank, world, local)
    if args.workload in ("stories", "q5km-long"):
        return run_config(args, fb, torch, dist, rank, world, local)
    if args.workload == "prefill":
        return run_prefill(args, fb, torch, dist, rank, world, local)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(local)

    P, D = args.prompt_len, args.decode_len
    path = MODEL_PATH if world == 1 else MODEL_PATH.replace(".gguf", f".r{rank}.gguf")
    make_model(path)
    hm = fb.HostModel(path)
    p = hm.params
    ctx = fb.Context(hm, device=local, max_seq=P + D)
    if args.step_mode is not None:
        ctx.set_mode(args.step_mode)
    kv = ctx.kv(P + D)
    prompt = prompt_ids(p.vocab_size)[:P]
    t0 = time.perf_counter()
    first = ctx.prefill(kv, prompt)  # first call: includes one-time set-up (padded Q6_K copies, maps)
    prefill_first_s = time.perf_counter() - t0
    pre_t = []
    for _ in range(5):  # warm: host call to result, median of 5
        t0 = time.perf_counter()
        ctx.prefill(kv, prompt)
        pre_t.append(time.perf_counter() - t0)
    prefill_tps = P / statistics.median(pre_t)

    ref_tokens = None
    for _ in range(args.warmup):
        toks, _ = ctx.decode_greedy(kv, first, P, D)
        ref_tokens = toks if ref_tokens is None else ref_tokens
    barrier()
    ms_total, deterministic = 0.0, True
    with Clocks(local) as clk:
        wall0 = time.perf_counter()
        for _ in range(args.steps):
            toks, ms = ctx.decode_greedy(kv, first, P, D)
            ms_total += ms
            if ref_tokens is not None and not np.array_equal(toks, ref_tokens):
                deterministic = False
            ref_tokens = toks if ref_tokens is None else ref_tokens
        barrier()
        wall = time.perf_counter() - wall0
    if dist is not None:
        t = torch.tensor([ms_total], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    value = world * args.steps * D / (ms_total / 1e3)

    # per-kernel device time: a graph of each kind's per-layer launches, CUDA events on the decode stream
    mid = P + D // 2
    kern = {}
    for kind, name in enumerate(fb.Context.KINDS):
        us, b = ctx.time_kernel(kv, kind, mid, reps=20)
        kern[name] = {"us_per_launch": us, "bytes_per_launch": b, "gbs": b / us / 1e3}

    e2e_val = None
    if not args.skip_extras:
        # e2e through the public C call with host buffers, one step
        barrier()
        e0 = time.perf_counter()
        tok = first
        for i in range(D):
            tok, _ = ctx.forward(kv, tok, P + i, want_logits=False)
        barrier()
        e2e_val = world * D / (time.perf_counter() - e0)

    phases = step_phase_times(ctx, kv, first, mid) if ctx.mode in (0, 2) else None

    extras = {}
    if not args.skip_extras:
        # config 5 at every N: the 7B model decoding tensor-parallel over all ranks (strong
        # scaling; the driver's 1..8-GPU runs record it beside the 1.1B replicas)
        try:
            extras["tp_7b"] = measure_7b_tp(fb, torch, dist, rank, world, local, 512, 64, 2, 1)
        except Exception as e:  # noqa: BLE001 -- recorded in the line, the 1.1B number stands
            extras["tp_7b"] = {"error": f"{type(e).__name__}: {e}"}
        if world == 1:  # configs 2 and 4 at batch 1 (short runs)
            for name, dd in (("stories", 256), ("q5km-long", 64)):
                try:
                    extras[name.replace("-", "_")] = measure_config(fb, torch, None, 0, 1, local, name, dd, 2, 1)
                except Exception as e:  # noqa: BLE001
                    extras[name.replace("-", "_")] = {"error": f"{type(e).__name__}: {e}"}

    if dist is not None:
        dist.barrier()
    if rank != 0:
        ctx.close()
        if dist is not None:
            dist.destroy_process_group()
        return

    peak, peak_kind = peaks()
    L = p.n_layers
    gemv_kinds = ["qkv", "wo", "gate_up", "down"]
    step_bytes = sum(kern[k]["bytes_per_launch"] * L for k in gemv_kinds + ["attention"]) + \
        kern["lm_head"]["bytes_per_launch"] + kern["embed"]["bytes_per_launch"]
    launches = ctx.step_launches() * D * args.steps
    mode = ctx.mode
    if mode in (0, 2):
        # one cooperative kernel per token: the step kernel is the dominant (only) kernel
        us_tok = ms_total * 1e3 / (args.steps * D)
        kname = "decode_flow_kernel" if mode == 2 else "decode_persistent_kernel"
        roof = {"kernel": f"{kname} (one launch per token)", "achieved": step_bytes / us_tok / 1e3,
                "algorithmic_bytes_per_launch": step_bytes, "us_per_launch": us_tok,
                "timing": "CUDA events on the decode stream around the timed steps"}
    else:
        dominant = max(gemv_kinds + ["attention", "lm_head"],
                       key=lambda k: kern[k]["us_per_launch"] * (1 if k == "lm_head" else L))
        dk = kern[dominant]
        roof = {"kernel": dominant, "achieved": dk["gbs"], "algorithmic_bytes_per_launch": dk["bytes_per_launch"],
                "us_per_launch": dk["us_per_launch"],
                "timing": "CUDA graph of the kernel's per-layer launches, CUDA events on the decode stream"}
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights, seeded prompt ids)",
        "config": {"workload": "1.1B Q4_K_M (TinyLlama shape) batch-1 greedy decode",
                   "model": "dim 2048, 22 layers, 32/4 heads, hd 64, ffn 5632, vocab 32000, Q4_K_M",
                   "prompt": P, "decode_tokens_per_step": D, "global_batch": 1,
                   "parallelism": f"replicas x{world}", "l2": "inputs larger than L2 (633 MB weights/token)",
                   "deterministic_tokens": deterministic, "prefill_tok_s": prefill_tps,
                   "prefill_timing": "median of 5 warm fiber_prefill calls, host call to returned token; the "
                                     f"first call took {prefill_first_s:.3f} s (one-time set-up)",
                   "step_mode": {0: "persistent kernel per token", 1: "one kernel per phase",
                                 2: "dataflow kernel per token"}[mode]},
        "roofline": dict(roof, bound="hbm", peak=peak, unit="GB/s", frac=roof["achieved"] / peak,
                         peak_source=peak_kind, **traffic_of(mode, roof)),
        "decode_roofline": {"bytes_per_token": step_bytes, "achieved_gbs": step_bytes * value / world / 1e9,
                            "frac": step_bytes * value / world / 1e9 / peak,
                            "step_phases": phases,
                            "per_phase_kernels_mode1": kern,
                            "kv_position_for_kernel_timing": mid,
                            "note": "step_phases: the timed one-kernel step traced at kv_position (critical-path "
                                    "us per phase kind, mean over layers); per_phase_kernels_mode1: each phase "
                                    "as its own kernel (decode mode 1), for the per-kind bytes"},
        "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": 32 * D, "d2h_bytes_per_step": 32 * D,
                "api": "fiber_forward_token (host token/pos in, argmax out)"},
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "wall_s": wall,
    }
    line.update(extras)
    if not args.skip_extras:
        single = gemv_bandwidth(local)
        line["gemv_single"] = dict(single, frac=single["gbs"] / peak)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_decode(path, budget_s=args.cpu_seconds, n_tokens_max=400)
    print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
