"""Tensor-parallel decode on two GPUs (one process per GPU; the exchange after Wo and
W_down fused into the dataflow step — each rank's epilogue stores its partial sums into
every rank over peer memory and the next phase adds them in rank order — or, with the
per-phase kernels, the one-shot peer-memory all-reduce or NCCL): both ranks produce the
oracle's greedy tokens, teacher-forced logits stay within the decode tolerances, and
where every rank adds the partials in the same order both ranks' logits are bit-identical;
steps that want only the token split the lm_head across the ranks. The batched layer pass (prefill,
several sequences per step) is sharded the same way and reproduces the oracle per
sequence. Skipped with fewer than two GPUs."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import fiber_b200 as fb
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

MAX_ABS, REL_RMS = 2e-2, 1e-3


def _worker(rank, world, nid, path, prompt, n_gen, q, coll):
    try:
        import os

        if coll == "nccl":
            os.environ["FIBER_TP_ALLREDUCE"] = "nccl"
        hm = fb.HostModel(path)
        ctx = fb.Context(hm, device=rank, max_seq=256, tp=(rank, world, nid), max_batch=3)
        if coll != "fused":
            ctx.set_mode(1)  # per-phase kernels with a separate all-reduce
        kv = ctx.kv(256)
        logits = []
        for pos, t in enumerate(prompt[:6]):  # teacher-forced, every rank in lockstep
            _, lg = ctx.forward(kv, int(t), pos)
            logits.append(lg)
        # token only (no logits wanted): in the dataflow step each rank runs its share of
        # the lm_head and the ranks exchange their best keys
        kv_am = ctx.kv(256)
        am_only = [ctx.forward(kv_am, int(t), pos, want_logits=False)[0] for pos, t in enumerate(prompt[:6])]
        kv2 = ctx.kv(256)
        first = ctx.prefill(kv2, np.asarray(prompt, np.int32))
        toks, _ = ctx.decode_greedy(kv2, first, len(prompt), n_gen)
        # batched: three sequences of different lengths on KV slots 0..2
        kv3 = ctx.kv(256, max_batch=3)
        prompts = [prompt[: 4 + 3 * i] for i in range(3)]
        firsts = [ctx.prefill(kv3, pr, slot=i) for i, pr in enumerate(prompts)]
        btoks, _ = ctx.decode_greedy_batch(kv3, firsts, [len(pr) for pr in prompts], 20)
        plan = ctx.plan
        q.put((rank, first, toks.tolist(), np.stack(logits),
               (plan.heads, plan.kv_heads, plan.ffn_blocks, ctx.tp_collective), None, firsts, btoks.tolist(),
               am_only))
        ctx.close()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, None, None, repr(e), None, None, None))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("coll", ["fused", "peer", "nccl"])
def test_tp2_matches_oracle(tiny_model, coll):
    path = tiny_model("tp")
    hm = fb.HostModel(path)
    p = hm.params
    rng = np.random.default_rng(5)
    prompt = rng.integers(1, p.vocab_size, 12).astype(np.int32)
    n_gen = 60
    nid = fb.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, nid, path, prompt, n_gen, q, coll)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = {}
    try:
        for _ in range(2):
            r = q.get(timeout=300)
            res[r[0]] = r
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    for r in (0, 1):
        assert res[r][5] is None, res[r][5]
    want_coll = {"fused": 3, "peer": 2, "nccl": 1}[coll]
    assert res[0][4] == (4, 2, 2, want_coll) and res[1][4] == (4, 2, 2, want_coll)
    if coll != "nccl":  # every rank adds the partial sums in the same order
        assert np.array_equal(res[0][3], res[1][3])

    om = orc.Model(path)
    st = om.state(256, kv_fp16=True)
    want_lg = np.stack([st.forward(int(t), pos) for pos, t in enumerate(prompt[:6])])
    for r in (0, 1):
        lg = res[r][3]
        assert np.abs(lg - want_lg).max() < MAX_ABS
        err = np.sqrt(np.mean((lg.astype(np.float64) - want_lg) ** 2) / np.mean(want_lg.astype(np.float64) ** 2))
        assert err < REL_RMS
        assert res[r][8] == [int(np.argmax(x)) for x in want_lg]
    st2 = om.state(256, kv_fp16=True)
    want = st2.generate(prompt, n_gen)
    for r in (0, 1):
        assert res[r][1] == want[0]
        assert res[r][2] == want[1:].tolist()
    # batched (tensor-parallel layer pass): each sequence equals the oracle run alone
    for i in range(3):
        pr = prompt[: 4 + 3 * i]
        wb = om.state(256, kv_fp16=True).generate(pr, 20)
        for r in (0, 1):
            assert res[r][6][i] == wb[0], (r, i)
            assert [row[i] for row in res[r][7]] == wb[1:].tolist(), (r, i)
