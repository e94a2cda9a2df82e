"""Tensor-parallel split plan (host logic, no GPU): fiber_tp_plan covers every
head, KV head and FFN super-block exactly once, rejects models that do not split
on super-block boundaries, and a world-size-2 gloo group agrees on the plan and
the communicator id the way the sharded decode's ranks do."""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import fiber_b200 as fb


def _params(**kw):
    p = fb.ModelParams()
    for k, v in dict(n_layers=32, n_heads=32, n_kv_heads=32, dim=4096, head_dim=128, ffn_dim=11008,
                     vocab_size=32000, context_length=4096).items():
        setattr(p, k, kw.get(k, v))
    return p


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_llama7b(world):
    p = _params()
    plans = [fb.tp_plan(p, r, world) for r in range(world)]
    assert sum(x.heads for x in plans) == 32 and sum(x.kv_heads for x in plans) == 32
    assert [x.head0 for x in plans] == [r * 32 // world for r in range(world)]
    blocks = [b for x in plans for b in range(x.ffn_block0, x.ffn_block0 + x.ffn_blocks)]
    assert blocks == list(range(11008 // 256))  # every super-block once, in order
    assert max(x.ffn_blocks for x in plans) - min(x.ffn_blocks for x in plans) <= 1
    for x in plans:  # Wo shards are whole super-blocks
        assert x.heads * 128 % 256 == 0


def test_plan_rejects_unsplittable():
    with pytest.raises(fb.FiberError):
        fb.tp_plan(_params(n_kv_heads=4, n_heads=32), 0, 8)  # 4 KV heads over 8 ranks
    with pytest.raises(fb.FiberError):
        fb.tp_plan(_params(n_heads=12, n_kv_heads=12, head_dim=64, dim=768, ffn_dim=2048), 0, 2)  # 6*64 cols
    with pytest.raises(fb.FiberError):
        fb.tp_plan(_params(ffn_dim=512), 0, 4)  # 2 FFN blocks over 4 ranks
    with pytest.raises(fb.FiberError):
        fb.tp_plan(_params(), 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        box = [fb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        plan = fb.tp_plan(_params(), rank, world)
        mine = (box[0], plan.head0, plan.heads, plan.kv_head0, plan.kv_heads, plan.ffn_block0, plan.ffn_blocks)
        allp = [None] * world
        dist.all_gather_object(allp, mine)
        q.put((rank, allp))
    finally:
        dist.destroy_process_group()


def test_gloo_ranks_agree_on_id_and_plan():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = got[0], got[1]
    assert a == b  # identical view on every rank
    assert len(a[0][0]) == fb.TP_ID_BYTES and a[0][0] == a[1][0]
    assert a[0][1:3] == (0, 16) and a[1][1:3] == (16, 16)
    assert a[0][5] + a[0][6] == a[1][5] and a[1][5] + a[1][6] == 43
