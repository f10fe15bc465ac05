"""Tensor-parallel host logic on CPU: two `gloo` ranks each compute their shard
(q_b200_tp_shape), gather them, and check that the shards partition every
split dimension exactly (query/KV heads, FFN rows, vocab rows); configs that
do not split evenly are rejected on every rank."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import qorus_b200 as Q

CFG8B = dict(vocab=128256, dim=4096, hidden=14336, layers=32, heads=32, kv_heads=8, max_seq=4096)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = {}
        for name, kw in (("tiny", Q.TINY), ("8b", CFG8B)):
            cfg = Q.config(**kw)
            mine = Q.tp_shape(cfg, rank, world)
            allv = [None] * world
            dist.all_gather_object(allv, mine)
            res[name] = allv
        bad = Q.config(**dict(Q.TINY, kv_heads=1))  # 1 KV head cannot split over 2 ranks
        out_arr = (Q.C.c_uint32 * 13)()
        res["bad_rc"] = Q.lib.q_b200_tp_shape(Q.C.byref(bad), rank, world, out_arr, 13)
        if rank == 0:
            out.put(res)
    finally:
        dist.destroy_process_group()


def _check_partition(shards, total, lo_key, n_key):
    cover = np.zeros(total, np.int32)
    for sh in shards:
        cover[sh[lo_key]: sh[lo_key] + sh[n_key]] += 1
    assert (cover == 1).all()


@pytest.mark.parametrize("world", [2])
def test_tp_shards_partition_over_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for name, kw in (("tiny", Q.TINY), ("8b", CFG8B)):
        shards = res[name]
        hd = kw["dim"] // kw["heads"]
        assert [s["rank"] for s in shards] == list(range(world))
        _check_partition(shards, kw["dim"], "q0", "d")                        # query rows
        _check_partition(shards, kw["kv_heads"] * hd, "kv0", "kvd")          # key / value rows
        _check_partition(shards, kw["hidden"], "h0", "h")                    # FFN rows
        _check_partition(shards, kw["vocab"], "v0", "v")                     # vocab rows
        for s in shards:
            assert s["d"] % 32 == 0 and s["h"] % 32 == 0                     # whole Q4_0 blocks
            assert s["v0"] == s["rank"] * s["v_pad"]                          # gather order
    assert res["bad_rc"] == -9  # Q_ERR_INVALID_CONFIG
