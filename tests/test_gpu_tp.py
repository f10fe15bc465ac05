"""Tensor parallelism on 2 GPUs (skipped on single-GPU machines): two ranks,
one process per GPU, each holding its shard; the decode graph all-reduces
either over NVLink peer memory (CUDA IPC; fused into the GEMVs, or the
separate exchange kernel with QORUS_B200_TP_FUSED=0) or with NCCL.  The gathered logits and greedy tokens must match the upstream
kernels' golden outputs for the tiny config (logits max-abs <= 1e-2,
identical tokens), and each rank's KV cache (its own KV heads) must match
the CPU oracle's rows for those heads."""
import os
import socket

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path, prompt, ipc, fused, out):
    os.environ["QORUS_B200_TP_FUSED"] = "1" if fused else "0"
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)  # host channel for the NCCL id
    try:
        box = [Q.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        def gather(b):
            allb = [None] * world
            dist.all_gather_object(allb, b)
            return allb
        m = Q.Model(path, tp=(rank, world, box[0]), tp_gather=gather if ipc else None)
        first = m.forward(prompt, 0).copy()
        toks = [int(np.argmax(first))]
        for i in range(31):
            lg = m.forward(np.array([toks[-1]], np.uint32), len(prompt) + i)
            toks.append(int(np.argmax(lg)))
        last = lg.copy()
        kv = np.zeros(m.kv_size // 4, np.float32)
        m.kv_read(kv)
        dev_loop = m.decode_loop(toks[-1], len(prompt) + 31, 8).tolist()
        shape = Q.tp_shape(m.cfg, rank, world)
        out.put((rank, first, last, toks, kv, shape, dev_loop))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ipc,fused", [(True, True), (True, False), (False, False)],
                         ids=["peer-memory-fused", "peer-memory-kernel", "nccl"])
def test_tp2_tiny_matches_upstream_and_oracle(tiny_path, golden, ipc, fused):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    prompt = golden["tiny_prompt"]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, tiny_path, prompt, ipc, fused, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q.get(timeout=300)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # the oracle's cache after the same 64 + 31 positions
    orc = O.OracleModel(tiny_path)
    orc.forward(prompt, 0)
    for i, t in enumerate(golden["tiny_tokens"][:31]):
        orc.forward(np.array([t], np.uint32), len(prompt) + i)
    cfg = Q.config(**Q.TINY)
    hd = cfg.dim // cfg.n_heads
    ref_kv = orc.kv.reshape(cfg.n_layers, cfg.n_kv_heads, cfg.max_seq_len, 2 * hd)
    valid = len(prompt) + 31
    for rank in range(2):
        _, first, last, toks, kv, sh, loop = res[rank]
        assert np.abs(first - golden["tiny_prefill_logits"]).max() <= LOGIT_TOL
        assert toks == list(golden["tiny_tokens"])
        assert np.abs(last - golden["tiny_last_logits"]).max() <= LOGIT_TOL
        h0 = sh["kv0"] // hd
        mine = kv[: cfg.n_layers * sh["nkv"] * cfg.max_seq_len * 2 * hd].reshape(
            cfg.n_layers, sh["nkv"], cfg.max_seq_len, 2 * hd)
        ref = ref_kv[:, h0: h0 + sh["nkv"], :valid].astype(np.float64)
        err = np.abs(mine[:, :, :valid] - ref)
        assert (err <= np.maximum(1.5e-4, 1e-4 * np.abs(ref))).all(), f"kv worst {err.max():.3e}"
    assert res[0][6] == res[1][6]  # device-fed decode agrees across ranks
    orc.close()


# ---- 2, 4 and 8 ranks on a config whose heads split 8 ways ---------------------

WIDE = dict(vocab=1000, dim=512, hidden=1536, layers=2, heads=8, kv_heads=8, max_seq=256)


def _wide_worker(rank, world, port, path, prompt, feed, fused, out):
    os.environ["QORUS_B200_TP_FUSED"] = "1" if fused else "0"
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        box = [Q.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)

        def gather(b):
            allb = [None] * world
            dist.all_gather_object(allb, b)
            return allb
        m = Q.Model(path, tp=(rank, world, box[0]), tp_gather=gather)
        logits = [m.forward(prompt, 0).copy()]
        for i, t in enumerate(feed):
            logits.append(m.forward(np.array([t], np.uint32), len(prompt) + i).copy())
        loop = m.decode_loop(int(feed[-1]), len(prompt) + len(feed), 12).tolist()
        out.put((rank, np.stack(logits), loop))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "kernel"])
def test_tp_wide_matches_oracle(tmp_path, world, fused):
    """Logits of a prompt and 15 fed tokens on `world` ranks against the CPU
    oracle (max-abs <= 1e-2), and the device-fed greedy loop (argmax keys
    exchanged between ranks) equal on every rank and to one GPU's loop."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cfg = Q.config(**WIDE)
    path = str(tmp_path / "wide.qorus")
    Q.write_model(path, cfg, seed=7, threads=8)
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, WIDE["vocab"], 40).astype(np.uint32)
    orc = O.OracleModel(path)
    ref = [orc.forward(prompt, 0).copy()]
    feed = []
    for i in range(15):
        feed.append(int(np.argmax(ref[-1])))
        ref.append(orc.forward(np.array([feed[-1]], np.uint32), len(prompt) + i).copy())
    orc.close()
    solo = Q.Model(path)
    solo.forward(prompt, 0)
    for i, t in enumerate(feed):
        solo.forward(np.array([t], np.uint32), len(prompt) + i)
    solo_loop = solo.decode_loop(feed[-1], len(prompt) + len(feed), 12).tolist()
    solo.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_wide_worker, args=(r, world, port, path, prompt, feed, fused, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=300)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        _, lg, loop = res[rank]
        err = np.abs(lg[:, : WIDE["vocab"]] - np.stack(ref)).max()
        assert err <= LOGIT_TOL, f"rank {rank}: logits max-abs {err:.3e}"
        assert loop == solo_loop, (rank, loop, solo_loop)


# ---- batched decode on 2, 4 and 8 ranks ---------------------------------------

def _batch_run(m, cfg, kvs, toks, pos, rank=0, world=1):
    import ctypes as C
    B = len(kvs)
    Q.check(Q.lib.q_b200_batch_init(C.byref(m.ctx), C.byref(m.model), B), "batch_init")
    hd = cfg.dim // cfg.n_heads
    for b, kv in enumerate(kvs):
        if world > 1:
            sh = Q.tp_shape(cfg, rank, world)
            h0 = sh["kv0"] // hd
            kv = np.ascontiguousarray(kv.reshape(cfg.n_layers, cfg.n_kv_heads, -1)[:, h0: h0 + sh["nkv"]]).ravel()
        Q.check(Q.lib.q_b200_batch_kv_write(C.byref(m.ctx), b, 0, Q.ptr(kv), kv.nbytes), "batch_kv_write")
    V = cfg.vocab_size
    logits = np.zeros(B * V, np.float32)
    nxt = np.zeros(B, np.uint32)
    Q.check(Q.lib.q_b200_decode_batch(C.byref(m.model), C.byref(m.ctx), Q.ptr(toks), Q.ptr(pos), Q.ptr(logits),
                                      Q.ptr(nxt)), "decode_batch")
    out = np.zeros(6 * B, np.uint32)
    pos1 = (pos + 1).astype(np.uint32)
    Q.check(Q.lib.q_b200_decode_batch_loop(C.byref(m.model), C.byref(m.ctx), Q.ptr(nxt), Q.ptr(pos1), 6,
                                           Q.ptr(out), 1), "decode_batch_loop")
    return logits.reshape(B, V), nxt, out.reshape(6, B)


def _batch_worker(rank, world, port, path, kvs, toks, pos, out):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        box = [Q.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)

        def gather(b):
            allb = [None] * world
            dist.all_gather_object(allb, b)
            return allb
        m = Q.Model(path, tp=(rank, world, box[0]), tp_gather=gather)
        out.put((rank, *_batch_run(m, Q.config(**WIDE), kvs, toks, pos, rank, world)))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_batched_decode_matches_single_gpu(tmp_path, world):
    """Five sequences with ragged pre-filled caches decoded together on
    `world` ranks (partial residuals and argmax keys all-reduced, vocabulary
    rows gathered): one step's logits of every sequence equal one GPU's
    batched step (max-abs <= 1e-2), and the next 6 device-fed tokens of every
    sequence are the same."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import ctypes as C
    import torch.multiprocessing as mp
    cfg = Q.config(**WIDE)
    path = str(tmp_path / "wide.qorus")
    Q.write_model(path, cfg, seed=7, threads=8)
    lens = [17, 60, 3, 111, 200]
    n = cfg.n_layers * cfg.n_kv_heads * cfg.max_seq_len * 2 * (cfg.dim // cfg.n_heads)
    kvs = []
    for b, ln in enumerate(lens):
        kv = np.zeros(n, np.float32)
        assert Q.lib.q_b200_fill_kv_prefill(Q.ptr(kv), C.byref(cfg), ln, 40 + b, 0) == 0
        kvs.append(kv)
    toks = np.array([5, 99, 700, 3, 256], np.uint32)
    pos = np.array(lens, np.uint32)
    solo = Q.Model(path)
    ref_logits, ref_next, ref_loop = _batch_run(solo, cfg, kvs, toks, pos)
    solo.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_batch_worker, args=(r, world, port, path, kvs, toks, pos, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=300)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        _, lg, nxt, loop = res[rank]
        err = np.abs(lg - ref_logits).max()
        assert err <= LOGIT_TOL, f"rank {rank}: logits max-abs {err:.3e}"
        assert list(nxt) == list(ref_next)
        assert (loop == ref_loop).all(), (rank, loop, ref_loop)


# ---- sampled generation on 2, 4 and 8 ranks -------------------------------------

def _generate_worker(rank, world, port, path, prompt, fused, out):
    """q_generate with temperature 0.8, top-k 40, top-p 0.9 from a fresh
    process (the thread's random state starts at upstream's seed)."""
    import ctypes as C
    os.environ["QORUS_B200_TP_FUSED"] = "1" if fused else "0"
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    tp = gather = None
    if world > 1:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        box = [Q.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = (rank, world, box[0])

        def gather(b):
            allb = [None] * world
            dist.all_gather_object(allb, b)
            return allb
    try:
        m = Q.Model(path, tp=tp, tp_gather=gather)
        tok = Q.q_tokenizer()
        tok.initialized = True
        tok.eos_token_id = 0xFFFFFFFF
        n = 20
        gen = np.zeros(n, np.uint32)
        st = Q.q_generation_state()
        st.ctx = C.pointer(m.ctx)
        st.model = C.pointer(m.model)
        st.tokenizer = C.pointer(tok)
        st.prompt_tokens = prompt.ctypes.data_as(C.POINTER(C.c_uint32))
        st.num_prompt_tokens = len(prompt)
        st.generated_tokens = gen.ctypes.data_as(C.POINTER(C.c_uint32))
        st.max_tokens = n
        st.temperature = 0.8
        st.top_k = 40
        st.top_p = 0.9
        Q.check(Q.lib.q_generate(C.byref(st)), "q_generate")
        out.put((rank, list(gen[: st.num_generated_tokens])))
        m.close()
    finally:
        if world > 1:
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "kernel"])
def test_tp_sampled_generate_matches_single_gpu(tmp_path, world, fused):
    """Temperature / top-k / top-p generation on `world` ranks (logits
    gathered on every rank, the same draw everywhere) gives the tokens one
    GPU gives from the same random state."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cfg = Q.config(**WIDE)
    path = str(tmp_path / "wide.qorus")
    Q.write_model(path, cfg, seed=7, threads=8)
    prompt = np.random.default_rng(5).integers(0, WIDE["vocab"], 24).astype(np.uint32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p1 = ctx.Process(target=_generate_worker, args=(0, 1, 0, path, prompt, fused, q))
    p1.start()
    ref = q.get(timeout=300)[1]
    p1.join(timeout=120)
    assert p1.exitcode == 0 and len(ref) == 20
    port = _free_port()
    procs = [ctx.Process(target=_generate_worker, args=(r, world, port, path, prompt, fused, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=300)
        res[r[0]] = r[1]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):
        assert res[rank] == ref, (rank, res[rank], ref)
