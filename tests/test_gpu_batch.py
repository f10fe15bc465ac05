"""Batched decode (several sequences per step) against the CPU oracle run
one sequence at a time.

Each sequence has its own KV cache, pre-filled to its own length (ragged),
and decodes greedily from its own position; every step's logits of every
sequence must match the oracle's forward of that sequence alone (max-abs
<= 1e-2, same argmax) and every cache row the step wrote must match within
the per-kernel bar |dev - ref| <= max(1.5e-4, 1e-4 |ref|).
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def close(dev, ref, rel=1e-4, floor=1.5e-4):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    err = np.abs(dev - ref)
    bad = err > np.maximum(floor, rel * np.abs(ref))
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {err.max():.3e}"


def run_batch_vs_oracle(path, cfg, B, lens, steps, seed):
    dev = Q.Model(path)
    orc = O.OracleModel(path, threads=os.cpu_count() or 1)
    Q.check(Q.lib.q_b200_batch_init(C.byref(dev.ctx), C.byref(dev.model), B), "batch_init")
    kv_elems = orc.kv.size
    kvs = []
    for b in range(B):
        kv = np.zeros(kv_elems, np.float32)
        assert Q.lib.q_b200_fill_kv_prefill(Q.ptr(kv), C.byref(cfg), lens[b], seed + b, 0) == 0
        Q.check(Q.lib.q_b200_batch_kv_write(C.byref(dev.ctx), b, 0, Q.ptr(kv), kv.nbytes), "kv_write")
        kvs.append(kv)
    toks = np.zeros(B, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), B, seed, 3, 0, cfg.vocab_size)
    pos = np.array(lens, np.uint32)
    V = cfg.vocab_size
    logits = np.zeros(B * V, np.float32)
    nxt = np.zeros(B, np.uint32)
    for step in range(steps):
        Q.check(Q.lib.q_b200_decode_batch(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(toks), Q.ptr(pos),
                                          Q.ptr(logits), Q.ptr(nxt)), "decode_batch")
        lg = logits.reshape(B, V)
        for b in range(B):
            orc.kv[:] = kvs[b]
            ref = orc.forward(np.array([toks[b]], np.uint32), int(pos[b])).copy()
            kvs[b][:] = orc.kv
            assert np.abs(lg[b] - ref).max() <= LOGIT_TOL, (step, b, float(np.abs(lg[b] - ref).max()))
            assert int(np.argmax(ref)) == int(nxt[b]) == int(np.argmax(lg[b])), (step, b)
        toks = nxt.copy()
        pos = pos + 1
    hd = cfg.dim // cfg.n_heads
    shp = (cfg.n_layers, cfg.n_kv_heads, cfg.max_seq_len, 2 * hd)
    for b in range(B):
        got = np.zeros(kv_elems, np.float32)
        Q.check(Q.lib.q_b200_batch_kv_read(C.byref(dev.ctx), b, 0, Q.ptr(got), got.nbytes), "kv_read")
        p0 = lens[b]
        d = got.reshape(shp)[:, :, p0:p0 + steps]
        r = kvs[b].reshape(shp)[:, :, p0:p0 + steps]
        close(d[0], r[0])
        for layer in range(1, cfg.n_layers):
            rl = np.asarray(r[layer], np.float64)
            err = np.abs(np.asarray(d[layer], np.float64) - rl)
            assert err.max() <= max(1.5e-4, 1e-4 * float(np.abs(rl).max())), (b, layer, float(err.max()))
    dev.close()
    orc.close()


@pytest.mark.parametrize("B", [5, 16])
def test_tiny_batch_vs_oracle(tiny_path, B):
    cfg = Q.config(**Q.TINY)
    lens = [3 + 29 * b % 200 for b in range(B)]
    run_batch_vs_oracle(tiny_path, cfg, B, lens, steps=4, seed=11)


def test_batch_loop_matches_single_steps(tiny_path):
    """q_b200_decode_batch_loop (tokens fed back on the device) gives each
    sequence the tokens its own greedy decode gives."""
    cfg = Q.config(**Q.TINY)
    B, n = 6, 8
    dev = Q.Model(tiny_path)
    Q.check(Q.lib.q_b200_batch_init(C.byref(dev.ctx), C.byref(dev.model), B), "batch_init")
    first = np.array([256, 1, 7, 99, 200, 258], np.uint32)
    pos = np.zeros(B, np.uint32)
    out = np.zeros(n * B, np.uint32)
    Q.check(Q.lib.q_b200_decode_batch_loop(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(first), Q.ptr(pos), n,
                                           Q.ptr(out), 1), "batch_loop")
    out = out.reshape(n, B)
    for b in range(B):
        solo = Q.Model(tiny_path)
        toks = solo.decode_loop(int(first[b]), 0, n)
        assert list(toks) == list(out[:, b]), b
        solo.close()
    dev.close()


@pytest.fixture(scope="module")
def llama70b_2layer(tmp_path_factory):
    # Llama-3-70B layer shapes, 2 layers, vocab cut to 32000 to keep the file small
    cfg = Q.config(32000, 8192, 28672, 2, 64, 8, 1024)
    path = tmp_path_factory.mktemp("m70b") / "l70b2.qorus"
    Q.write_model(str(path), cfg, seed=3)
    return str(path), cfg


def test_llama70b_shapes_batch16_vs_oracle(llama70b_2layer):
    """BASELINE configs[4]'s layer shapes at batch 16 (2 layers): ragged
    pre-filled caches, 2 greedy steps, every sequence against the oracle."""
    path, cfg = llama70b_2layer
    lens = [300 + 41 * b for b in range(16)]
    run_batch_vs_oracle(path, cfg, 16, lens, steps=2, seed=21)


def _paged_vs_contiguous(path, cfg, B, lens, page_rows, seed):
    """The same batched steps on contiguous caches and on a page pool sized
    for the rows actually used: logits, tokens and caches must be identical
    (the same arithmetic, only the addresses differ)."""
    dev = Q.Model(path)
    V = cfg.vocab_size
    n_elems = cfg.n_layers * cfg.n_kv_heads * cfg.max_seq_len * 2 * (cfg.dim // cfg.n_heads)
    kvs = []
    for b in range(B):
        kv = np.zeros(n_elems, np.float32)
        assert Q.lib.q_b200_fill_kv_prefill(Q.ptr(kv), C.byref(cfg), lens[b], seed + b, 0) == 0
        kvs.append(kv)
    toks = np.zeros(B, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), B, seed, 3, 0, V)
    pos = np.array(lens, np.uint32)
    steps = 6

    def run(paged):
        if paged:
            need = sum((ln + 1 + steps + page_rows - 1) // page_rows for ln in lens)
            Q.check(Q.lib.q_b200_batch_init_paged(C.byref(dev.ctx), C.byref(dev.model), B, page_rows, need),
                    "batch_init_paged")
        else:
            Q.check(Q.lib.q_b200_batch_init(C.byref(dev.ctx), C.byref(dev.model), B), "batch_init")
        for b in range(B):
            # only the rows the prefill wrote: the rest of a paged cache has no pages yet
            rows = np.ascontiguousarray(kvs[b].reshape(cfg.n_layers * cfg.n_kv_heads, cfg.max_seq_len, -1)[:, : lens[b]])
            hd2 = rows.shape[-1]
            for plane in range(rows.shape[0]):
                off = (plane * cfg.max_seq_len) * hd2 * 4
                Q.check(Q.lib.q_b200_batch_kv_write(C.byref(dev.ctx), b, off, Q.ptr(rows[plane]), rows[plane].nbytes),
                        "kv_write")
        logits = np.zeros(B * V, np.float32)
        nxt = np.zeros(B, np.uint32)
        Q.check(Q.lib.q_b200_decode_batch(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(toks), Q.ptr(pos),
                                          Q.ptr(logits), Q.ptr(nxt)), "decode_batch")
        out = np.zeros(steps * B, np.uint32)
        p1 = (pos + 1).astype(np.uint32)
        Q.check(Q.lib.q_b200_decode_batch_loop(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(nxt), Q.ptr(p1), steps,
                                               Q.ptr(out), 1), "decode_batch_loop")
        caches = []
        for b in range(B):
            kv = np.zeros(n_elems, np.float32)
            Q.check(Q.lib.q_b200_batch_kv_read(C.byref(dev.ctx), b, 0, Q.ptr(kv), kv.nbytes), "kv_read")
            caches.append(kv)
        return logits, out, caches

    lc, oc, cc = run(False)
    lp, op, cp = run(True)
    np.testing.assert_array_equal(lp, lc)
    np.testing.assert_array_equal(op, oc)
    for b in range(B):
        np.testing.assert_array_equal(cp[b], cc[b])
    # a pool one page short of the next step fails cleanly, and releasing a
    # sequence's pages lets the same step go through
    Q.check(Q.lib.q_b200_batch_init_paged(C.byref(dev.ctx), C.byref(dev.model), B, page_rows,
                                          sum((ln + 1 + page_rows - 1) // page_rows for ln in lens) - 1), "init")
    nxt = np.zeros(B, np.uint32)
    rc = Q.lib.q_b200_decode_batch(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(toks), Q.ptr(pos), None, Q.ptr(nxt))
    assert rc == -8  # Q_ERR_ARENA_OOM
    big = int(np.argmax(lens))  # the longest sequence restarts from position 0 in an empty slot
    Q.check(Q.lib.q_b200_batch_release(C.byref(dev.ctx), big), "release")
    pos0 = pos.copy()
    pos0[big] = 0
    Q.check(Q.lib.q_b200_decode_batch(C.byref(dev.model), C.byref(dev.ctx), Q.ptr(toks), Q.ptr(pos0), None,
                                      Q.ptr(nxt)), "decode_batch after release")
    dev.close()


def test_tiny_paged_matches_contiguous(tiny_path):
    cfg = Q.config(**Q.TINY)
    _paged_vs_contiguous(tiny_path, cfg, 5, [3, 130, 29, 255, 200], page_rows=128, seed=31)


def test_llama70b_shapes_paged_matches_contiguous(llama70b_2layer):
    path, cfg = llama70b_2layer
    _paged_vs_contiguous(path, cfg, 16, [300 + 41 * b for b in range(16)], page_rows=64, seed=41)
