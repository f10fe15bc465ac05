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
