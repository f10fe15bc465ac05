"""The prompt path on the B200 tensor cores against the CPU oracle.

q_b200_gemm_q4 is the prompt contraction (tcgen05 GEMM over fp16 hi/lo
operand halves) on its own: every row must equal the oracle's Q4_0 GEMV of
that row (upstream src/ops/avx2/matmul.c:98-271) within the per-kernel bar
|dev - ref| <= max(1.5e-4, 1e-4 |ref|).  The model tests run whole prompts
through llama_forward (which takes the prefill path for seq_len > 1) and
compare the last row's logits (max-abs <= 1e-2, same argmax) and every KV
row the prompt wrote with the oracle's: layer 0's rows are one kernel's
output from the same inputs (per-kernel bar); a later layer's rows depend on
every kernel of the layers before, so they are held to the per-kernel bar
relative to the layer's largest value (normwise,
|dev - ref| <= max(1.5e-4, 1e-4 max|ref|)) — the decode path's own rows
measured against the oracle sit at the same level (1.4e-4 at |ref| 22).
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


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    assert t.cuda.is_available()
    return t


@pytest.mark.parametrize("M,K,S", [(4096, 4096, 256), (1000, 800, 100), (6144, 4096, 129),
                                   (256, 256, 64), (28672, 4096, 40), (4096, 14336, 300), (32, 32, 1)])
def test_gemm_q4_rows_vs_oracle(torch, M, K, S):
    nblk = M * K // 32
    w = np.zeros(nblk * 20, np.uint8)
    Q.lib.q_b200_fill_q4(Q.ptr(w), nblk, M + K, 11, 0, 0.001, 0.01, 0)
    x = np.zeros(S * K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(x), x.size, S, 12, 0, 0.0, 1.0, 0)
    x.reshape(S, K)[S // 2] *= 1e-3  # rows of very different magnitude
    dw = torch.from_numpy(w).cuda()
    packed = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((S, M), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    Q.check(Q.lib.q_b200_q4_pack(dw.data_ptr(), M, K, packed.data_ptr(), None), "pack")
    Q.check(Q.lib.q_b200_gemm_q4(packed.data_ptr(), M, K, dx.data_ptr(), S, dy.data_ptr(), None), "gemm")
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    O.orc.orc_set_threads(os.cpu_count() or 1)
    rows = sorted({0, S // 2, S - 1} | set(range(0, S, max(1, S // 16))))
    for r in rows:
        ref = np.zeros(M, np.float32)
        xr = np.ascontiguousarray(x.reshape(S, K)[r])
        assert O.orc.orc_gemv_q4(O.p(w), M, K, O.p(xr), O.p(ref)) == 0
        close(got[r], ref)


def kv_rows_close(dev, ref, cfg, p0, p1):
    hd = cfg.dim // cfg.n_heads
    shp = (cfg.n_layers, cfg.n_kv_heads, cfg.max_seq_len, 2 * hd)
    d, r = dev.reshape(shp)[:, :, p0:p1], ref.reshape(shp)[:, :, p0:p1]
    close(d[0], r[0])
    for layer in range(1, cfg.n_layers):
        rl = np.asarray(r[layer], np.float64)
        err = np.abs(np.asarray(d[layer], np.float64) - rl)
        tol = max(1.5e-4, 1e-4 * float(np.abs(rl).max()))
        assert err.max() <= tol, f"layer {layer}: worst {err.max():.3e} > {tol:.3e}"


def test_tiny_prompt_chunks_vs_oracle(tiny_path):
    """Prompts through the prefill path: a fresh 200-row prompt, then a
    37-row chunk at pos 200 (causal mask inside the chunk, earlier rows from
    the cache), then decode steps that read what the prompt wrote."""
    dev, orc = Q.Model(tiny_path), O.OracleModel(tiny_path)
    toks = np.zeros(237, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), toks.size, 3, 1, 0, 259)
    for lo, hi in ((0, 200), (200, 237)):
        a = dev.forward(toks[lo:hi], lo).copy()
        b = orc.forward(toks[lo:hi], lo)
        assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
        kv = np.zeros(orc.kv.size, np.float32)
        dev.kv_read(kv)
        kv_rows_close(kv, orc.kv, dev.cfg, 0, hi)
    tok = int(np.argmax(b))
    for i in range(4):
        a = dev.forward(np.array([tok], np.uint32), 237 + i).copy()
        b = orc.forward(np.array([tok], np.uint32), 237 + i)
        assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))
    dev.close()
    orc.close()


def test_prefill_matches_row_replay(tiny_path, monkeypatch):
    """The tensor-core prompt path and the decode-graph row replay
    (QORUS_B200_PREFILL=0) agree on logits and KV rows."""
    toks = np.zeros(97, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), toks.size, 4, 1, 0, 259)
    dev = Q.Model(tiny_path)
    a = dev.forward(toks, 0).copy()
    kva = np.zeros(Q.kv_bytes(dev.cfg) // 4, np.float32)
    dev.kv_read(kva)
    dev.close()
    monkeypatch.setenv("QORUS_B200_PREFILL", "0")
    dev = Q.Model(tiny_path)
    b = dev.forward(toks, 0).copy()
    kvb = np.zeros_like(kva)
    dev.kv_read(kvb)
    dev.close()
    assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
    close(kva, kvb)


@pytest.fixture(scope="module")
def llama8b_2layer(tmp_path_factory):
    cfg = Q.config(32000, 4096, 14336, 2, 32, 8, 2304)
    path = tmp_path_factory.mktemp("m8b") / "l8b2_prefill.qorus"
    Q.write_model(str(path), cfg, seed=2)
    return str(path), cfg


def test_llama8b_shapes_prompt_2048_vs_oracle(llama8b_2layer):
    """BASELINE configs[3]'s prompt (2048 seeded uniform ids) on two
    Llama-3-8B-shaped layers: last-row logits, argmax and every KV row."""
    path, cfg = llama8b_2layer
    dev = Q.Model(path)
    orc = O.OracleModel(path, threads=os.cpu_count() or 1)
    S = 2048
    toks = np.zeros(S, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), S, 0, 9, 0, cfg.vocab_size)
    a = dev.forward(toks, 0).copy()
    b = orc.forward(toks, 0)
    assert np.abs(a - b).max() <= LOGIT_TOL, np.abs(a - b).max()
    assert int(np.argmax(a)) == int(np.argmax(b))
    kv = np.zeros(orc.kv.size, np.float32)
    dev.kv_read(kv)
    kv_rows_close(kv, orc.kv, cfg, 0, S)
    # a decode step after the prompt reads the cache the prompt wrote
    tok = int(np.argmax(b))
    a = dev.forward(np.array([tok], np.uint32), S).copy()
    b = orc.forward(np.array([tok], np.uint32), S)
    assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
    dev.close()
    orc.close()


@pytest.fixture(scope="module")
def hd128_path(tmp_path_factory):
    # a small model with Llama-3's head size (128) and grouping (4 query heads per KV head)
    cfg = Q.config(259, 512, 1024, 2, 4, 1, 640)
    path = tmp_path_factory.mktemp("hd128") / "hd128.qorus"
    Q.write_model(str(path), cfg, seed=5)
    return str(path), cfg


def test_head128_prompt_chunks_vs_oracle(hd128_path):
    """The tensor-core prompt attention (head_dim 128): a 300-row prompt, then
    a 77-row chunk at pos 300 (keys from the earlier call in the cache, the
    causal mask inside the chunk, a row length that is not a multiple of 8 so
    the tail takes expf), then a decode step over what the prompts wrote."""
    path, cfg = hd128_path
    dev, orc = Q.Model(path), O.OracleModel(path)
    toks = np.zeros(377, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), toks.size, 8, 1, 0, 259)
    for lo, hi in ((0, 300), (300, 377)):
        a = dev.forward(toks[lo:hi], lo).copy()
        b = orc.forward(toks[lo:hi], lo)
        assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
        kv = np.zeros(orc.kv.size, np.float32)
        dev.kv_read(kv)
        kv_rows_close(kv, orc.kv, cfg, 0, hi)
    tok = int(np.argmax(b))
    a = dev.forward(np.array([tok], np.uint32), 377).copy()
    b = orc.forward(np.array([tok], np.uint32), 377)
    assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
    dev.close()
    orc.close()
