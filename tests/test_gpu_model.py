"""Model parity on the B200 through the upstream C API (llama_forward,
q_generate) and the additive decode entry points, against the upstream
kernels' outputs (golden fixtures) and the CPU oracle.

Bars (north star): logits max-abs <= 1e-2, identical greedy argmax over 32
steps, KV-cache rows within the per-kernel tolerance
|dev - ref| <= max(1.5e-4, 1e-4 |ref|).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def kv_close(dev, ref, rel=1e-4, floor=1.5e-4):
    err = np.abs(dev.astype(np.float64) - ref)
    assert (err <= np.maximum(floor, rel * np.abs(ref))).all(), f"worst {err.max():.3e}"


def test_tiny_prefill_and_32_greedy_steps(tiny_path, golden):
    dev = Q.Model(tiny_path)
    prompt = golden["tiny_prompt"]
    lg = dev.forward(prompt, 0)
    assert np.abs(lg - golden["tiny_prefill_logits"]).max() <= LOGIT_TOL
    toks = [int(np.argmax(lg))]
    for i in range(31):
        lg = dev.forward(np.array([toks[-1]], np.uint32), 64 + i)
        toks.append(int(np.argmax(lg)))
    assert toks == list(golden["tiny_tokens"])
    assert np.abs(lg - golden["tiny_last_logits"]).max() <= LOGIT_TOL
    dev.close()


def test_tiny_kv_cache_and_logits_vs_oracle(tiny_path):
    dev = Q.Model(tiny_path)
    orc = O.OracleModel(tiny_path)
    toks = np.array([256, 4, 8, 15, 16, 23, 42, 108, 7, 9, 11, 13, 250], np.uint32)  # N = 13
    a = dev.forward(toks, 0).copy()
    b = orc.forward(toks, 0)
    assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
    kv = np.zeros(orc.kv.size, np.float32)
    dev.kv_read(kv)
    kv_close(kv, orc.kv)
    # chunked prefill at pos > 0 (row length N = 13 + 4, mask inside the chunk)
    more = np.array([3, 1, 4, 1], np.uint32)
    a = dev.forward(more, 13).copy()
    b = orc.forward(more, 13)
    assert np.abs(a - b).max() <= LOGIT_TOL and int(np.argmax(a)) == int(np.argmax(b))
    dev.kv_read(kv)
    kv_close(kv, orc.kv)
    dev.close()
    orc.close()


def test_single_token_at_pos0(tiny_path):
    dev, orc = Q.Model(tiny_path), O.OracleModel(tiny_path)
    a = dev.forward(np.array([256], np.uint32), 0).copy()  # N = 1: the all-expf softmax path
    b = orc.forward(np.array([256], np.uint32), 0)
    assert np.abs(a - b).max() <= LOGIT_TOL
    dev.close()


def test_decode_loop_matches_stepwise(tiny_path, golden):
    dev = Q.Model(tiny_path)
    prompt = golden["tiny_prompt"]
    lg = dev.forward(prompt, 0)
    first = int(np.argmax(lg))
    toks = dev.decode_loop(first, 64, 31)
    assert [first] + list(toks) == list(golden["tiny_tokens"])
    nxt = C.c_uint32()
    Q.check(Q.lib.q_b200_decode_greedy(C.byref(dev.model), C.byref(dev.ctx), int(toks[-1]), 95,
                                       C.byref(nxt)), "decode_greedy")
    assert 0 <= nxt.value < 259
    dev.close()


def test_q_generate_greedy(tiny_path, golden):
    dev = Q.Model(tiny_path)
    tok = Q.q_tokenizer()
    tok.initialized = True
    tok.eos_token_id = 0xFFFFFFFF  # unreachable: always 32 tokens
    prompt = np.ascontiguousarray(golden["tiny_prompt"], np.uint32)
    out = np.zeros(32, np.uint32)
    st = Q.q_generation_state()
    st.ctx = C.pointer(dev.ctx)
    st.model = C.pointer(dev.model)
    st.tokenizer = C.pointer(tok)
    st.prompt_tokens = prompt.ctypes.data_as(C.POINTER(C.c_uint32))
    st.num_prompt_tokens = 64
    st.generated_tokens = out.ctypes.data_as(C.POINTER(C.c_uint32))
    st.max_tokens = 32
    st.temperature = 0.0
    Q.check(Q.lib.q_generate(C.byref(st)), "q_generate")
    # upstream main.c:1071-1115 runs a forward after every kept token
    assert st.num_generated_tokens == 32 and st.current_pos == 64 + 32
    assert list(out) == list(golden["tiny_tokens"])
    dev.close()


def test_forward_rejects_bad_tokens(tiny_path):
    dev = Q.Model(tiny_path)
    with pytest.raises(Q.QorusError) as e:
        dev.forward(np.array([259], np.uint32), 0)
    assert e.value.code == -10
    dev.close()


@pytest.fixture(scope="module")
def llama8b_2layer(tmp_path_factory):
    # Llama-3-8B layer shapes, 2 layers, vocab cut to 32000 to keep the file small
    cfg = Q.config(32000, 4096, 14336, 2, 32, 8, 2304)
    path = tmp_path_factory.mktemp("m8b") / "l8b2.qorus"
    Q.write_model(str(path), cfg, seed=1)
    return str(path), cfg


def test_llama8b_shapes_decode_over_prefilled_cache(llama8b_2layer):
    path, cfg = llama8b_2layer
    dev = Q.Model(path)
    orc = O.OracleModel(path, threads=32)
    npos = 2048
    assert Q.lib.q_b200_fill_kv_prefill(Q.ptr(orc.kv), C.byref(cfg), npos, 7, 0) == 0
    dev.kv_write(orc.kv)
    tok = 1234
    for step in range(3):
        a = dev.forward(np.array([tok], np.uint32), npos + step).copy()
        b = orc.forward(np.array([tok], np.uint32), npos + step)
        assert np.abs(a - b).max() <= LOGIT_TOL
        assert int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))
    kv = np.zeros(orc.kv.size, np.float32)
    dev.kv_read(kv)
    kv_close(kv, orc.kv)
    dev.close()
    orc.close()


def test_profile_step_stamps_and_result(tiny_path, golden):
    """The traced step writes the same KV rows as an untraced one and stamps
    every kernel of the step in launch order."""
    dev = Q.Model(tiny_path)
    prompt = golden["tiny_prompt"]
    tok = int(np.argmax(dev.forward(prompt, 0)))
    kv0 = np.zeros(Q.kv_bytes(dev.cfg) // 4, np.float32)
    dev.kv_read(kv0)
    st = dev.profile_step(tok, len(prompt))
    L = dev.cfg.n_layers
    # QKV of layer 0; per layer: attention, then wo, gate/up, down and the
    # next layer's QKV (one launch each, or one chained launch); head, advance
    assert st.shape in ((5 * L + 2, 3), (2 * L + 3, 3))
    assert (st[:, 0] <= st[:, 1]).all() and (st[:, 1] <= st[:, 2]).all()
    assert (st[1:, 2] >= st[:-1, 2]).all()
    kv_traced = np.zeros_like(kv0)
    dev.kv_read(kv_traced)
    dev.kv_write(kv0)
    nxt = C.c_uint32()
    Q.check(Q.lib.q_b200_decode_greedy(C.byref(dev.model), C.byref(dev.ctx), tok, len(prompt),
                                       C.byref(nxt)), "decode_greedy")
    assert nxt.value == golden["tiny_tokens"][1]
    kv_plain = np.zeros_like(kv0)
    dev.kv_read(kv_plain)
    assert np.array_equal(kv_traced, kv_plain)
    dev.close()


def test_llama8b_full_decode_32_steps_vs_oracle(tmp_path):
    """The benchmarked configuration itself: 32 layers,
    dim 4096, 32/8 heads, FFN 14336, vocab 128256, KV cache pre-filled with
    2048 positions of N(0,1), then 32 greedy steps through llama_forward,
    each step's logits against the oracle's (max-abs <= 1e-2, same argmax),
    and the 32 new KV rows of every layer within the per-kernel bar."""
    import os
    from pathlib import Path
    shm = Path("/dev/shm")
    d = shm if shm.exists() and os.access(shm, os.W_OK) else tmp_path
    npos, steps = 2048, 32
    cfg = Q.config(128256, 4096, 14336, 32, 32, 8, npos + 64)
    path = d / f"qorus_parity_l8b_{os.getpid()}.qorus"
    try:
        Q.write_model(str(path), cfg, seed=0)
        dev = Q.Model(str(path))
        orc = O.OracleModel(str(path), threads=os.cpu_count() or 1)
        assert Q.lib.q_b200_fill_kv_prefill(Q.ptr(orc.kv), C.byref(cfg), npos, 1, 0) == 0
        dev.kv_write(orc.kv)
        tok, worst = 1, 0.0
        for step in range(steps):
            a = dev.forward(np.array([tok], np.uint32), npos + step)
            b = orc.forward(np.array([tok], np.uint32), npos + step)
            worst = max(worst, float(np.abs(a - b).max()))
            assert np.abs(a - b).max() <= LOGIT_TOL, f"step {step}: {np.abs(a - b).max():.3e}"
            assert int(np.argmax(a)) == int(np.argmax(b)), f"step {step}"
            tok = int(np.argmax(b))
        kv = np.zeros(orc.kv.size, np.float32)
        dev.kv_read(kv)
        hd = 128
        shp = (cfg.n_layers, cfg.n_kv_heads, cfg.max_seq_len, 2 * hd)
        kv_close(kv.reshape(shp)[:, :, npos: npos + steps], orc.kv.reshape(shp)[:, :, npos: npos + steps])
        dev.close()
        orc.close()
    finally:
        if path.exists():
            path.unlink()
