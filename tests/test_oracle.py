"""The CPU oracle pinned against the upstream implementation (no GPU).

Fixtures in tests/golden/ were produced by the upstream code itself
(tests/golden/make_golden.py): its shipped dequantisation vectors, its AVX2
kernels on seeded inputs, its kernels composed into the intended forward,
and its own llama_forward on a square config.
"""
import hashlib
import struct

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q
from conftest import GOLDEN


@pytest.mark.parametrize("case", [1, 2, 3, 4])
def test_dequantize_upstream_vectors(case):
    # upstream tests/test_dequantize.c + test_data/dequantize_test*.bin
    blk = np.frombuffer((GOLDEN / f"dequantize_test{case}_block.bin").read_bytes(), np.uint8).copy()
    raw = (GOLDEN / f"dequantize_test{case}_expected.bin").read_bytes()
    n = struct.unpack("<I", raw[:4])[0]
    exp = np.frombuffer(raw[4:], np.float32)
    assert n == 32
    out = np.zeros(32, np.float32)
    O.orc.orc_dequantize_block(O.p(blk), O.p(out))
    np.testing.assert_allclose(out, exp, rtol=0, atol=1e-6)


def test_gemv_bit_exact(golden):
    for key in [k for k in golden.files if k.startswith("gemv_") and k.endswith("_w")]:
        M, K = map(int, key.split("_")[1].split("x"))
        w, x, y = golden[key], golden[key[:-1] + "x"], golden[key[:-1] + "y"]
        out = np.zeros(M, np.float32)
        assert O.orc.orc_gemv_q4(O.p(w), M, K, O.p(x), O.p(out)) == 0
        assert np.array_equal(out, y), key


def test_softmax_silu_bit_exact(golden):
    for N in (1, 3, 7, 8, 9, 15, 16, 33, 100, 2049):
        x = golden[f"softmax_{N}_x"]
        a, b = np.zeros(N, np.float32), np.zeros(N, np.float32)
        O.orc.orc_softmax(O.p(x), O.p(a), N)
        O.orc.orc_silu(O.p(x), O.p(b), N)
        assert np.array_equal(a, golden[f"softmax_{N}_y"]), N
        assert np.array_equal(b, golden[f"silu_{N}_y"]), N


def test_rmsnorm_rope(golden):
    for N in (8, 64, 256, 4096):
        x, w = golden[f"rms_{N}_x"], golden[f"rms_{N}_w"]
        o = np.zeros(N, np.float32)
        O.orc.orc_rmsnorm(O.p(x), O.p(w), O.p(o), N, 1e-5)
        # upstream's hardware rsqrt estimate differs from 1/sqrtf by <= 1 ulp
        # after its Newton step
        np.testing.assert_allclose(o, golden[f"rms_{N}_y"], rtol=3e-7, atol=0)
        r = np.zeros(N, np.float32)
        c, s = golden[f"rope_{N}_c"], golden[f"rope_{N}_s"]  # keep alive across the call
        O.orc.orc_rope(O.p(x), O.p(c), O.p(s), O.p(r), N)
        assert np.array_equal(r, golden[f"rope_{N}_y"])


def test_exp_poly_shape():
    # avx_math.h:10-61 — clamps and the zero floor
    e = O.orc.orc_exp_approx
    assert e(-11.0) == 0.0 and e(11.0) == 22026.0
    assert e(-6.0) == 0.0          # clamped to -5, polynomial negative, floored
    assert abs(e(0.0) - 1.0) < 1e-7
    assert e(-2.5) == 0.0          # Taylor-5 is negative below ~ -2.18


def test_tiny_model_file_is_reproducible(golden, tiny_path):
    digest = hashlib.sha256(open(tiny_path, "rb").read()).digest()
    assert digest == bytes(golden["tiny_sha256"])


def test_forward_tiny_vs_upstream_kernels(golden, tiny_path):
    m = O.OracleModel(tiny_path)
    prompt = golden["tiny_prompt"]
    lg = m.forward(prompt, 0)
    # only the rsqrt ulp separates the restatement from the upstream kernels
    np.testing.assert_allclose(lg, golden["tiny_prefill_logits"], rtol=0, atol=2e-6)
    toks = [int(np.argmax(lg))]
    for i in range(31):
        lg = m.forward(np.array([toks[-1]], np.uint32), 64 + i)
        toks.append(int(O.orc.orc_argmax(O.p(lg), m.vocab)))
    assert toks == list(golden["tiny_tokens"])
    np.testing.assert_allclose(m.logits, golden["tiny_last_logits"], rtol=0, atol=2e-6)
    m.close()


def test_forward_square_vs_upstream_llama_forward(golden, tmp_path):
    # upstream llama_forward is a correct Llama-3 forward only for square
    # shapes at seq_len 1, pos 0; there the restatement must agree with it
    cfg = Q.config(259, 256, 256, 2, 8, 8, 64)
    path = tmp_path / "square.qorus"
    Q.write_model(str(path), cfg, seed=3, threads=1)
    m = O.OracleModel(str(path))
    lg = m.forward(golden["square_token"], 0)
    np.testing.assert_allclose(lg, golden["square_logits"], rtol=0, atol=1e-6)
    m.close()


def test_prefill_equals_token_by_token(tiny_path):
    # masked entries contribute exact zeros, so with every row length below
    # 8 (all-expf softmax path) a chunked prefill equals split calls bit for bit
    m1, m2 = O.OracleModel(tiny_path), O.OracleModel(tiny_path)
    toks = np.array([256, 5, 17, 99, 3], np.uint32)
    a = m1.forward(toks, 0).copy()
    m2.forward(toks[:3], 0)
    b = m2.forward(toks[3:], 3).copy()
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(m1.kv, m2.kv)


@pytest.mark.skipif(O.rf is None, reason="upstream objects (oracle/_ref) not built")
def test_restatement_matches_upstream_kernels_live(tiny_path):
    a, b = O.OracleModel(tiny_path), O.RefModel(tiny_path, threads=2)
    toks = np.array([256, 1, 2, 3, 4, 5, 6, 7, 8, 9], np.uint32)
    np.testing.assert_allclose(a.forward(toks, 0), b.forward(toks, 0), rtol=0, atol=2e-6)
    np.testing.assert_allclose(a.kv, b.kv, rtol=0, atol=2e-6)
