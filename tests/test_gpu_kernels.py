"""Kernel parity on the B200: every device kernel against the upstream outputs
(golden fixtures) and the CPU oracle, through the C-ABI.

Tolerances (from the north star and upstream tests/test_matmul.c:63-64):
per kernel |dev - ref| <= max(1.5e-4, 1e-4 * |ref|); softmax outputs 1e-3.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def close(dev, ref, rel=1e-4, floor=1.5e-4):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    err = np.abs(dev - ref)
    bad = err > np.maximum(floor, rel * np.abs(ref))
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; worst {err.max():.3e}"


def al(n, dt=np.float32):
    return Q.aligned_empty(n, dt)


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    assert t.cuda.is_available()
    return t


def test_gemv_host_api_vs_upstream(golden):
    for key in [k for k in golden.files if k.startswith("gemv_") and k.endswith("_w")]:
        M, K = map(int, key.split("_")[1].split("x"))
        w = golden[key]
        x = al(K)
        x[:] = golden[key[:-1] + "x"]
        y = al(M)
        t = Q.q_tensor()
        t.data = w.ctypes.data
        t.ne[:] = [M, K, 1, 1]
        t.nb[:] = [K // 32 * 20, 20, 20, 20]
        t.type = Q.Q_Q4_0
        Q.check(Q.lib.q_gemv_q4_f32_avx2(C.byref(t), Q.ptr(x), Q.ptr(y)), "gemv")
        close(y, golden[key[:-1] + "y"])


def _device_gemv(torch, M, K, seed, x=None):
    nblk = M * K // 32
    w = np.zeros(nblk * 20, np.uint8)
    Q.lib.q_b200_fill_q4(Q.ptr(w), nblk, seed, 11, 0, 0.001, 0.01, 0)
    if x is None:
        x = np.zeros(K, np.float32)
        Q.lib.q_b200_fill_normal(Q.ptr(x), K, seed, 12, 0, 0.0, 1.0, 0)
    dw = torch.from_numpy(w).cuda()
    packed = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(M, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    Q.check(Q.lib.q_b200_q4_pack(dw.data_ptr(), M, K, packed.data_ptr(), None), "pack")
    Q.check(Q.lib.q_b200_gemv_q4(packed.data_ptr(), M, K, dx.data_ptr(), dy.data_ptr(), None), "gemv")
    torch.cuda.synchronize()
    ref = np.zeros(M, np.float32)
    O.orc.orc_set_threads(16)
    assert O.orc.orc_gemv_q4(O.p(w), M, K, O.p(x), O.p(ref)) == 0
    return dy.cpu().numpy(), ref


@pytest.mark.parametrize("M,K", [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096),
                                 (1000, 4096), (8, 256), (100, 768), (6144, 4096), (3, 14336)])
def test_gemv_device_vs_oracle(torch, M, K):
    dev, ref = _device_gemv(torch, M, K, seed=M + K)
    close(dev, ref)


@pytest.mark.parametrize("scale", [1e-33, 1e-30, 1e20, 1e-41, 0.0])
def test_gemv_input_magnitudes(torch, scale):
    """The fixed-point input grid follows each block's exponent: tiny, huge,
    subnormal and all-zero inputs, with every third block zero and one block
    holding a single non-zero value."""
    M, K = 512, 4096
    x = np.zeros(K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(x), K, 5, 12, 0, 0.0, 1.0, 0)
    x = (x.astype(np.float64) * scale).astype(np.float32)
    x.reshape(-1, 32)[::3] = 0.0
    x.reshape(-1, 32)[1, 1:] = 0.0
    dev, ref = _device_gemv(torch, M, K, 9, x)
    assert np.isfinite(dev).all()
    if scale == 0.0:
        assert (dev == 0).all()
        return
    if scale < 1e-38:
        # subnormal inputs: upstream's own fp32 products keep only a few bits
        # here, so only the magnitude is compared
        assert np.abs(dev).max() <= 1e-36 and np.abs(ref).max() <= 1e-36
        return
    unit = max(float(np.abs(ref).max()), np.finfo(np.float32).tiny)
    close(dev / unit, ref / unit)


def test_gemv_f32_vs_oracle(torch):
    M, K = 32000, 4096
    w = np.zeros(M * K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(w), w.size, 1, 21, 0, 0.0, 0.02, 0)
    x = np.zeros(K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(x), K, 1, 22, 0, 0.0, 1.0, 0)
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    dy = torch.empty(M, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    Q.check(Q.lib.q_b200_gemv_f32(dw.data_ptr(), M, K, dx.data_ptr(), dy.data_ptr(), None), "f32")
    torch.cuda.synchronize()
    ref = np.zeros(M, np.float32)
    O.orc.orc_set_threads(16)
    O.orc.orc_gemv_f32(O.p(w), M, K, O.p(x), O.p(ref))
    close(dy.cpu().numpy(), ref)


def test_softmax_silu_vs_upstream(golden):
    for N in (1, 3, 7, 8, 9, 15, 16, 33, 100, 2049):
        x = al(N)
        x[:] = golden[f"softmax_{N}_x"]
        a, b = al(N), al(N)
        Q.check(Q.lib.q_softmax_f32_avx2(Q.ptr(x), Q.ptr(a), N), "softmax")
        Q.check(Q.lib.q_silu_f32_avx2(Q.ptr(x), Q.ptr(b), N), "silu")
        close(a, golden[f"softmax_{N}_y"], rel=1e-3, floor=1e-6)
        close(b, golden[f"silu_{N}_y"])


def test_rmsnorm_rope_vs_upstream(golden):
    for N in (8, 64, 256, 4096):
        x, w, o = al(N), al(N), al(N)
        x[:], w[:] = golden[f"rms_{N}_x"], golden[f"rms_{N}_w"]
        Q.check(Q.lib.q_rmsnorm_f32_avx2(Q.ptr(x), Q.ptr(w), Q.ptr(o), N, 1e-5), "rmsnorm")
        close(o, golden[f"rms_{N}_y"])
        c, s, r = al(N), al(N), al(N)
        c[:], s[:] = golden[f"rope_{N}_c"], golden[f"rope_{N}_s"]
        Q.check(Q.lib.q_rope_f32_avx2(Q.ptr(x), Q.ptr(c), Q.ptr(s), Q.ptr(r), N), "rope")
        assert np.array_equal(r, golden[f"rope_{N}_y"])  # unfused products: bit-exact


@pytest.mark.parametrize("case", [1, 2, 3, 4])
def test_dequantize_block_vs_upstream_vectors(case):
    blk = np.frombuffer((GOLDEN / f"dequantize_test{case}_block.bin").read_bytes(), np.uint8).copy()
    exp = np.frombuffer((GOLDEN / f"dequantize_test{case}_expected.bin").read_bytes()[4:], np.float32)
    out = al(32)
    Q.lib.q_dequantize_q4_0_block_avx2_public(Q.ptr(blk), Q.ptr(out))
    np.testing.assert_allclose(out, exp, rtol=0, atol=1e-6)


def _t(a, ne0, ne1, nb0):
    t = Q.q_tensor()
    t.data = a.ctypes.data
    t.ne[:] = [ne0, ne1, 1, 1]
    t.nb[:] = [nb0, 4, 4, 4]
    t.type = Q.Q_F32
    return t


def test_add_mul_mask_matmul():
    rng = np.random.default_rng(3)
    n = 1000
    a, b, o = al(n), al(n), al(n)
    a[:], b[:] = rng.standard_normal(n), rng.standard_normal(n)
    ta, tb, to = _t(a, n, 1, n * 4), _t(b, n, 1, n * 4), _t(o, n, 1, n * 4)
    Q.check(Q.lib.q_add_f32_avx2(C.byref(ta), C.byref(tb), C.byref(to)), "add")
    assert np.array_equal(o, a + b)
    Q.check(Q.lib.q_mul_f32_avx2(C.byref(ta), C.byref(tb), C.byref(to)), "mul")
    assert np.array_equal(o, a * b)
    S = 37
    sc = al(S * 40)
    sc[:] = 1.0
    ts = _t(sc, S, S, 40 * 4)
    Q.check(Q.lib.q_causal_mask_f32_avx2(C.byref(ts), -1e9), "mask")
    m = sc.reshape(S, 40)[:, :S]
    assert (m[np.triu_indices(S, 1)] == -1e9).all() and (m[np.tril_indices(S)] == 1.0).all()
    M, K, N = 5, 64, 48
    A, B, Cc = al(M * K), al(K * N), al(M * N)
    A[:], B[:] = rng.standard_normal(M * K), rng.standard_normal(K * N)
    ctx = Q.q_context()
    tA, tB, tC = _t(A, M, K, K * 4), _t(B, K, N, N * 4), _t(Cc, M, N, N * 4)
    Q.check(Q.lib.q_matmul_f32_avx2(C.byref(tA), C.byref(tB), C.byref(tC), C.byref(ctx)), "matmul")
    close(Cc.reshape(M, N), A.reshape(M, K).astype(np.float64) @ B.reshape(K, N), rel=1e-4, floor=1e-4)
