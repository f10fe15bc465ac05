"""Failure detection on the GPU without a GPU fault: a bounded device wait is
made to run out on purpose and the error must come back to the host as a
status code, with the context still usable afterwards.

The wait that runs out is the fused tensor-parallel receive of the Q4_0 GEMV
(the prologue that waits for every peer rank's flag), launched on one GPU
with an exchange buffer that no sender writes.  Nothing faults, traps or
hangs: every CTA gives up after the limit (20 ms here), records the peer
timeout code (6) in the device status word and returns.
"""
import time

import numpy as np
import pytest

import oracle as O
import qorus_b200 as Q

pytestmark = pytest.mark.gpu

QDEV_PEER_TIMEOUT = 6


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    assert t.cuda.is_available()
    return t


def _gemv_ok(torch, M=1000, K=4096, seed=4):
    nblk = M * K // 32
    w = np.zeros(nblk * 20, np.uint8)
    Q.lib.q_b200_fill_q4(Q.ptr(w), nblk, seed, 11, 0, 0.001, 0.01, 0)
    x = np.zeros(K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(x), K, seed, 12, 0, 0.0, 1.0, 0)
    dw = torch.from_numpy(w).cuda()
    packed = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
    dx, dy = torch.from_numpy(x).cuda(), torch.empty(M, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    Q.check(Q.lib.q_b200_q4_pack(dw.data_ptr(), M, K, packed.data_ptr(), None), "pack")
    Q.check(Q.lib.q_b200_gemv_q4(packed.data_ptr(), M, K, dx.data_ptr(), dy.data_ptr(), None), "gemv")
    torch.cuda.synchronize()
    ref = np.zeros(M, np.float32)
    assert O.orc.orc_gemv_q4(O.p(w), M, K, O.p(x), O.p(ref)) == 0
    err = np.abs(dy.cpu().numpy().astype(np.float64) - ref)
    assert (err <= np.maximum(1.5e-4, 1e-4 * np.abs(ref))).all()


def test_peer_wait_runs_out_and_reports(torch):
    import ctypes as C
    _gemv_ok(torch)  # a clean start
    assert Q.lib.q_b200_device_status() == 0
    st = C.c_uint32(0)
    t0 = time.perf_counter()
    Q.check(Q.lib.q_b200_selftest_exchange_timeout(20_000_000, C.byref(st)), "selftest")
    waited = time.perf_counter() - t0
    assert st.value == QDEV_PEER_TIMEOUT
    assert 0.02 <= waited < 10.0  # the wait gave up after its limit, not at once, not never
    # the status word was read and cleared; the device and the library work on
    assert Q.lib.q_b200_device_status() == 0
    _gemv_ok(torch, M=4096, K=14336, seed=5)
    # the default limit is back: a second run of the self-test behaves the same
    Q.check(Q.lib.q_b200_selftest_exchange_timeout(5_000_000, C.byref(st)), "selftest")
    assert st.value == QDEV_PEER_TIMEOUT


def test_wait_limit_setter_validates():
    assert Q.lib.q_b200_set_wait_limit_ns(0) == -10
    assert Q.lib.q_b200_set_wait_limit_ns(2_000_000_000) == 0
