"""q_b200_gemv_q4_noalloc (scratch in a fixed device array, no allocation)
against q_b200_gemv_q4 on the same packed weights, through the C-ABI.

Collected last so it runs both alone and after every other test.  Tolerance
is the per-kernel bar |a - b| <= max(1.5e-4, 1e-4 |b|); both entry points run
the same kernel, so the results are in fact identical.
"""
import numpy as np
import pytest

import qorus_b200 as Q

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    assert t.cuda.is_available()
    return t


def _packed(torch, M, K, seed):
    nblk = M * K // 32
    w = np.zeros(nblk * 20, np.uint8)
    Q.lib.q_b200_fill_q4(Q.ptr(w), nblk, seed, 11, 0, 0.001, 0.01, 0)
    x = np.zeros(K, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(x), K, seed, 12, 0, 0.0, 1.0, 0)
    dw = torch.from_numpy(w).cuda()
    packed = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    Q.check(Q.lib.q_b200_q4_pack(dw.data_ptr(), M, K, packed.data_ptr(), None), "pack")
    return packed, torch.from_numpy(x).cuda()


@pytest.mark.parametrize("M,K", [(4096, 4096), (28672, 4096), (4096, 14336), (100, 768)])
def test_noalloc_matches_gemv_q4_twice(torch, M, K):
    packed, dx = _packed(torch, M, K, seed=M ^ K)
    ref = torch.empty(M, dtype=torch.float32, device="cuda")
    Q.check(Q.lib.q_b200_gemv_q4(packed.data_ptr(), M, K, dx.data_ptr(), ref.data_ptr(), None), "gemv")
    torch.cuda.synchronize()
    ref = ref.cpu().numpy().astype(np.float64)
    for _ in range(2):  # second call: tickets left zero by the first
        out = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
        Q.check(Q.lib.q_b200_gemv_q4_noalloc(packed.data_ptr(), M, K, dx.data_ptr(),
                                             out.data_ptr(), None), "gemv noalloc")
        torch.cuda.synchronize()
        got = out.cpu().numpy().astype(np.float64)
        err = np.abs(got - ref)
        assert (err <= np.maximum(1.5e-4, 1e-4 * np.abs(ref))).all(), f"worst {err.max():.3e}"


def test_noalloc_allocates_nothing(torch):
    """The point of the entry point: its calls make no device allocation.
    Checked with the library's own count of cudaMalloc calls, in a fresh
    process so that no earlier test has grown a shared buffer already."""
    import subprocess
    import sys
    from pathlib import Path
    code = r"""
import sys
sys.path.insert(0, %r)
import numpy as np, torch, qorus_b200 as Q
M, K = 4096, 4096
nblk = M * K // 32
w = np.zeros(nblk * 20, np.uint8)
Q.lib.q_b200_fill_q4(Q.ptr(w), nblk, 5, 11, 0, 0.001, 0.01, 0)
dw = torch.from_numpy(w).cuda()
packed = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
x = torch.randn(K, device="cuda")
y = torch.empty(M, device="cuda")
torch.cuda.synchronize()
Q.check(Q.lib.q_b200_q4_pack(dw.data_ptr(), M, K, packed.data_ptr(), None), "pack")
torch.cuda.synchronize()
before = Q.lib.q_b200_device_allocations()
for _ in range(3):
    Q.check(Q.lib.q_b200_gemv_q4_noalloc(packed.data_ptr(), M, K, x.data_ptr(), y.data_ptr(), None), "noalloc")
torch.cuda.synchronize()
after = Q.lib.q_b200_device_allocations()
Q.check(Q.lib.q_b200_gemv_q4(packed.data_ptr(), M, K, x.data_ptr(), y.data_ptr(), None), "gemv")
torch.cuda.synchronize()
print(before, after, Q.lib.q_b200_device_allocations())
""" % str(Path(__file__).resolve().parents[1] / "project-ia_b200")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    before, after, with_alloc = map(int, out.stdout.split()[-3:])
    assert after == before
    assert with_alloc > after  # the allocating entry point does allocate: the count is live


def test_noalloc_rejects_oversized_plan(torch):
    # 262144 x 32: 16384 slabs of one block each, whose partial sums
    # (about 3 MiB) exceed the fixed scratch
    M, K = 262144, 32
    packed, dx = _packed(torch, M, K, seed=3)
    out = torch.empty(M, dtype=torch.float32, device="cuda")
    rc = Q.lib.q_b200_gemv_q4_noalloc(packed.data_ptr(), M, K, dx.data_ptr(), out.data_ptr(), None)
    assert rc == -15  # Q_ERR_INVALID_SIZE
    assert "limit" in Q.last_error()
