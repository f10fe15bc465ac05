"""Regenerate tests/golden/ from the upstream implementation (run in the build
container, where the upstream tree and oracle/_ref are present):

    python tests/golden/make_golden.py

Writes:
  dequantize_test{1..4}_{block,expected}.bin   upstream test_data fixtures
      (tools/gen_test_dequantize.py output shipped upstream), copied verbatim
  golden.npz   outputs of the UPSTREAM code itself on seeded inputs:
      - q_gemv_q4_f32_avx2 on the upstream tests/test_matmul.c:92-107 shapes
        plus the Llama-3-8B projection widths (4 rows each)
      - q_softmax / q_silu on lengths that exercise the vector/tail split
      - q_rmsnorm / q_rope
      - rf_forward (upstream kernels, intended graph) on the tiny config:
        prompt logits and 32 greedy tokens
      - upstream llama_forward itself on a square config (seq_len 1, pos 0)
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "project-ia_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402
import qorus_b200 as Q  # noqa: E402

# the upstream source tree: $QORUS_REFERENCE, else a "reference" directory beside this repository
UPSTREAM = Path(os.environ.get("QORUS_REFERENCE", str(Path(__file__).resolve().parents[3] / "reference")))
OUT = Path(__file__).resolve().parent


def al(n, dt=np.float32):
    return Q.aligned_empty(n, dt)


def main():
    assert O.ref is not None and O.rf is not None, "build oracle/_ref first (make -C oracle)"
    for i in range(1, 5):
        for kind in ("block", "expected"):
            name = f"dequantize_test{i}_{kind}.bin"
            shutil.copyfile(UPSTREAM / "test_data" / name, OUT / name)

    g = {}
    rng = np.random.default_rng(42)
    ref = O.ref
    ref.q_gemv_q4_f32_avx2.argtypes = [C.c_void_p] * 3
    shapes = [(1, 32), (4, 64), (16, 128), (64, 256), (32, 512), (128, 1024),
              (4, 4096), (4, 14336)]
    for M, K in shapes:
        w = al(M * K // 32 * 20, np.uint8)
        Q.lib.q_b200_fill_q4(Q.ptr(w), M * K // 32, 42, M * 100003 + K, 0, 0.001, 0.01, 1)
        x = al(K)
        x[:] = rng.standard_normal(K).astype(np.float32)
        y = al(M)
        t = Q.q_tensor()
        t.data = w.ctypes.data
        t.ne[:] = [M, K, 1, 1]
        t.nb[:] = [K // 32 * 20, 20, 20, 20]
        t.type = Q.Q_Q4_0
        assert ref.q_gemv_q4_f32_avx2(C.addressof(t), x.ctypes.data, y.ctypes.data) == 0
        g[f"gemv_{M}x{K}_w"] = w.copy()
        g[f"gemv_{M}x{K}_x"] = x.copy()
        g[f"gemv_{M}x{K}_y"] = y.copy()
    ref.q_softmax_f32_avx2.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32]
    ref.q_silu_f32_avx2.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32]
    for N in (1, 3, 7, 8, 9, 15, 16, 33, 100, 2049):
        x = al(N)
        x[:] = (rng.standard_normal(N) * 3).astype(np.float32)
        a, b = al(N), al(N)
        assert ref.q_softmax_f32_avx2(x.ctypes.data, a.ctypes.data, N) == 0
        assert ref.q_silu_f32_avx2(x.ctypes.data, b.ctypes.data, N) == 0
        g[f"softmax_{N}_x"], g[f"softmax_{N}_y"], g[f"silu_{N}_y"] = x.copy(), a.copy(), b.copy()
    ref.q_rmsnorm_f32_avx2.argtypes = [C.c_void_p] * 3 + [C.c_uint32, C.c_float]
    ref.q_rope_f32_avx2.argtypes = [C.c_void_p] * 4 + [C.c_uint32]
    for N in (8, 64, 256, 4096):
        x, w, o = al(N), al(N), al(N)
        x[:] = rng.standard_normal(N).astype(np.float32)
        w[:] = (1 + 0.02 * rng.standard_normal(N)).astype(np.float32)
        assert ref.q_rmsnorm_f32_avx2(x.ctypes.data, w.ctypes.data, o.ctypes.data, N, 1e-5) == 0
        c, s, r = al(N), al(N), al(N)
        c[:] = np.repeat(rng.standard_normal(N // 2), 2).astype(np.float32)
        s[:] = np.repeat(rng.standard_normal(N // 2), 2).astype(np.float32)
        assert ref.q_rope_f32_avx2(x.ctypes.data, c.ctypes.data, s.ctypes.data, r.ctypes.data, N) == 0
        g[f"rms_{N}_x"], g[f"rms_{N}_w"], g[f"rms_{N}_y"] = x.copy(), w.copy(), o.copy()
        g[f"rope_{N}_c"], g[f"rope_{N}_s"], g[f"rope_{N}_y"] = c.copy(), s.copy(), r.copy()

    with tempfile.TemporaryDirectory() as td:
        cfg = Q.config(**Q.TINY)
        path = Path(td) / "tiny.qorus"
        Q.write_model(str(path), cfg, seed=0, threads=1)
        g["tiny_sha256"] = np.frombuffer(hashlib.sha256(path.read_bytes()).digest(), np.uint8)
        prompt = np.zeros(64, np.uint32)
        Q.lib.q_b200_fill_tokens(Q.ptr(prompt), 64, 0, 7, 0, cfg.vocab_size)
        prompt[0] = 256
        m = O.RefModel(str(path))
        logits = m.forward(prompt, 0).copy()
        toks = [int(np.argmax(logits))]
        for i in range(31):
            lg = m.forward(np.array([toks[-1]], np.uint32), 64 + i)
            toks.append(int(np.argmax(lg)))
        g["tiny_prompt"], g["tiny_prefill_logits"] = prompt, logits
        g["tiny_tokens"] = np.array(toks, np.uint32)
        g["tiny_last_logits"] = m.logits.copy()
        m.close()
        # the upstream llama_forward itself, square config, seq_len 1, pos 0
        sq = Q.config(259, 256, 256, 2, 8, 8, 64)
        spath = Path(td) / "square.qorus"
        Q.write_model(str(spath), sq, seed=3, threads=1)
        ctx = (C.c_uint8 * 256)()
        model = (C.c_uint8 * 1024)()
        ref.q_init_memory.argtypes = [C.c_void_p, C.c_char_p]
        ref.q_alloc_kv_cache.argtypes = [C.c_void_p, C.c_size_t]
        ref.q_alloc_arena.argtypes = [C.c_void_p, C.c_size_t]
        ref.llama_build_graph.argtypes = [C.c_void_p, C.c_void_p]
        ref.llama_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32,
                                      C.c_void_p]
        ref.q_free_memory.argtypes = [C.c_void_p]
        assert ref.q_init_memory(ctx, str(spath).encode()) == 0
        assert ref.q_alloc_kv_cache(ctx, Q.kv_bytes(sq)) == 0
        assert ref.q_alloc_arena(ctx, 64 << 20) == 0
        assert ref.llama_build_graph(ctx, model) == 0
        lg = al(259)
        tok = np.array([17], np.uint32)
        assert ref.llama_forward(model, ctx, tok.ctypes.data, 1, 0, lg.ctypes.data) == 0
        g["square_token"], g["square_logits"] = tok, lg.copy()
        ref.q_free_memory(ctx)
    np.savez_compressed(OUT / "golden.npz", **g)
    print("wrote", OUT / "golden.npz", sum(v.nbytes for v in g.values()), "bytes")


if __name__ == "__main__":
    main()
