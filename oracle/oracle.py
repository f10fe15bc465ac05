"""ctypes bindings of the CPU checkers — TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs, never by the product.  Three libraries:

  liboracle.so             the C restatement (oracle.c), always built
  _ref/libqorus_ref.so     the upstream sources compiled in place (optional:
                           needs the upstream tree at build time; the built
                           .so travels with the repository snapshot)
  _ref/libref_forward.so   ref_forward.c over libqorus_ref.so
  libqgen.so               the package's synthetic-input generators (qgen.c)
                           alone, so a CPU-only process can write the model
                           file and KV image without loading the CUDA library
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_vp, _u32, _sz, _f, _i = C.c_void_p, C.c_uint32, C.c_size_t, C.c_float, C.c_int


def _load(name: str) -> C.CDLL | None:
    p = HERE / name
    return C.CDLL(str(p)) if p.exists() else None


orc = _load("liboracle.so")
if orc is None:
    raise ImportError("oracle/liboracle.so missing: run `make -C oracle`")
for fn, res, args in [
    ("orc_exp_approx", _f, [_f]),
    ("orc_dequantize_block", None, [_vp, _vp]),
    ("orc_gemv_q4", _i, [_vp, _u32, _u32, _vp, _vp]),
    ("orc_dot_f32", _f, [_vp, _vp, _u32]),
    ("orc_gemv_f32", _i, [_vp, _u32, _u32, _vp, _vp]),
    ("orc_rmsnorm", _i, [_vp, _vp, _vp, _u32, _f]),
    ("orc_rope", _i, [_vp, _vp, _vp, _vp, _u32]),
    ("orc_softmax", _i, [_vp, _vp, _u32]),
    ("orc_silu", _i, [_vp, _vp, _u32]),
    ("orc_rope_tables", None, [_f, _u32, _u32, _vp, _vp]),
    ("orc_model_open", _i, [_vp, _vp, _sz]),
    ("orc_model_close", None, [_vp]),
    ("orc_forward", _i, [_vp, _vp, _vp, _u32, _u32, _vp]),
    ("orc_argmax", _u32, [_vp, _u32]),
    ("orc_set_threads", None, [_i]),
]:
    f = getattr(orc, fn)
    f.restype, f.argtypes = res, args

try:
    ref = _load("_ref/libqorus_ref.so")
    rf = _load("_ref/libref_forward.so")
except OSError:  # built for a CPU feature this host lacks
    ref = rf = None
if rf is not None:
    rf.rf_open.restype, rf.rf_open.argtypes = _vp, [_vp, _sz]
    rf.rf_close.restype, rf.rf_close.argtypes = None, [_vp]
    rf.rf_forward.restype, rf.rf_forward.argtypes = _i, [_vp, _vp, _vp, _u32, _u32, _vp]
    rf.rf_set_threads.restype, rf.rf_set_threads.argtypes = None, [_i]


def p(a: np.ndarray) -> int:
    return a.ctypes.data


# ---- synthetic inputs without the CUDA library (libqgen.so) --------------------

class Config(C.Structure):
    """q_llama_config (include/qorus_types.h)."""
    _fields_ = [(n, C.c_uint32) for n in (
        "vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "max_seq_len")] + [
        ("rope_freq_base", C.c_float), ("rms_norm_eps", C.c_float)]


gen = _load("libqgen.so")
if gen is not None:
    gen.q_b200_model_file_size.restype, gen.q_b200_model_file_size.argtypes = _sz, [_vp]
    gen.q_b200_write_model_file.restype = _i
    gen.q_b200_write_model_file.argtypes = [C.c_char_p, _vp, C.c_uint64, _i]
    gen.q_b200_fill_kv_prefill.restype, gen.q_b200_fill_kv_prefill.argtypes = _i, [_vp, _vp, _u32, C.c_uint64, _i]
    gen.q_b200_fill_q4.restype = None
    gen.q_b200_fill_q4.argtypes = [_vp, _sz, C.c_uint64, C.c_uint64, C.c_uint64, _f, _f, _i]
    gen.q_b200_fill_normal.restype = None
    gen.q_b200_fill_normal.argtypes = [_vp, _sz, C.c_uint64, C.c_uint64, C.c_uint64, _f, _f, _i]


def config(vocab, dim, hidden, layers, heads, kv_heads, max_seq, theta=500000.0, eps=1e-5) -> Config:
    return Config(vocab, dim, hidden, layers, heads, kv_heads, max_seq, theta, eps)


# ---- the upstream GEMV itself (oracle/_ref), for timing beside the device -------

class _QTensor(C.Structure):
    """q_tensor (include/qorus_types.h: 64-byte aligned)."""
    _fields_ = [("data", C.c_void_p), ("scales", C.c_void_p), ("ne", C.c_uint32 * 4),
                ("nb", C.c_size_t * 4), ("type", C.c_int), ("name", C.c_char * 32),
                ("_pad", C.c_uint8 * 28)]


def upstream_gemv_q4(w_aos: np.ndarray, M: int, K: int, x: np.ndarray, y: np.ndarray) -> str:
    """y = W x with upstream q_gemv_q4_f32_avx2 when oracle/_ref is built
    (returns "reference"), else the restatement orc_gemv_q4 ("port").
    x and y must be 32-byte aligned."""
    if ref is not None:
        t = _QTensor()
        t.data = w_aos.ctypes.data
        t.ne[:] = [M, K, 1, 1]
        t.nb[:] = [K // 32 * 20, 20, 20, 20]
        t.type = 2  # Q_Q4_0
        rc = ref.q_gemv_q4_f32_avx2(C.byref(t), C.c_void_p(p(x)), C.c_void_p(p(y)))
        if rc:
            raise RuntimeError(f"q_gemv_q4_f32_avx2: {rc}")
        return "reference"
    orc.orc_set_threads(1)
    if orc.orc_gemv_q4(p(w_aos), M, K, p(x), p(y)):
        raise RuntimeError("orc_gemv_q4")
    return "port"


def _header(mm):
    hdr = np.frombuffer(mm[:64].tobytes(), np.uint32)
    return (int(v) for v in hdr[2:9])


class OracleModel:
    """orc_forward over a .qorus file (mmapped read-only) with a host KV image."""

    def __init__(self, path: str, threads: int = 1):
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.h = (C.c_uint8 * (16384 * 8))()  # sizeof(orc_model) is < 64 KiB
        rc = orc.orc_model_open(self.h, p(self.mm), self.mm.size)
        if rc:
            raise RuntimeError(f"orc_model_open: {rc}")
        (self.vocab, self.dim, self.hidden, self.layers, self.heads, self.kv_heads,
         self.max_seq) = _header(self.mm)
        self.hd = self.dim // self.heads
        self.kv = np.zeros(self.layers * self.kv_heads * self.max_seq * 2 * self.hd, np.float32)
        self.logits = np.zeros(self.vocab, np.float32)
        orc.orc_set_threads(threads)

    def forward(self, tokens, pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        rc = orc.orc_forward(self.h, p(self.kv), p(t), len(t), pos, p(self.logits))
        if rc:
            raise RuntimeError(f"orc_forward: {rc}")
        return self.logits

    def close(self):
        orc.orc_model_close(self.h)


class RefModel:
    """rf_forward: the intended graph over the upstream AVX2 kernels."""

    def __init__(self, path: str, threads: int = 1):
        if rf is None:
            raise RuntimeError("oracle/_ref/libref_forward.so not built")
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.h = rf.rf_open(p(self.mm), self.mm.size)
        if not self.h:
            raise RuntimeError("rf_open failed")
        (self.vocab, self.dim, self.hidden, self.layers, self.heads, self.kv_heads,
         self.max_seq) = _header(self.mm)
        self.hd = self.dim // self.heads
        self.kv = np.zeros(self.layers * self.kv_heads * self.max_seq * 2 * self.hd, np.float32)
        self.logits = np.zeros(self.vocab, np.float32)
        rf.rf_set_threads(threads)

    def forward(self, tokens, pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        rc = rf.rf_forward(self.h, p(self.kv), p(t), len(t), pos, p(self.logits))
        if rc:
            raise RuntimeError(f"rf_forward: {rc}")
        return self.logits

    def close(self):
        if self.h:
            rf.rf_close(self.h)
            self.h = None
