"""qorus_b200 — Python bindings of libqorus_b200.so (the Qorus-IA C API on a B200).

The library exports the upstream C API (include/qorus.h: q_init_memory,
q_alloc_kv_cache, q_alloc_arena, llama_build_graph, llama_forward,
q_generate, the kernel-level q_*_f32_avx2 entry points) and the additive
entry points of include/qorus_b200.h.  This module binds them with ctypes and
adds a small `Model` wrapper whose methods call exactly those entry points in
upstream's required order (init -> kv -> arena -> build, as in upstream
tests/test_llama_forward.c:58-107).

There is no CPU fallback: importing raises if the shared library is missing,
and every call returns the library's q_error_code (raised as QorusError).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE.parent / "lib" / "libqorus_b200.so"

Q_OK = 0
ERRORS = {
    0: "Q_OK", -1: "Q_ERR_NULL_PTR", -2: "Q_ERR_FILE_OPEN", -3: "Q_ERR_FILE_STAT",
    -4: "Q_ERR_FILE_TOO_SMALL", -5: "Q_ERR_MMAP_FAILED", -6: "Q_ERR_INVALID_MAGIC",
    -7: "Q_ERR_ALLOC_FAILED", -8: "Q_ERR_ARENA_OOM", -9: "Q_ERR_INVALID_CONFIG",
    -10: "Q_ERR_INVALID_ARG", -11: "Q_ERR_ALIASING", -12: "Q_ERR_OVERFLOW",
    -13: "Q_ERR_MISALIGNED", -14: "Q_ERR_INVALID_DTYPE", -15: "Q_ERR_INVALID_SIZE",
}
Q_F32, Q_Q8_0, Q_Q4_0 = 0, 1, 2


class QorusError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        msg = f"{where}: {ERRORS.get(code, code)}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


# ---- ABI structs (include/qorus_types.h) -------------------------------------

class q_llama_config(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in (
        "vocab_size", "dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads", "max_seq_len")] + [
        ("rope_freq_base", C.c_float), ("rms_norm_eps", C.c_float)]


class q_context(C.Structure):
    _fields_ = [("weights_mmap", C.c_void_p), ("weights_size", C.c_size_t), ("header", C.c_void_p),
                ("kv_buffer", C.c_void_p), ("kv_size", C.c_size_t),
                ("scratch_buffer", C.c_void_p), ("scratch_size", C.c_size_t),
                ("scratch_head", C.c_size_t), ("scratch_base_offset", C.c_size_t)]


class q_tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scales", C.c_void_p), ("ne", C.c_uint32 * 4),
                ("nb", C.c_size_t * 4), ("type", C.c_int), ("name", C.c_char * 32),
                ("_pad", C.c_uint8 * 28)]  # the C struct is aligned (and padded) to 64 bytes


class q_llama_layer(C.Structure):
    _fields_ = [("layer_idx", C.c_uint32)] + [(n, C.POINTER(q_tensor)) for n in (
        "attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")]


class q_llama_model(C.Structure):
    _fields_ = [("config", q_llama_config), ("token_embd", C.POINTER(q_tensor)),
                ("output_norm", C.POINTER(q_tensor)), ("output", C.POINTER(q_tensor)),
                ("layers", C.POINTER(q_llama_layer)), ("rope_freqs", C.POINTER(C.c_float)),
                ("rope_cache_enabled", C.c_bool), ("rope_cos_cache", C.POINTER(C.c_float)),
                ("rope_sin_cache", C.POINTER(C.c_float)), ("ctx", C.POINTER(q_context))]


class q_tokenizer(C.Structure):
    _fields_ = [("vocab", C.c_void_p), ("vocab_size", C.c_uint32), ("merges", C.c_void_p),
                ("num_merges", C.c_uint32), ("merge_hash_table", C.c_void_p),
                ("bos_token_id", C.c_uint32), ("eos_token_id", C.c_uint32),
                ("pad_token_id", C.c_uint32), ("initialized", C.c_bool)]


class q_generation_state(C.Structure):
    _fields_ = [("ctx", C.POINTER(q_context)), ("model", C.POINTER(q_llama_model)),
                ("tokenizer", C.POINTER(q_tokenizer)),
                ("prompt_tokens", C.POINTER(C.c_uint32)), ("num_prompt_tokens", C.c_uint32),
                ("generated_tokens", C.POINTER(C.c_uint32)), ("num_generated_tokens", C.c_uint32),
                ("max_tokens", C.c_uint32), ("temperature", C.c_float), ("top_k", C.c_uint32),
                ("top_p", C.c_float), ("current_pos", C.c_uint32)]


_vp, _sz, _u32, _u64, _f, _i = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_float, C.c_int
# Every function include/qorus.h and include/qorus_b200.h declare.
_SIGS = {
    "q_init_memory": (_i, [_vp, C.c_char_p]),
    "q_init_memory_ex": (_i, [_vp, C.c_char_p, _i]),
    "q_alloc_kv_cache": (_i, [_vp, _sz]),
    "q_alloc_arena": (_i, [_vp, _sz]),
    "q_arena_alloc": (_vp, [_vp, _sz]),
    "q_arena_reset": (None, [_vp]),
    "q_free_memory": (None, [_vp]),
    "q_strerror": (C.c_char_p, [_i]),
    "q_dequantize_q4_0_block_avx2_public": (None, [_vp, _vp]),
    "q_gemv_q4_f32_avx2": (_i, [_vp, _vp, _vp]),
    "q_matmul_f32_avx2": (_i, [_vp, _vp, _vp, _vp]),
    "q_causal_mask_f32_avx2": (_i, [_vp, _f]),
    "q_add_f32_avx2": (_i, [_vp, _vp, _vp]),
    "q_mul_f32_avx2": (_i, [_vp, _vp, _vp]),
    "q_rmsnorm_f32_avx2": (_i, [_vp, _vp, _vp, _u32, _f]),
    "q_rope_f32_avx2": (_i, [_vp, _vp, _vp, _vp, _u32]),
    "q_silu_f32_avx2": (_i, [_vp, _vp, _u32]),
    "q_softmax_f32_avx2": (_i, [_vp, _vp, _u32]),
    "llama_build_graph": (_i, [_vp, _vp]),
    "llama_free_graph": (None, [_vp]),
    "llama_forward": (_i, [_vp, _vp, _vp, _u32, _u32, _vp]),
    "q_sample_token": (_i, [_vp, _u32, _f, _u32, _f, _vp, _vp]),
    "q_generate": (_i, [_vp]),
    "q_tokenizer_load": (_i, [_vp, C.c_char_p]),
    "q_tokenizer_encode": (_i, [_vp, C.c_char_p, _vp, _vp, C.c_uint32, C.c_bool, C.c_bool]),
    "q_tokenizer_decode": (_i, [_vp, _vp, C.c_uint32, _vp, _sz]),
    "q_tokenizer_free": (None, [_vp]),
    "q_b200_model_file_size": (_sz, [_vp]),
    "q_b200_write_model_file": (_i, [C.c_char_p, _vp, _u64, _i]),
    "q_b200_fill_normal": (None, [_vp, _sz, _u64, _u64, _u64, _f, _f, _i]),
    "q_b200_fill_tokens": (None, [_vp, _sz, _u64, _u64, _u64, _u32]),
    "q_b200_fill_q4": (None, [_vp, _sz, _u64, _u64, _u64, _f, _f, _i]),
    "q_b200_fill_kv_prefill": (_i, [_vp, _vp, _u32, _u64, _i]),
    "q_b200_kv_write": (_i, [_vp, _sz, _vp, _sz]),
    "q_b200_kv_read": (_i, [_vp, _sz, _vp, _sz]),
    "q_b200_stream": (_vp, [_vp]),
    "q_b200_decode_greedy": (_i, [_vp, _vp, _u32, _u32, _vp]),
    "q_b200_decode_loop": (_i, [_vp, _vp, _u32, _u32, _u32, _vp, _i]),
    "q_b200_profile_step": (_i, [_vp, _vp, _u32, _u32, _vp, _u32, _vp]),
    "q_b200_device_logits": (_vp, [_vp]),
    "q_b200_batch_init": (_i, [_vp, _vp, _u32]),
    "q_b200_batch_init_paged": (_i, [_vp, _vp, _u32, _u32, _u32]),
    "q_b200_batch_release": (_i, [_vp, _u32]),
    "q_b200_batch_kv_write": (_i, [_vp, _u32, _sz, _vp, _sz]),
    "q_b200_batch_kv_read": (_i, [_vp, _u32, _sz, _vp, _sz]),
    "q_b200_decode_batch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "q_b200_decode_batch_loop": (_i, [_vp, _vp, _vp, _vp, _u32, _vp, _i]),
    "q_b200_q4_packed_bytes": (_sz, [_u32, _u32]),
    "q_b200_q4_pack": (_i, [_vp, _u32, _u32, _vp, _vp]),
    "q_b200_gemv_q4": (_i, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "q_b200_gemv_q4_noalloc": (_i, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "q_b200_gemm_q4": (_i, [_vp, _u32, _u32, _vp, _u32, _vp, _vp]),
    "q_b200_gemv_f32": (_i, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "q_b200_tp_unique_id": (_i, [_vp, _sz]),
    "q_b200_tp_init": (_i, [_vp, _u32, _u32, _vp, _sz]),
    "q_b200_tp_ipc_handle": (_i, [_vp, _vp, _sz]),
    "q_b200_tp_ipc_open": (_i, [_vp, _vp, _sz]),
    "q_b200_tp_shape": (_i, [_vp, _u32, _u32, _vp, _u32]),
    "q_b200_set_wait_limit_ns": (_i, [_u64]),
    "q_b200_device_status": (_u32, []),
    "q_b200_selftest_exchange_timeout": (_i, [_u64, _vp]),
    "q_b200_kernel_launches": (_u64, []),
    "q_b200_device_allocations": (_u64, []),
    "q_b200_last_error": (C.c_char_p, []),
}
EXPORTS = tuple(_SIGS)


def load_library(path: os.PathLike | str | None = None) -> C.CDLL:
    """Load libqorus_b200.so and set every prototype.  Raises if it is missing."""
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} not built: run `make -C project-ia_b200` (or __graft_entry__.build())")
    lib = C.CDLL(str(p))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load_library()


def last_error() -> str:
    s = lib.q_b200_last_error()
    return s.decode() if s else ""


def check(rc: int, where: str) -> None:
    if rc != Q_OK:
        raise QorusError(rc, where, last_error())


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def aligned_empty(n: int, dtype=np.float32, align: int = 64) -> np.ndarray:
    """A host array whose data pointer is `align`-byte aligned (upstream wants 32)."""
    dt = np.dtype(dtype)
    raw = np.empty(n * dt.itemsize + align, np.uint8)
    off = (-raw.ctypes.data) % align
    return raw[off:off + n * dt.itemsize].view(dt)


def config(vocab, dim, hidden, layers, heads, kv_heads, max_seq, theta=500000.0, eps=1e-5):
    return q_llama_config(vocab, dim, hidden, layers, heads, kv_heads, max_seq, theta, eps)


# Configurations of the benchmark suite (BASELINE.json "configs").
TINY = dict(vocab=259, dim=256, hidden=768, layers=2, heads=8, kv_heads=2, max_seq=512)
LLAMA3_8B = dict(vocab=128256, dim=4096, hidden=14336, layers=32, heads=32, kv_heads=8)


def tp_unique_id() -> bytes:
    """128-byte NCCL id for q_b200_tp_init (made once, on rank 0)."""
    buf = C.create_string_buffer(128)
    check(lib.q_b200_tp_unique_id(buf, 128), "q_b200_tp_unique_id")
    return buf.raw


def tp_shape(cfg: q_llama_config, rank: int, world: int) -> dict:
    """Shard geometry of a tensor-parallel rank (q_b200_tp_shape)."""
    out = (C.c_uint32 * 13)()
    check(lib.q_b200_tp_shape(C.byref(cfg), rank, world, out, 13), "q_b200_tp_shape")
    keys = ("rank", "world", "nh", "nkv", "d", "kvd", "q0", "kv0", "h", "h0", "v", "v0", "v_pad")
    return dict(zip(keys, list(out)))


def write_model(path: str, cfg: q_llama_config, seed: int = 0, threads: int = 0) -> int:
    check(lib.q_b200_write_model_file(str(path).encode(), C.byref(cfg), seed, threads),
          "q_b200_write_model_file")
    return int(lib.q_b200_model_file_size(C.byref(cfg)))


def kv_bytes(cfg: q_llama_config) -> int:
    hd = cfg.dim // cfg.n_heads
    return cfg.n_layers * cfg.n_kv_heads * cfg.max_seq_len * hd * 2 * 4


class Model:
    """A model loaded through the upstream API: init -> kv -> arena -> build."""

    def __init__(self, path: str, arena_bytes: int | None = None, tp: tuple | None = None,
                 tp_gather=None):
        """tp = (rank, world, nccl_id bytes) for a tensor-parallel rank (one process per GPU,
        its device current); the id comes from tp_unique_id() on rank 0.  tp_gather, if given,
        maps one bytes object per rank to the list of all ranks' (rank order); with it the
        ranks share CUDA IPC handles and all-reduce over peer memory instead of NCCL."""
        self.ctx = q_context()
        self.model = q_llama_model()
        check(lib.q_init_memory(C.byref(self.ctx), str(path).encode()), "q_init_memory")
        if tp is not None:
            rank, world, uid = tp
            buf = C.create_string_buffer(bytes(uid), len(uid))
            check(lib.q_b200_tp_init(C.byref(self.ctx), rank, world, buf, len(uid)), "q_b200_tp_init")
            if tp_gather is not None and world > 1:
                h = C.create_string_buffer(64)
                check(lib.q_b200_tp_ipc_handle(C.byref(self.ctx), h, 64), "q_b200_tp_ipc_handle")
                allh = b"".join(tp_gather(h.raw))
                hb = C.create_string_buffer(allh, len(allh))
                check(lib.q_b200_tp_ipc_open(C.byref(self.ctx), hb, len(allh)), "q_b200_tp_ipc_open")
        hdr = np.frombuffer((C.c_uint32 * 16).from_address(self.ctx.header), np.uint32)
        cfg = config(int(hdr[2]), int(hdr[3]), int(hdr[4]), int(hdr[5]), int(hdr[6]),
                     int(hdr[7]), int(hdr[8]))
        self.kv_size = kv_bytes(cfg)
        check(lib.q_alloc_kv_cache(C.byref(self.ctx), self.kv_size), "q_alloc_kv_cache")
        if arena_bytes is None:
            hd = cfg.dim // cfg.n_heads
            arena_bytes = (64 << 20) + 2 * cfg.max_seq_len * hd * 4 + \
                cfg.n_heads * cfg.max_seq_len * (8 + hd) + cfg.vocab_size * 8
        check(lib.q_alloc_arena(C.byref(self.ctx), arena_bytes), "q_alloc_arena")
        check(lib.llama_build_graph(C.byref(self.ctx), C.byref(self.model)), "llama_build_graph")
        self.cfg = self.model.config
        self.logits = aligned_empty(self.cfg.vocab_size)

    def forward(self, tokens, pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        check(lib.llama_forward(C.byref(self.model), C.byref(self.ctx), ptr(t), len(t), pos,
                                ptr(self.logits)), "llama_forward")
        return self.logits

    def decode_loop(self, first_token: int, pos: int, n: int, sync: bool = True) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        check(lib.q_b200_decode_loop(C.byref(self.model), C.byref(self.ctx), first_token, pos, n,
                                     ptr(out), 1 if sync else 0), "q_b200_decode_loop")
        return out

    def profile_step(self, token: int, pos: int) -> np.ndarray:
        """[kernel][entry, wait-end, exit] globaltimer ns of one traced decode step."""
        out = np.zeros((1024, 3), np.uint64)
        n = C.c_uint32()
        check(lib.q_b200_profile_step(C.byref(self.model), C.byref(self.ctx), token, pos, ptr(out),
                                      1024, C.byref(n)), "q_b200_profile_step")
        return out[: n.value]

    def kv_write(self, host: np.ndarray, offset: int = 0) -> None:
        check(lib.q_b200_kv_write(C.byref(self.ctx), offset, ptr(host), host.nbytes), "kv_write")

    def kv_read(self, host: np.ndarray, offset: int = 0) -> None:
        check(lib.q_b200_kv_read(C.byref(self.ctx), offset, ptr(host), host.nbytes), "kv_read")

    @property
    def stream(self) -> int:
        return lib.q_b200_stream(C.byref(self.ctx)) or 0

    def close(self) -> None:
        if self.ctx.weights_mmap or self.ctx.kv_buffer or self.ctx.scratch_buffer:
            lib.llama_free_graph(C.byref(self.model))
            lib.q_free_memory(C.byref(self.ctx))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

