"""The C-ABI boundary without a GPU: the library loads, exports every symbol the
headers declare, its structs have upstream's layout, the host-side logic
(file parsing, validation order, generators, greedy sampling) behaves like
upstream.  No call here launches a kernel."""
import ctypes as C
import os
import re
import subprocess
from pathlib import Path

import numpy as np

import qorus_b200 as Q
from conftest import ROOT

HEADERS = [ROOT / "include" / "qorus.h", ROOT / "include" / "qorus_b200.h"]
# upstream headers: $QORUS_REFERENCE/include, else a "reference" directory beside this repository
UPSTREAM_INCLUDE = Path(os.environ.get("QORUS_REFERENCE", str(Path(__file__).resolve().parents[2] / "reference"))) / "include"


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"^#.*$", "", text, flags=re.M)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 40
    for n in sorted(names):
        assert hasattr(Q.lib, n), n
    assert set(Q.EXPORTS) == names


LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "qorus.h"
#define P(T) printf(#T " %zu %zu\n", sizeof(T), _Alignof(T));
#define O(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  P(q_block_q4_0) P(q_model_header) P(q_tensor) P(q_context) P(q_llama_config)
  P(q_llama_layer) P(q_llama_model) P(q_generation_state) P(q_tokenizer)
  O(q_tensor, nb) O(q_tensor, type) O(q_tensor, name) O(q_context, kv_buffer)
  O(q_context, scratch_base_offset) O(q_llama_model, layers) O(q_llama_model, ctx)
  O(q_model_header, rms_norm_eps) O(q_generation_state, current_pos)
  return 0;
}
"""


def _layout(include: Path, tmp_path: Path, tag: str) -> str:
    src = tmp_path / f"layout_{tag}.c"
    exe = tmp_path / f"layout_{tag}"
    src.write_text(LAYOUT_C)
    subprocess.run(["gcc", "-std=c11", "-D_GNU_SOURCE", f"-I{include}", str(src), "-o", str(exe)],
                   check=True, capture_output=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout


def test_struct_layout(tmp_path):
    mine = _layout(ROOT / "include", tmp_path, "mine")
    assert "q_block_q4_0 20 1" in mine and "q_model_header 64 64" in mine
    if UPSTREAM_INCLUDE.exists():  # the build container: compare with upstream's header
        assert mine == _layout(UPSTREAM_INCLUDE, tmp_path, "upstream")
    # and the ctypes mirror
    sizes = dict(line.split()[:2] for line in mine.splitlines() if "." not in line.split()[0])
    assert C.sizeof(Q.q_context) == int(sizes["q_context"])
    assert C.sizeof(Q.q_llama_config) == int(sizes["q_llama_config"])
    assert C.sizeof(Q.q_tensor) == int(sizes["q_tensor"])
    assert C.sizeof(Q.q_llama_model) == int(sizes["q_llama_model"])
    assert C.sizeof(Q.q_generation_state) == int(sizes["q_generation_state"])


def test_strerror_and_file_errors(tmp_path):
    assert Q.lib.q_strerror(0) == b"Success"
    assert Q.lib.q_strerror(-8) == b"Arena Out of Memory"
    assert Q.lib.q_strerror(-99) == b"Unknown error"
    ctx = Q.q_context()
    assert Q.lib.q_init_memory(C.byref(ctx), str(tmp_path / "missing").encode()) == -2
    small = tmp_path / "small.qorus"
    small.write_bytes(b"\0" * 10)
    assert Q.lib.q_init_memory(C.byref(ctx), str(small).encode()) == -4
    bad = tmp_path / "bad.qorus"
    bad.write_bytes(b"\1" * 128)
    assert Q.lib.q_init_memory(C.byref(ctx), str(bad).encode()) == -6
    assert Q.lib.q_init_memory(None, b"x") == -10


def test_build_graph_validation_without_gpu(tiny_path):
    ctx, model = Q.q_context(), Q.q_llama_model()
    assert Q.lib.llama_build_graph(None, C.byref(model)) == -1
    assert Q.lib.llama_build_graph(C.byref(ctx), C.byref(model)) == -1  # nothing mapped
    assert Q.lib.q_init_memory(C.byref(ctx), tiny_path.encode()) == 0
    # no arena yet: upstream fails allocating its views (Q_ERR_ARENA_OOM)
    assert Q.lib.llama_build_graph(C.byref(ctx), C.byref(model)) == -8
    assert model.config.dim == 256 and model.config.n_kv_heads == 2
    assert abs(model.config.rms_norm_eps - 1e-5) < 1e-12
    Q.lib.q_free_memory(C.byref(ctx))
    assert ctx.weights_mmap is None


def test_forward_validation_without_gpu():
    ctx, model = Q.q_context(), Q.q_llama_model()
    model.config.max_seq_len = 16
    model.config.vocab_size = 10
    logits = np.zeros(10, np.float32)
    tok = np.array([1], np.uint32)
    f = Q.lib.llama_forward
    assert f(None, C.byref(ctx), Q.ptr(tok), 1, 0, Q.ptr(logits)) == -10
    assert f(C.byref(model), C.byref(ctx), Q.ptr(tok), 0, 0, Q.ptr(logits)) == -15
    assert f(C.byref(model), C.byref(ctx), Q.ptr(tok), 17, 0, Q.ptr(logits)) == -15
    assert f(C.byref(model), C.byref(ctx), Q.ptr(tok), 1, 16, Q.ptr(logits)) == -10
    assert f(C.byref(model), C.byref(ctx), Q.ptr(tok), 1, 0, Q.ptr(logits)) == -10  # no arena/kv


def test_sample_token_greedy_first_max():
    lg = np.array([0.5, 2.0, -1.0, 2.0], np.float32)
    out = C.c_uint32(99)
    assert Q.lib.q_sample_token(Q.ptr(lg), 4, 0.0, 0, 0.0, C.byref(out), None) == 0
    assert out.value == 1  # upstream main.c:870-881: strict '>' keeps the first
    assert Q.lib.q_sample_token(Q.ptr(lg), 0, 0.0, 0, 0.0, C.byref(out), None) == -15
    assert Q.lib.q_sample_token(Q.ptr(lg), 4, -1.0, 0, 0.0, C.byref(out), None) == -10


def test_generators_are_counter_based():
    a = np.zeros(100000, np.float32)
    b = np.zeros(60000, np.float32)
    Q.lib.q_b200_fill_normal(Q.ptr(a), a.size, 5, 9, 0, 0.0, 1.0, 4)
    Q.lib.q_b200_fill_normal(Q.ptr(b), b.size, 5, 9, 40000, 0.0, 1.0, 1)
    assert np.array_equal(a[40000:], b)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02
    q = np.zeros(64 * 20, np.uint8)
    Q.lib.q_b200_fill_q4(Q.ptr(q), 64, 1, 2, 0, 0.001, 0.01, 1)
    blocks = q.reshape(64, 20)
    sc = blocks[:, 16:].copy().view(np.float32).ravel()
    assert (sc >= 0.001).all() and (sc < 0.01).all()
    nib = np.concatenate([blocks[:, :16] & 15, blocks[:, :16] >> 4])
    assert nib.min() == 0 and nib.max() == 15


def test_model_file_size_matches_layout(tiny_path):
    cfg = Q.config(**Q.TINY)
    assert Q.lib.q_b200_model_file_size(C.byref(cfg)) == Path(tiny_path).stat().st_size
    bad = Q.config(259, 250, 768, 2, 8, 2, 512)  # dim % 32 != 0
    assert Q.lib.q_b200_model_file_size(C.byref(bad)) == 0


def test_kernel_entry_validation_without_gpu():
    x = Q.aligned_empty(16)
    raw = Q.aligned_empty(17)
    mis = raw[1:]
    out = Q.aligned_empty(16)
    assert Q.lib.q_rmsnorm_f32_avx2(None, Q.ptr(x), Q.ptr(out), 16, 1e-5) == -10
    assert Q.lib.q_rmsnorm_f32_avx2(Q.ptr(mis), Q.ptr(x), Q.ptr(out), 16, 1e-5) == -13
    assert Q.lib.q_rmsnorm_f32_avx2(Q.ptr(x), Q.ptr(x), Q.ptr(out), 12, 1e-5) == -15
    assert Q.lib.q_softmax_f32_avx2(Q.ptr(x), Q.ptr(out), 0) == -15
    t = Q.q_tensor()
    t.ne[:] = [4, 33, 1, 1]
    t.type = Q.Q_Q4_0
    assert Q.lib.q_gemv_q4_f32_avx2(C.byref(t), Q.ptr(x), Q.ptr(out)) == -15
    assert Q.lib.q_gemv_q4_f32_avx2(C.byref(t), Q.ptr(x), Q.ptr(x)) == -11
