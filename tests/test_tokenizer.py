"""q_tokenizer_* (host code in libqorus_b200.so) against the Python
restatement of upstream's BPE tokenizer (oracle/bpe.py), which is itself
pinned to upstream's known answers (tests/test_bpe_tokenizer.c) and, where
oracle/_ref is built, to upstream's own q_tokenizer_* on random cases.
No GPU: the tokenizer never touches the device."""
import ctypes as C
import random

import pytest

import bpe as B
import oracle as O
import qorus_b200 as Q


class Tok(C.Structure):
    """q_tokenizer (include/qorus_types.h)."""
    _fields_ = [("vocab", C.c_void_p), ("vocab_size", C.c_uint32), ("merges", C.c_void_p),
                ("num_merges", C.c_uint32), ("merge_hash_table", C.c_void_p), ("bos", C.c_uint32),
                ("eos", C.c_uint32), ("pad", C.c_uint32), ("initialized", C.c_bool)]


IMPLS = [("b200", Q.lib)] + ([("upstream", O.ref)] if O.ref is not None else [])


def _bind(lib):
    lib.q_tokenizer_load.restype, lib.q_tokenizer_load.argtypes = C.c_int, [C.c_void_p, C.c_char_p]
    lib.q_tokenizer_encode.restype = C.c_int
    lib.q_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_void_p, C.c_uint32,
                                       C.c_bool, C.c_bool]
    lib.q_tokenizer_decode.restype = C.c_int
    lib.q_tokenizer_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_size_t]
    lib.q_tokenizer_free.restype, lib.q_tokenizer_free.argtypes = None, [C.c_void_p]
    return lib


class Loaded:
    def __init__(self, lib, path):
        self.lib, self.tok = _bind(lib), Tok()
        self.rc = lib.q_tokenizer_load(C.byref(self.tok), str(path).encode())

    def encode(self, text: bytes, max_tokens: int, bos=False, eos=False):
        out = (C.c_uint32 * max(max_tokens, 1))()
        n = C.c_uint32(0xDEAD)
        rc = self.lib.q_tokenizer_encode(C.byref(self.tok), text, out, C.byref(n), max_tokens, bos, eos)
        return rc, (list(out[: n.value]) if rc == 0 else [])

    def decode(self, ids, buf_size: int):
        arr = (C.c_uint32 * max(len(ids), 1))(*ids)
        buf = C.create_string_buffer(max(buf_size, 1))
        rc = self.lib.q_tokenizer_decode(C.byref(self.tok), arr, len(ids), buf, buf_size)
        return rc, buf.value

    def free(self):
        self.lib.q_tokenizer_free(C.byref(self.tok))


def byte_vocab(extra: list[bytes]) -> list[bytes]:
    return [bytes([i]) for i in range(256)] + extra


def make(tmp_path, name, vocab, merges, bos, eos, pad, **kw):
    p = tmp_path / name
    B.write_file(p, vocab, merges, bos, eos, pad, **kw)
    return p


# ---- upstream's known answers (tests/test_bpe_tokenizer.c) -------------------

@pytest.mark.parametrize("name,lib", IMPLS)
def test_upstream_known_answers(tmp_path, name, lib):
    vocab = byte_vocab([b"<s>", b"</s>", b"<pad>"]) + [b"x%d" % i for i in range(259, 600)]
    vocab[500], vocab[501] = b"ll", b"el"
    plain = make(tmp_path, "a.bin", vocab, [], 256, 257, 258)
    one = make(tmp_path, "b.bin", vocab, [(108, 108, 500)], 256, 257, 258)
    two = make(tmp_path, "c.bin", vocab, [(108, 108, 500), (101, 108, 501)], 256, 257, 258)
    cases = [  # (file, text, max_tokens, bos, eos, rc, ids) — test_bpe_tokenizer.c cases 1-6
        (plain, b"Hello", 256, False, False, 0, [72, 101, 108, 108, 111]),
        (one, b"hello", 256, False, False, 0, [104, 101, 500, 111]),
        (plain, b"Hi", 256, True, True, 0, [256, 72, 105, 257]),
        (plain, b"This is a long text", 5, False, False, B.Q_ERR_ARENA_OOM, []),
        (plain, b"", 256, False, False, 0, []),
        (plain, b"", 256, True, True, 0, [256, 257]),
        (two, b"hello", 256, False, False, 0, [104, 101, 500, 111]),
    ]
    for path, text, mx, bos, eos, rc, ids in cases:
        t = Loaded(lib, path)
        assert t.rc == 0
        assert t.encode(text, mx, bos, eos) == (rc, ids), (name, text)
        ref = B.Tokenizer(vocab, [] if path == plain else ([(108, 108, 500)] if path == one else
                                                            [(108, 108, 500), (101, 108, 501)]), 256, 257, 258)
        assert ref.encode(text, mx, bos, eos) == (rc, ids)
        t.free()
        assert t.tok.vocab is None and not t.tok.initialized


# ---- file validation, in upstream's order ------------------------------------

@pytest.mark.parametrize("name,lib", IMPLS)
def test_load_errors(tmp_path, name, lib):
    vocab = byte_vocab([b"<s>", b"</s>", b"<pad>"])
    ok = make(tmp_path, "ok.bin", vocab, [(1, 2, 258)], 256, 257, 258)
    raw = ok.read_bytes()
    cases = {
        "missing": (tmp_path / "nope.bin", B.Q_ERR_FILE_OPEN),
        "magic": (make(tmp_path, "m.bin", vocab, [], 256, 257, 258, magic=0x1234), B.Q_ERR_INVALID_MAGIC),
        "version": (make(tmp_path, "v.bin", vocab, [], 256, 257, 258, version=2), B.Q_ERR_INVALID_ARG),
        "empty_vocab": (make(tmp_path, "e.bin", [], [], 0, 0, 0), B.Q_ERR_INVALID_SIZE),
        "merge_range": (make(tmp_path, "r.bin", vocab, [(1, 2, 259)], 256, 257, 258), B.Q_ERR_INVALID_ARG),
        "truncated_vocab": (None, B.Q_ERR_FILE_OPEN),
        "truncated_merges": (None, B.Q_ERR_FILE_OPEN),
        "short_bad_magic": (None, B.Q_ERR_INVALID_MAGIC),
        "zero_length_token": (None, B.Q_ERR_INVALID_SIZE),
    }
    (tmp_path / "tv.bin").write_bytes(raw[:32 + 100])
    cases["truncated_vocab"] = (tmp_path / "tv.bin", B.Q_ERR_FILE_OPEN)
    (tmp_path / "tm.bin").write_bytes(raw[:-4])
    cases["truncated_merges"] = (tmp_path / "tm.bin", B.Q_ERR_FILE_OPEN)
    (tmp_path / "sm.bin").write_bytes(b"XXXX")
    cases["short_bad_magic"] = (tmp_path / "sm.bin", B.Q_ERR_INVALID_MAGIC)
    z = bytearray(raw)
    z[32 + 2 * 5] = 0  # token 5's length byte
    (tmp_path / "z.bin").write_bytes(bytes(z))
    cases["zero_length_token"] = (tmp_path / "z.bin", B.Q_ERR_INVALID_SIZE)
    for what, (path, rc) in cases.items():
        t = Loaded(lib, path)
        assert t.rc == rc, (name, what, t.rc)
        assert not t.tok.initialized
        if name == "b200":  # upstream leaves a freed pointer behind on some error paths
            assert t.tok.vocab is None
    t = Loaded(lib, ok)
    assert t.rc == 0 and t.tok.vocab_size == 259 and t.tok.num_merges == 1 and t.tok.initialized
    assert (t.tok.bos, t.tok.eos, t.tok.pad) == (256, 257, 258)
    t.free()


@pytest.mark.parametrize("name,lib", IMPLS)
def test_call_errors_and_decode_limits(tmp_path, name, lib):
    vocab = byte_vocab([b"<s>", b"</s>", b"<pad>", b"hello world"])
    t = Loaded(lib, make(tmp_path, "t.bin", vocab, [], 256, 257, 258))
    assert t.rc == 0
    assert t.encode(b"abc", 0) == (B.Q_ERR_INVALID_SIZE, [])
    assert t.encode(b"", 1, True, True) == (B.Q_ERR_ARENA_OOM, [])
    assert t.encode(b"abc", 4, True, True) == (B.Q_ERR_ARENA_OOM, [])
    assert t.encode(b"abc", 5, True, True) == (0, [256, 97, 98, 99, 257])
    assert t.encode(b"a" * ((1 << 20) + 1), 8) == (B.Q_ERR_ARENA_OOM, [])
    ref = B.Tokenizer(vocab, [], 256, 257, 258)
    ids = [256, 104, 259, 9999, 258, 0, 105, 257]
    for size in (0, 1, 2, 3, 13, 14, 15, 64):
        got = t.decode(ids, size)
        assert got == ref.decode(ids, size), (name, size, got)
    assert t.decode(ids, 64) == (0, b"hhello worldi")
    assert t.decode(ids, 14) == (B.Q_ERR_ARENA_OOM, b"hhello world")
    assert t.decode(ids, 13) == (B.Q_ERR_ARENA_OOM, b"h")
    t.free()
    # a tokenizer that was never loaded
    u = Loaded.__new__(Loaded)
    u.lib, u.tok = _bind(lib), Tok()
    assert u.encode(b"a", 4)[0] == B.Q_ERR_INVALID_ARG
    assert u.decode([1], 4)[0] == B.Q_ERR_INVALID_ARG


# ---- random tokenizers: library == restatement (== upstream) -----------------

def random_tokenizer(rng: random.Random, V: int, n_merges: int, wide: bool):
    vocab = byte_vocab([]) + [bytes(rng.randrange(1, 256) for _ in range(rng.randrange(1, 6)))
                              for _ in range(V - 256)]
    bos, eos, pad = V - 3, V - 2, V - 1
    common = [ord(c) for c in "aeiou lnrst"]
    merges = []
    for _ in range(n_merges):
        a = rng.choice(common) if rng.random() < 0.5 else rng.randrange(V)
        b = rng.choice(common) if rng.random() < 0.5 else rng.randrange(V)
        merges.append((a, b, rng.randrange(256, V)))
    if wide:  # pairs whose (first << 16) | second keys coincide: (0, 65538) and (1, 65538)
        merges += [(1, 65538, 300), (0, 65538, 301), (ord("a"), ord("b"), 65538), (0, 65538, 302)]
    return vocab, merges, bos, eos, pad


@pytest.mark.parametrize("seed,V,n_merges,wide", [(1, 300, 40, False), (2, 1000, 400, False),
                                                   (3, 70000, 200, True), (4, 260, 0, False)])
def test_random_against_restatement_and_upstream(tmp_path, seed, V, n_merges, wide):
    rng = random.Random(seed)
    vocab, merges, bos, eos, pad = random_tokenizer(rng, V, n_merges, wide)
    path = make(tmp_path, "r.bin", vocab, merges, bos, eos, pad)
    ref = B.Tokenizer(vocab, merges, bos, eos, pad)
    libs = [Loaded(lib, path) for _, lib in IMPLS]
    assert all(t.rc == 0 for t in libs)
    alphabet = b"aeiou lnrstab\x00\xff" if V > 256 else bytes(range(1, 256))
    for k in range(60):
        n = rng.choice([1, 2, 3, 7, 40, 300])
        text = bytes(rng.choice(alphabet) for _ in range(n)).replace(b"\0", b"a")
        mx = rng.choice([n + 2, n, max(1, n // 2), 512])
        bos_, eos_ = rng.random() < 0.5, rng.random() < 0.5
        want = ref.encode(text, mx, bos_, eos_)
        for t in libs:
            assert t.encode(text, mx, bos_, eos_) == want, (seed, k, text, mx)
        if want[0] == 0:
            size = rng.choice([1, 5, 64, 4096])
            dw = ref.decode(want[1], size)
            for t in libs:
                assert t.decode(want[1], size) == dw
    for t in libs:
        t.free()


@pytest.mark.parametrize("name,lib", IMPLS)
def test_pad_for_bytes_outside_a_small_vocabulary(tmp_path, name, lib):
    """Bytes >= vocab_size become PAD before merging (bpe.c:518-546)."""
    vocab = [bytes([i + 1]) for i in range(100)]
    merges = [(96, 97, 5), (99, 99, 7)]
    path = make(tmp_path, "s.bin", vocab, merges, 0, 1, 99)
    ref = B.Tokenizer(vocab, merges, 0, 1, 99)
    t = Loaded(lib, path)
    for text in (b"\x60\x61zz", b"\xc3\xa9t\x60\x61", b"\x60\x61\x60\x61\x60", b"\xff\xff\xff"):
        want = ref.encode(text, 64, False, False)
        assert t.encode(text, 64) == want
    assert ref.encode(b"\xff\xff\xff", 64, False, False) == (0, [7, 99])
    t.free()
