"""Test infrastructure only: a pure-Python restatement of upstream's byte-level
BPE tokenizer (src/tokenizer/bpe.c), the checker for the library's
q_tokenizer_* entry points.  Nothing shipped imports this module.

Pinned by tests/test_tokenizer.py against upstream's own known answers
(tests/test_bpe_tokenizer.c cases 1-6) and, where oracle/_ref is built,
against upstream's q_tokenizer_* on random tokenizers and texts.
"""
from __future__ import annotations

import struct

MAGIC = 0x51544B52        # 'QTKR' (bpe.c:25)
VERSION = 1
MAX_TEXT_BYTES = 1 << 20  # bpe.c:58
DELETED = 0xFFFFFFFF      # soft-deleted slot (bpe.c:62)

Q_OK, Q_ERR_FILE_OPEN, Q_ERR_INVALID_MAGIC, Q_ERR_ALLOC_FAILED = 0, -2, -6, -7
Q_ERR_ARENA_OOM, Q_ERR_INVALID_ARG, Q_ERR_INVALID_SIZE = -8, -10, -15


def write_file(path, vocab: list[bytes], merges: list[tuple[int, int, int]],
               bos: int, eos: int, pad: int, magic=MAGIC, version=VERSION) -> None:
    """The 'QTKR' v1 layout read by q_tokenizer_load (bpe.c:279-487)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<8I", magic, version, len(vocab), len(merges), bos, eos, pad, 0))
        for s in vocab:
            f.write(struct.pack("B", len(s)) + s)
        for m in merges:
            f.write(struct.pack("<3I", *m))


class Tokenizer:
    def __init__(self, vocab: list[bytes], merges: list[tuple[int, int, int]], bos: int, eos: int, pad: int):
        self.vocab, self.merges = vocab, merges
        self.bos, self.eos, self.pad = bos, eos, pad
        # bpe.c:106-176: chains are head-inserted and a lookup takes the first
        # key match, so of several rules with the same key (first << 16) | second
        # the last one's merged id is returned; the key is not unique once an
        # id reaches 65536.
        self.table = {}
        for a, b, m in merges:
            self.table[(a << 16) | b] = m

    def encode(self, text: bytes, max_tokens: int, add_bos: bool, add_eos: bool):
        """(error code, ids) — bpe.c:697-799."""
        if max_tokens == 0:
            return Q_ERR_INVALID_SIZE, []
        if not text:
            out = ([self.bos] if add_bos else []) + ([self.eos] if add_eos else [])
            return (Q_ERR_ARENA_OOM, []) if len(out) > max_tokens else (Q_OK, out)
        if len(text) > MAX_TEXT_BYTES:
            return Q_ERR_ARENA_OOM, []
        cap = max(len(text), max_tokens)
        V = len(self.vocab)
        ids = [b if b < V else self.pad for b in text]          # bpe.c:518-546
        n = len(ids)
        if self.merges and n >= 2:                               # bpe.c:553-641
            deleted, compact_at = 0, n // 2
            changed = True
            while changed:
                changed = False
                for a, b, m in self.merges:
                    merged = self.table.get((a << 16) | b, m)
                    j = 0
                    while j < n:
                        if ids[j] == DELETED:
                            j += 1
                            continue
                        nx = j + 1
                        while nx < n and ids[nx] == DELETED:
                            nx += 1
                        if nx >= n:
                            break
                        if ids[j] == a and ids[nx] == b:
                            ids[j], ids[nx] = merged, DELETED
                            deleted += 1
                            changed = True
                        j += 1
                if deleted > compact_at:
                    ids = [t for t in ids[:n] if t != DELETED]
                    n, deleted = len(ids), 0
            ids = [t for t in ids[:n] if t != DELETED]
        out = ([self.bos] if add_bos else []) + ids + ([self.eos] if add_eos else [])
        if len(out) > cap or len(out) > max_tokens:             # bpe.c:650-657, 783
            return Q_ERR_ARENA_OOM, []
        return Q_OK, out

    def decode(self, ids, buf_size: int):
        """(error code, bytes) — bpe.c:803-857; truncated output on overflow."""
        if buf_size == 0:
            return Q_ERR_INVALID_SIZE, b""
        out = b""
        for t in ids:
            if t in (self.bos, self.eos, self.pad) or t >= len(self.vocab):
                continue
            s = self.vocab[t].split(b"\0", 1)[0]  # upstream measures with strlen
            if len(out) + len(s) >= buf_size - 1:
                return Q_ERR_ARENA_OOM, out
            out += s
        return Q_OK, out
