"""Convert a Hugging Face Llama checkpoint (safetensors) into a .qorus v2 file.

    python -m qorus_b200.convert <checkpoint_dir> <out.qorus> [--max-seq N]

Upstream's converter (tools/convert_llama.py:22-40, 116-239) writes version-1
headers and FP32 payloads where its loader expects Q4_0, so no real model
reaches upstream's graph through it.  This one writes what the loader
(src/models/model.c:294-673, this library's llama_build_graph) reads:

* a 64-byte version-2 header with rms_norm_eps (include/qorus_types.h);
* token_embd [vocab][dim] f32, output_norm [dim] f32, output [vocab][dim] f32
  (the embedding again when the checkpoint ties them), then per layer
  attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up, w_down, every tensor
  padded to 64 bytes (model.c:355-619);
* linear weights as Q4_0 blocks in [out][in] order: 32 weights per block,
  byte b holding elements 2b (low nibble) and 2b + 1 (high nibble), then the
  fp32 scale (include/qorus_types.h: q_block_q4_0).

Quantization of a block x[0..31]: d = m / -8 with m the element of largest
magnitude (sign kept), q = clamp(floor(x / d + 8.5), 0, 15), so x = (q - 8) d
exactly at the extreme and within |d| / 2 elsewhere on its side (within |d|
next to the opposite extreme, as level 8 does not exist): the usual 4-bit
block scheme of this format.

Query and key rows are reordered per head from the rotate-half pairing of
Hugging Face checkpoints (i, i + hd/2) into the interleaved pairs (2i, 2i + 1)
that upstream's RoPE (src/ops/avx2/rope.c) rotates.

Reading needs only numpy: safetensors is an 8-byte header length, a JSON
header and raw little-endian arrays (f32, f16 or bf16 here).
"""
from __future__ import annotations

import argparse
import json
import struct
from pathlib import Path

import numpy as np

Q_MAGIC = 0x514F5231
Q_ALIGN = 64
Q_HEADER_SIZE = 64


def _align(n: int) -> int:
    return (n + Q_ALIGN - 1) // Q_ALIGN * Q_ALIGN


def read_safetensors(path: Path) -> dict:
    """name -> float32 array, for every tensor of one .safetensors file."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    n = struct.unpack("<Q", bytes(raw[:8]))[0]
    header = json.loads(bytes(raw[8:8 + n]))
    base = 8 + n
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        lo, hi = meta["data_offsets"]
        buf = raw[base + lo: base + hi]
        dt = meta["dtype"]
        if dt == "F32":
            a = np.frombuffer(buf, np.float32)
        elif dt == "F16":
            a = np.frombuffer(buf, np.float16).astype(np.float32)
        elif dt == "BF16":
            a = (np.frombuffer(buf, np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError(f"{name}: dtype {dt} not supported")
        out[name] = a.reshape(meta["shape"])
    return out


def quantize_q4_0(w: np.ndarray) -> bytes:
    """[rows][cols] float -> Q4_0 blocks (cols % 32 == 0), row-major."""
    rows, cols = w.shape
    if cols % 32:
        raise ValueError("Q4_0 rows need a multiple of 32 columns")
    x = np.ascontiguousarray(w, np.float32).reshape(-1, 32)
    idx = np.argmax(np.abs(x), axis=1)
    m = x[np.arange(x.shape[0]), idx]
    d = (m / -8.0).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.floor(x * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    nib = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)  # byte b: elements 2b, 2b + 1
    blocks = np.empty((x.shape[0], 20), np.uint8)
    blocks[:, :16] = nib
    blocks[:, 16:] = d.view(np.uint8).reshape(-1, 4)
    return blocks.tobytes()


def dequantize_q4_0(data: bytes, rows: int, cols: int) -> np.ndarray:
    """Inverse of quantize_q4_0 (upstream's block decode, model.c / dequantize.c)."""
    b = np.frombuffer(data, np.uint8).reshape(-1, 20)
    d = b[:, 16:].copy().view(np.float32)[:, 0]
    q = np.empty((b.shape[0], 32), np.float32)
    q[:, 0::2] = b[:, :16] & 15
    q[:, 1::2] = b[:, :16] >> 4
    return ((q - 8.0) * d[:, None]).reshape(rows, cols)


def rope_interleave(w: np.ndarray, n_heads: int) -> np.ndarray:
    """Rows of each head from (i, i + hd/2) pairing to (2i, 2i + 1)."""
    rows, cols = w.shape
    hd = rows // n_heads
    return w.reshape(n_heads, 2, hd // 2, cols).swapaxes(1, 2).reshape(rows, cols)


def convert(ckpt: Path, out: Path, max_seq: int | None = None) -> dict:
    cfg = json.loads((ckpt / "config.json").read_text())
    t = {}
    for f in sorted(ckpt.glob("*.safetensors")):
        t.update(read_safetensors(f))
    D = int(cfg["hidden_size"])
    H = int(cfg["intermediate_size"])
    L = int(cfg["num_hidden_layers"])
    nh = int(cfg["num_attention_heads"])
    nkv = int(cfg.get("num_key_value_heads", nh))
    V = int(cfg["vocab_size"])
    seq = int(max_seq or cfg.get("max_position_embeddings", 8192))
    theta = float(cfg.get("rope_theta", 10000.0))
    eps = float(cfg.get("rms_norm_eps", 1e-5))
    if D % 32 or H % 32 or D % nh or nh % nkv:
        raise ValueError("dim and FFN width must be multiples of 32, heads must divide dim")
    emb = t["model.embed_tokens.weight"]
    head = t.get("lm_head.weight", emb)
    pieces = []

    def f32(a):
        pieces.append(np.ascontiguousarray(a, np.float32).tobytes())

    def q4(a):
        pieces.append(quantize_q4_0(a))

    f32(emb)
    f32(t["model.norm.weight"])
    f32(head)
    for i in range(L):
        p = f"model.layers.{i}."
        f32(t[p + "input_layernorm.weight"])
        q4(rope_interleave(t[p + "self_attn.q_proj.weight"], nh))
        q4(rope_interleave(t[p + "self_attn.k_proj.weight"], nkv))
        q4(t[p + "self_attn.v_proj.weight"])
        q4(t[p + "self_attn.o_proj.weight"])
        f32(t[p + "post_attention_layernorm.weight"])
        q4(t[p + "mlp.gate_proj.weight"])
        q4(t[p + "mlp.up_proj.weight"])
        q4(t[p + "mlp.down_proj.weight"])
    header = struct.pack("<9If f5I", Q_MAGIC, 2, V, D, H, L, nh, nkv, seq, theta, eps, *([0] * 5))
    assert len(header) == Q_HEADER_SIZE
    with open(out, "wb") as fh:
        fh.write(header)
        for b in pieces:
            fh.write(b)
            fh.write(b"\0" * (_align(len(b)) - len(b)))
    return {"vocab": V, "dim": D, "hidden": H, "layers": L, "heads": nh, "kv_heads": nkv,
            "max_seq": seq, "rope_theta": theta, "rms_norm_eps": eps}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("checkpoint", type=Path)
    ap.add_argument("out", type=Path)
    ap.add_argument("--max-seq", type=int, default=None)
    a = ap.parse_args()
    print(json.dumps(convert(a.checkpoint, a.out, a.max_seq)))


if __name__ == "__main__":
    main()
