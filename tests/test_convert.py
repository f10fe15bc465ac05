"""The checkpoint converter (qorus_b200.convert) on CPU: a small Hugging Face
style Llama checkpoint written here (safetensors, bf16 and f32 tensors) is
converted to .qorus v2 and read back through the oracle's loader."""
import json
import struct

import numpy as np

import oracle as O
from qorus_b200 import convert as CV


def write_safetensors(path, tensors):
    header, blobs, off = {}, [], 0
    for name, (arr, dt) in tensors.items():
        if dt == "BF16":
            raw = (np.ascontiguousarray(arr, np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
        else:
            raw = np.ascontiguousarray(arr, np.float32).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def bf16(a):
    return ((np.asarray(a, np.float32).view(np.uint32) >> 16) << 16).view(np.float32)


def make_checkpoint(d, V=259, D=128, H=256, L=2, nh=4, nkv=2):
    rng = np.random.default_rng(0)
    cfg = {"hidden_size": D, "intermediate_size": H, "num_hidden_layers": L, "num_attention_heads": nh,
           "num_key_value_heads": nkv, "vocab_size": V, "max_position_embeddings": 512,
           "rope_theta": 500000.0, "rms_norm_eps": 1e-5}
    (d / "config.json").write_text(json.dumps(cfg))
    hd = D // nh
    t = {"model.embed_tokens.weight": (rng.normal(0, 0.02, (V, D)), "F32"),
         "model.norm.weight": (1 + rng.normal(0, 0.02, D), "F32"),
         "lm_head.weight": (rng.normal(0, 0.02, (V, D)), "BF16")}
    for i in range(L):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = (1 + rng.normal(0, 0.02, D), "F32")
        t[p + "post_attention_layernorm.weight"] = (1 + rng.normal(0, 0.02, D), "F32")
        for n, shp in (("self_attn.q_proj", (D, D)), ("self_attn.k_proj", (nkv * hd, D)),
                       ("self_attn.v_proj", (nkv * hd, D)), ("self_attn.o_proj", (D, D)),
                       ("mlp.gate_proj", (H, D)), ("mlp.up_proj", (H, D)), ("mlp.down_proj", (D, H))):
            t[p + n + ".weight"] = (rng.normal(0, 0.05, shp), "BF16")
    write_safetensors(d / "model.safetensors", t)
    return cfg, {k: (bf16(v) if dt == "BF16" else np.asarray(v, np.float32)) for k, (v, dt) in t.items()}


def test_quantize_q4_0_roundtrip():
    rng = np.random.default_rng(1)
    w = rng.normal(0, 1, (64, 96)).astype(np.float32)
    w[3, 0:32] = 0.0  # an all-zero block
    data = CV.quantize_q4_0(w)
    assert len(data) == 64 * 3 * 20
    back = CV.dequantize_q4_0(data, 64, 96)
    blocks, bb = w.reshape(-1, 32), back.reshape(-1, 32)
    d = np.abs(blocks).max(axis=1) / 8
    # the 16 levels -8..7 are asymmetric: |d| / 2 on the extreme's side, up to |d| next to the
    # opposite extreme (whose level 8 does not exist)
    assert (np.abs(bb - blocks) <= d[:, None] * (1 + 1e-5) + 1e-7).all()
    i = np.argmax(np.abs(blocks), axis=1)
    r = np.arange(blocks.shape[0])
    np.testing.assert_allclose(bb[r, i], blocks[r, i], rtol=1e-6, atol=0)  # the extreme is exact
    assert (bb[3 * 3] == 0).all()  # row 3, first block
    # byte b holds elements 2b (low nibble) and 2b + 1 (high nibble), as upstream's block decode
    blk = np.frombuffer(data[:20], np.uint8).copy()
    out = np.zeros(32, np.float32)
    O.orc.orc_dequantize_block(O.p(blk), O.p(out))
    np.testing.assert_array_equal(out, back.reshape(-1)[:32])


def test_convert_checkpoint_reads_back(tmp_path):
    cfg, t = make_checkpoint(tmp_path)
    out = tmp_path / "m.qorus"
    info = CV.convert(tmp_path, out, max_seq=256)
    assert info["max_seq"] == 256 and info["rms_norm_eps"] == 1e-5
    size = O.gen.q_b200_model_file_size(__import__("ctypes").byref(
        O.config(cfg["vocab_size"], cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"],
                 cfg["num_attention_heads"], cfg["num_key_value_heads"], 256)))
    assert out.stat().st_size == size
    raw = out.read_bytes()
    hdr = struct.unpack("<9If f5I", raw[:64])
    assert hdr[0] == CV.Q_MAGIC and hdr[1] == 2 and hdr[2:9] == (259, 128, 256, 2, 4, 2, 256)
    V, D = 259, 128
    emb = np.frombuffer(raw[64:64 + V * D * 4], np.float32).reshape(V, D)
    np.testing.assert_array_equal(emb, t["model.embed_tokens.weight"])
    # layer 0's wq: rows re-paired for interleaved RoPE, then Q4_0
    off = 64 + CV._align(V * D * 4) + CV._align(D * 4) + CV._align(V * D * 4) + CV._align(D * 4)
    wq = CV.dequantize_q4_0(raw[off:off + D * (D // 32) * 20], D, D)
    ref = CV.rope_interleave(t["model.layers.0.self_attn.q_proj.weight"], 4)
    assert np.abs(wq - ref).max() <= np.abs(ref).max() / 8 + 1e-6
    hd = D // 4
    assert np.abs(wq[1] - t["model.layers.0.self_attn.q_proj.weight"][hd // 2]).max() < 0.01  # row 1 <- i + hd/2
    # the oracle's loader opens it and a prompt runs through it
    m = O.OracleModel(str(out), threads=2)
    lg = m.forward(np.array([5, 17, 200], np.uint32), 0)
    assert np.isfinite(lg).all() and lg.size == V
    m.close()


@__import__("pytest").mark.gpu
def test_converted_checkpoint_on_the_device(tmp_path):
    """The converted file through the upstream API on the B200 (prompt path
    and decode steps) against the oracle on the same file."""
    import qorus_b200 as Q
    make_checkpoint(tmp_path)
    out = tmp_path / "m.qorus"
    CV.convert(tmp_path, out, max_seq=256)
    dev, orc = Q.Model(str(out)), O.OracleModel(str(out))
    toks = np.array([1, 5, 17, 200, 33, 90, 7, 258], np.uint32)
    a = dev.forward(toks, 0).copy()
    b = orc.forward(toks, 0)
    assert np.abs(a - b).max() <= 1e-2 and int(np.argmax(a)) == int(np.argmax(b))
    tok = int(np.argmax(b))
    for i in range(8):
        a = dev.forward(np.array([tok], np.uint32), len(toks) + i).copy()
        b = orc.forward(np.array([tok], np.uint32), len(toks) + i)
        assert np.abs(a - b).max() <= 1e-2 and int(np.argmax(a)) == int(np.argmax(b))
        tok = int(np.argmax(b))
    dev.close()
    orc.close()
