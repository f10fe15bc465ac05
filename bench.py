#!/usr/bin/env python3
"""Benchmark: Llama-3-8B-shaped Q4_0 batch-1 greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: 32 layers, dim 4096, 32 query / 8 KV
heads (head_dim 128), FFN 14336, vocab 128256, random-init Q4_0 weights
(FP32 embedding / LM head), KV cache pre-filled with 2048 positions of
N(0,1), then greedy decode.  A step is one decoded token.  Synthetic data
from the library's counter-based generators; the per-token stream (7 GB of
weights + LM head + KV) is ~55x the 126 MB L2, so no L2 flush is needed.

`value` times K device-resident decode steps (the captured per-token CUDA
graph replayed, the argmax fed back on the device) with CUDA events on the
library's stream.  `e2e` times K calls of the upstream entry point
llama_forward (host token in, host logits out, so each step copies the token
and step scalars H2D and 513 KB of logits D2H).  With --gpus N each rank
is one rank of a tensor-parallel decode of the same sequence (heads, FFN
rows and vocab rows split over the ranks, NCCL all-reduce after wo and down;
strong scaling: value is the sequence's tok/s).

--impl reference times the upstream CPU implementation of the same path:
the upstream AVX2 kernels (compiled from the upstream sources into
oracle/_ref) composed into the same graph, all host threads.  That process
never loads the CUDA library: its model file and KV image come from
oracle/libqgen.so (the same generator source, built on its own).

The line also carries the GEMV sweep of BASELINE configs[1] (`sweep`: the
four Llama-3-8B projection shapes, GB/s against the measured HBM peak,
upstream's q_gemv_q4_f32_avx2 on one host thread beside each), and
`cpu_baseline` is upstream's decode on ONE host thread (the reference has no
threading), with the all-threads figure under cpu_baseline.threaded.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "project-ia_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "Llama-3-8B Q4_0 decode tok/s"
CFG8B = dict(vocab=128256, dim=4096, hidden=14336, layers=32, heads=32, kv_heads=8)
PREFILL = 2048
SEED = 0
# the workload, printed identically by both arms
CONFIG = {"workload": "llama3-8b-q4_0 decode, batch 1, kv prefill 2048 (BASELINE configs[2])",
          "layers": 32, "dim": 4096, "heads": "32/8", "ffn": 14336, "vocab": 128256,
          "global_batch": 1, "prefill": PREFILL,
          "l2": "inputs larger than L2 (7 GB streamed per token)"}
SWEEP = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


def q4_linear_bytes(c) -> int:
    D, H = c["dim"], c["hidden"]
    kvd = c["kv_heads"] * (D // c["heads"])
    per_layer = (D * D * 2 + kvd * D * 2 + H * D * 3) * 5 // 8  # 0.625 B / weight
    return per_layer * c["layers"]


def token_bytes(c, ctx_len: int) -> int:
    """Algorithmic HBM bytes of one decode token at context length ctx_len."""
    D = c["dim"]
    hd = D // c["heads"]
    lm_head = c["vocab"] * D * 4
    kv = c["layers"] * c["kv_heads"] * ctx_len * hd * 2 * 4
    small = D * 4 * (1 + 2 * c["layers"] + 1)  # embedding row, norm gains, final norm
    return q4_linear_bytes(c) + lm_head + kv + small


def model_path(max_seq: int) -> str:
    d = Path(os.environ.get("QORUS_TMPDIR", "/dev/shm" if Path("/dev/shm").exists() else "/tmp"))
    return str(d / f"qorus_llama3_8b_q4_{max_seq}_s{SEED}.qorus")


def ensure_model(gen, cfg, max_seq: int, rank: int, barrier) -> str:
    """Write the seed-0 model file once.  `gen` is a library exporting the
    synthetic-input generators: the product library in our arm, the
    CPU-only oracle/libqgen.so (same C source) in the reference arm."""
    path = model_path(max_seq)
    size = int(gen.q_b200_model_file_size(C.byref(cfg)))
    if rank == 0 and not (Path(path).exists() and Path(path).stat().st_size == size):
        rc = gen.q_b200_write_model_file(path.encode(), C.byref(cfg), SEED, 0)
        if rc:
            raise RuntimeError(f"q_b200_write_model_file: {rc}")
    barrier()
    return path


def kv_image(gen, cfg) -> np.ndarray:
    hd = cfg.dim // cfg.n_heads
    kv = np.zeros(cfg.n_layers * cfg.n_kv_heads * cfg.max_seq_len * 2 * hd, np.float32)
    rc = gen.q_b200_fill_kv_prefill(kv.ctypes.data, C.byref(cfg), PREFILL, SEED + 1, 0)
    if rc:
        raise RuntimeError(f"q_b200_fill_kv_prefill: {rc}")
    return kv


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (read + write) of one gate/up launch, from an ncu capture of
# `bench.py --only gemv` (profiles/gemv_q4_gate_up_28672x4096.txt).
GEMV_GU_TRAFFIC = 74_275_840


def gemv_roofline(Q, torch, peak_gbs: float) -> dict:
    """Dominant kernel: the fused gate/up Q4_0 GEMV shape of the 8B layer
    (28672 x 4096), launched back to back over 4 distinct weight sets (294 MB
    > L2) on torch's stream and timed with CUDA events."""
    M, K, n_sets, iters = 2 * CFG8B["hidden"], CFG8B["dim"], 4, 64
    nblk = M * K // 32
    packed = []
    host = np.zeros(nblk * 20, np.uint8)
    for i in range(n_sets):
        Q.lib.q_b200_fill_q4(Q.ptr(host), nblk, SEED + 10 + i, 3, 0, 0.001, 0.01, 0)
        src = torch.from_numpy(host).cuda()
        dst = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        Q.check(Q.lib.q_b200_q4_pack(src.data_ptr(), M, K, dst.data_ptr(), None), "pack")
        torch.cuda.synchronize()
        packed.append(dst)
        del src
    x = torch.randn(K, device="cuda")
    y = torch.empty(M, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for i in range(8):
        Q.check(Q.lib.q_b200_gemv_q4(packed[i % n_sets].data_ptr(), M, K, x.data_ptr(), y.data_ptr(), s), "gemv")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        Q.lib.q_b200_gemv_q4(packed[i % n_sets].data_ptr(), M, K, x.data_ptr(), y.data_ptr(), s)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    bytes_launch = M * K * 5 // 8 + 4 * K + 4 * M
    achieved = bytes_launch / (us * 1e-6) / 1e9
    return {"kernel": "q4_slab_kernel (fused gate/up 28672x4096)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "us_per_launch": round(us, 2),
            "bytes_per_launch": bytes_launch, "traffic": GEMV_GU_TRAFFIC,
            "traffic_source": "ncu dram__bytes_read+write of one launch, profiles/gemv_q4_gate_up_28672x4096.txt",
            "peak_source": "of measured"}


def cpu_reference_decode(path: str, cfg, steps: int, threads: int, budget_s: float = 1e9):
    """Upstream AVX2 kernels (oracle/_ref) over the same model and KV image:
    `steps` decode steps (fewer if they would pass budget_s of wall time)."""
    import oracle as O
    kind = "reference"
    try:
        m = O.RefModel(path, threads=threads)
    except (RuntimeError, OSError):
        m = O.OracleModel(path, threads=threads)
        kind = "port"
    m.kv[:] = kv_image(O.gen, cfg)
    tok = 1
    times = []
    for i in range(steps):
        t0 = time.perf_counter()
        lg = m.forward(np.array([tok], np.uint32), PREFILL + i)
        times.append(time.perf_counter() - t0)
        tok = int(np.argmax(lg))
        if sum(times) * (len(times) + 1) / len(times) > budget_s:
            break
    m.close()
    return kind, times


def gemv_sweep(Q, torch, peak_gbs: float, host: bool) -> list:
    """each Llama-3-8B projection shape as one Q4_0 GEMV
    launch (q_b200_gemv_q4), CUDA events over back-to-back launches that
    rotate over enough distinct weight sets to exceed L2 (>= 300 MB), beside
    upstream q_gemv_q4_f32_avx2 on one host thread (1 warm-up + 5 timed
    calls, as upstream tools/benchmark.c:22-50)."""
    import oracle as O  # the upstream kernel, timed as the CPU baseline
    out = []
    s = torch.cuda.current_stream().cuda_stream
    for M, K in SWEEP:
        nblk = M * K // 32
        bytes_launch = M * K * 5 // 8 + 4 * K + 4 * M
        n_sets = max(1, -(-300_000_000 // bytes_launch))
        n_sets = min(n_sets, 32)
        host_w = np.zeros(nblk * 20, np.uint8)
        packed = []
        for i in range(n_sets):
            Q.lib.q_b200_fill_q4(Q.ptr(host_w), nblk, SEED + 100 + i, 5, 0, 0.001, 0.01, 0)
            src = torch.from_numpy(host_w).cuda()
            dst = torch.empty(Q.lib.q_b200_q4_packed_bytes(M, K), dtype=torch.uint8, device="cuda")
            torch.cuda.synchronize()
            Q.check(Q.lib.q_b200_q4_pack(src.data_ptr(), M, K, dst.data_ptr(), None), "pack")
            torch.cuda.synchronize()
            packed.append(dst)
            del src
        x = Q.aligned_empty(K)
        Q.lib.q_b200_fill_normal(Q.ptr(x), K, SEED, 12, 0, 0.0, 1.0, 0)
        dx = torch.from_numpy(x.copy()).cuda()
        dy = torch.empty(M, device="cuda")
        iters = max(64, 4 * n_sets)
        for i in range(8):
            Q.check(Q.lib.q_b200_gemv_q4(packed[i % n_sets].data_ptr(), M, K, dx.data_ptr(), dy.data_ptr(), s), "gemv")
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(iters):
            Q.lib.q_b200_gemv_q4(packed[i % n_sets].data_ptr(), M, K, dx.data_ptr(), dy.data_ptr(), s)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / iters
        gbs = bytes_launch / (us * 1e-6) / 1e9
        row = {"shape": f"{M}x{K}", "bytes": bytes_launch, "us": round(us, 2), "gbs": round(gbs, 1),
               "frac": round(gbs / peak_gbs, 4), "weight_sets": n_sets}
        del packed
        if host:
            y = Q.aligned_empty(M)
            kind = O.upstream_gemv_q4(host_w, M, K, x, y)
            ts = []
            for _ in range(5):
                t0 = time.perf_counter()
                O.upstream_gemv_q4(host_w, M, K, x, y)
                ts.append(time.perf_counter() - t0)
            cms = 1e3 * sum(ts) / len(ts)
            row["cpu"] = {"kind": kind, "cores": 1, "ms": round(cms, 3),
                          "gbs": round(bytes_launch / (cms * 1e-3) / 1e9, 2)}
            row["speedup_vs_cpu"] = round(cms * 1e3 / us, 1)
        out.append(row)
    return out


def prefill_measure(Q, m, torch, peak_tf: float, reps: int = 3) -> dict:
    """one prompt of 2048 seeded uniform ids in
    [0, 128256) through llama_forward (the tensor-core prompt path), host
    ids in and the last row's logits out.  TTFT = wall time of the call;
    device time = CUDA events on the library stream around the same call.
    One untimed call first (workspace allocation, first-use set-up)."""
    S = PREFILL
    toks = np.zeros(S, np.uint32)
    Q.lib.q_b200_fill_tokens(Q.ptr(toks), S, SEED, 9, 0, CFG8B["vocab"])
    stream = torch.cuda.ExternalStream(m.stream)
    m.forward(toks, 0)
    walls, devs = [], []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0.record(stream)
        m.forward(toks, 0)
        e1.record(stream)
        walls.append(time.perf_counter() - t0)
        torch.cuda.synchronize()
        devs.append(e0.elapsed_time(e1) * 1e-3)
    D, H, L = CFG8B["dim"], CFG8B["hidden"], CFG8B["layers"]
    kvd = CFG8B["kv_heads"] * (D // CFG8B["heads"])
    lin = L * (D * D * 2 + kvd * D * 2 + H * D * 3)
    flop = 2.0 * lin * S + 2.0 * D * CFG8B["vocab"]  # projections + the last row's head
    attn = L * 2.0 * 2 * D * (S * (S + 1) / 2)          # causal q.k and p.v
    ttft = min(walls)
    dev = min(devs)
    return {"tokens": S, "ttft_ms": round(ttft * 1e3, 2), "device_ms": round(dev * 1e3, 2),
            "prompt_tok_s": round(S / ttft, 1), "flop": flop + attn,
            "tflops": round((flop + attn) / dev / 1e12, 1),
            "frac_of_bf16_peak": round((flop + attn) / dev / 1e12 / peak_tf, 4),
            "note": "the projections run 3 fp16 MMAs (hi*hi, hi*lo, lo*hi) per product for fp32-grade "
                    "results, so tensor-pipe work is 3x the flop counted here",
            "reps": reps, "source": "llama_forward(2048 ids, pos 0) with host buffers"}


CFG70B = dict(vocab=128256, dim=8192, hidden=28672, layers=80, heads=64, kv_heads=8)
BATCH = 16


def batch_measure(Q, torch, peak: float, steps: int = 16) -> dict:
    """BASELINE configs[4] (Llama-3-70B, batch 16) on one GPU, measured per
    layer: models with 2 and 4 layers of the 70B shapes (vocabulary cut to
    4096 so the files stay small), 16 sequences each with its own cache
    pre-filled to 2048 positions, q_b200_decode_batch_loop (argmax fed back
    on the device) timed with CUDA events on the library stream.  One layer
    = the difference of the two step times over 2.  A third model, 2 layers
    with the full 128256-row vocabulary, measures the step's fixed part (LM
    head, final norm, token feedback); the 80-layer step is estimated as
    that step + 78 measured layers."""
    import ctypes as C
    ms = {}
    for L, V in ((2, 4096), (4, 4096), (2, CFG70B["vocab"])):
        cfg = Q.config(V, CFG70B["dim"], CFG70B["hidden"], L, CFG70B["heads"], CFG70B["kv_heads"], 2304)
        p = str(Path(model_path(2304)).with_name(f"qorus_llama3_70b_{L}layer_v{V}.qorus"))
        if not (Path(p).exists() and Path(p).stat().st_size == int(Q.lib.q_b200_model_file_size(C.byref(cfg)))):
            Q.write_model(p, cfg, seed=SEED, threads=0)
        m = Q.Model(p)
        Q.check(Q.lib.q_b200_batch_init(C.byref(m.ctx), C.byref(m.model), BATCH), "batch_init")
        kv = np.zeros(L * CFG70B["kv_heads"] * 2304 * 256, np.float32)
        for b in range(BATCH):
            Q.check(Q.lib.q_b200_fill_kv_prefill(Q.ptr(kv), C.byref(cfg), PREFILL, SEED + b, 0), "fill_kv")
            Q.check(Q.lib.q_b200_batch_kv_write(C.byref(m.ctx), b, 0, Q.ptr(kv), kv.nbytes), "batch_kv_write")
        del kv
        toks = np.arange(1, BATCH + 1, dtype=np.uint32)
        pos = np.full(BATCH, PREFILL, np.uint32)
        out = np.zeros((steps + 3) * BATCH, np.uint32)
        Q.check(Q.lib.q_b200_decode_batch_loop(C.byref(m.model), C.byref(m.ctx), Q.ptr(toks), Q.ptr(pos), 3,
                                               Q.ptr(out), 1), "batch_loop")
        stream = torch.cuda.ExternalStream(m.stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        pos += 3
        e0.record(stream)
        Q.check(Q.lib.q_b200_decode_batch_loop(C.byref(m.model), C.byref(m.ctx), Q.ptr(toks), Q.ptr(pos), steps,
                                               Q.ptr(out), 0), "batch_loop")
        e1.record(stream)
        torch.cuda.synchronize()
        ms[(L, V)] = e0.elapsed_time(e1) / steps
        m.close()
        if V != 4096:  # 9 GB of host memory in /dev/shm: not kept
            Path(p).unlink(missing_ok=True)
    layer_ms = (ms[(4, 4096)] - ms[(2, 4096)]) / 2
    c = dict(CFG70B, layers=1)
    ctx = PREFILL + 3 + steps // 2
    layer_bytes = q4_linear_bytes(c) + BATCH * CFG70B["kv_heads"] * ctx * (CFG70B["dim"] // CFG70B["heads"]) * 8
    step_ms = ms[(2, CFG70B["vocab"])] + (CFG70B["layers"] - 2) * layer_ms
    fixed_ms = ms[(2, CFG70B["vocab"])] - 2 * layer_ms  # LM head, final norm, feedback
    head_bytes = CFG70B["vocab"] * CFG70B["dim"] * 4
    return {"batch": BATCH, "context": ctx, "steps": steps,
            "step_ms_2layer": round(ms[(2, 4096)], 4), "step_ms_4layer": round(ms[(4, 4096)], 4),
            "step_ms_2layer_full_vocab": round(ms[(2, CFG70B["vocab"])], 4),
            "head_us": round(fixed_ms * 1e3, 1), "head_gbs": round(head_bytes / (fixed_ms * 1e-3) / 1e9, 1),
            "layer_us": round(layer_ms * 1e3, 2), "layer_bytes": layer_bytes,
            "layer_gbs": round(layer_bytes / (layer_ms * 1e-3) / 1e9, 1),
            "layer_frac": round(layer_bytes / (layer_ms * 1e-3) / 1e9 / peak, 4),
            "est_tok_s_80_layers": round(BATCH / (step_ms * 1e-3), 1),
            "source": "q_b200_decode_batch_loop, 70B layer shapes: 2- and 4-layer models (vocab 4096) for the "
                      "layer, a 2-layer model with the full vocabulary for the head; 80-layer figure = that "
                      "step + 78 measured layers (estimate)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-batch", action="store_true")
    ap.add_argument("--only", choices=["gemv", "attention", "head", "prefill", "batch"],
                    help="profiling runs: the gate/up GEMV alone, a few decode steps of a "
                         "2-layer 8B-shaped model (small vocab) over a 2048-position cache, "
                         "the FP32 LM-head GEMV (128256 x 4096) alone, a 2048-row prompt through "
                         "2 8B-shaped layers, or the batch-16 decode of 70B-shaped layers")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    max_seq = PREFILL + 2 * (args.steps + args.warmup) + 64 + 320  # + the clock soak

    if args.impl == "reference":
        # CPU only: the upstream kernels; the CUDA library is never loaded here
        if rank != 0:
            return
        import oracle as O
        cfg = O.config(CFG8B["vocab"], CFG8B["dim"], CFG8B["hidden"], CFG8B["layers"],
                       CFG8B["heads"], CFG8B["kv_heads"], max_seq)
        path = ensure_model(O.gen, cfg, max_seq, 0, lambda: None)
        threads = os.cpu_count() or 1
        warm = args.warmup
        kind, times = cpu_reference_decode(path, cfg, warm + args.steps, threads, budget_s=150.0)
        warm = min(warm, max(1, len(times) - 1))  # the time budget may stop the run early
        times = times[warm:]
        tps = len(times) / sum(times)
        line = {"metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": len(times), "warmup": warm,
                "ms_per_step": round(1e3 * sum(times) / len(times), 2), "higher_is_better": True,
                "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
                "dtype": "f32 (q4_0 weights)", "data": "synthetic", "config": CONFIG,
                "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": threads,
                                 "kind": kind, "sample": f"{len(times)} decode steps of the "
                                 "8B-shaped model at context 2049+ (every step a full token; "
                                 "upstream AVX2 kernels, row-parallel over all host threads)"},
                "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    if args.only == "gemv":
        import qorus_b200 as Q
        print(json.dumps(gemv_roofline(Q, torch, 6450.9)), flush=True)
        return
    if args.only == "head":
        import qorus_b200 as Q
        M, K = CFG8B["vocab"], CFG8B["dim"]
        g = torch.Generator(device="cuda").manual_seed(SEED)
        w = torch.randn(M, K, device="cuda", generator=g) * 0.02
        x = torch.randn(K, device="cuda", generator=g)
        y = torch.empty(M, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        n = max(4, args.steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(n):
            if i == 2:
                e0.record()
            Q.check(Q.lib.q_b200_gemv_f32(w.data_ptr(), M, K, x.data_ptr(), y.data_ptr(), s), "gemv_f32")
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (n - 2)
        print(json.dumps({"only": "head", "launches": n, "us_per_launch": round(us, 1),
                          "gbs": round(M * K * 4 / (us * 1e-6) / 1e9, 1)}), flush=True)
        return
    if args.only == "prefill":
        # profiling run: a 2048-row prompt through 2 Llama-3-8B-shaped layers
        import qorus_b200 as Q
        small = Q.config(32000, CFG8B["dim"], CFG8B["hidden"], 2, CFG8B["heads"], CFG8B["kv_heads"], 2304)
        spath = str(Path(model_path(2304)).with_name("qorus_llama3_8b_2layer_prefill.qorus"))
        Q.write_model(spath, small, seed=SEED, threads=0)
        ms = Q.Model(spath)
        toks = np.zeros(PREFILL, np.uint32)
        Q.lib.q_b200_fill_tokens(Q.ptr(toks), PREFILL, SEED, 9, 0, 32000)
        for _ in range(max(1, args.steps)):
            ms.forward(toks, 0)
        print(json.dumps({"only": "prefill", "calls": max(1, args.steps)}), flush=True)
        return
    if args.only == "batch":
        import qorus_b200 as Q
        print(json.dumps({"only": "batch", **batch_measure(Q, torch, 6450.9, max(4, args.steps))}), flush=True)
        return
    if args.only == "attention":
        import qorus_b200 as Q
        small = Q.config(4096, CFG8B["dim"], CFG8B["hidden"], 2, CFG8B["heads"], CFG8B["kv_heads"], 4096)
        spath = str(Path(model_path(4096)).with_name("qorus_llama3_8b_2layer_small.qorus"))
        Q.write_model(spath, small, seed=SEED, threads=0)
        ms = Q.Model(spath)
        ms.kv_write(kv_image(Q.lib, small))
        toks = ms.decode_loop(1, PREFILL, max(4, args.steps), sync=True)
        print(json.dumps({"only": "attention", "steps": int(len(toks))}), flush=True)
        return
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()

    import qorus_b200 as Q
    cfg = Q.config(CFG8B["vocab"], CFG8B["dim"], CFG8B["hidden"], CFG8B["layers"],
                   CFG8B["heads"], CFG8B["kv_heads"], max_seq)
    path = ensure_model(Q.lib, cfg, max_seq, rank, barrier)
    t_load = time.perf_counter()
    tp = None
    if world > 1:
        # tensor parallel: rank 0 makes the NCCL id, the process group carries it
        box = [Q.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = (rank, world, box[0])

    def gather(b):  # CUDA IPC handles of the peer-memory all-reduce buffers
        allb = [None] * world
        dist.all_gather_object(allb, b)
        return allb
    m = Q.Model(path, tp=tp, tp_gather=gather if world > 1 else None)
    kv = kv_image(Q.lib, cfg)
    if world > 1:  # this rank's KV heads: [L][n_kv/W][max_seq][K|V]
        sh = Q.tp_shape(cfg, rank, world)
        h0 = sh["kv0"] // (cfg.dim // cfg.n_heads)
        kv = np.ascontiguousarray(kv.reshape(cfg.n_layers, cfg.n_kv_heads, -1)[:, h0: h0 + sh["nkv"]]).ravel()
    m.kv_write(kv)
    del kv
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(m.stream)

    # warm-up: W device steps
    pos = PREFILL
    m.decode_loop(1, pos, args.warmup, sync=True)
    pos += args.warmup
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        # the same decode steps for ~0.6 s before the timed region, untimed,
        # so the clock sampler sees this load and not only the region's
        # few milliseconds
        soak = 300
        Q.check(Q.lib.q_b200_decode_loop(C.byref(m.model), C.byref(m.ctx), 1, pos, soak, None, 0),
                "decode_loop")
        torch.cuda.synchronize()
        pos += soak
        barrier()
        torch.cuda.synchronize()
        launches0 = Q.lib.q_b200_kernel_launches()
        t_pos = pos
        e0.record(stream)
        Q.check(Q.lib.q_b200_decode_loop(C.byref(m.model), C.byref(m.ctx), 1, pos, args.steps,
                                         None, 0), "decode_loop")
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    launches = Q.lib.q_b200_kernel_launches() - launches0
    pos += args.steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = args.steps / (ms * 1e-3)  # one sequence (tensor parallel over all ranks)

    # e2e: the upstream entry point, host token in / host logits out
    tok = np.array([1], np.uint32)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        lg = m.forward(tok, pos + i)
        tok[0] = int(np.argmax(lg))
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = args.steps / e2e_s

    # in-graph kernel times of one traced step (outside the timed region):
    # gate/up GEMV (the roofline kernel) and the LM head, with their bytes
    in_graph = None
    if world == 1:
        st = m.profile_step(int(tok[0]), pos + args.steps).astype(np.int64)
        L = CFG8B["layers"]
        if len(st) == 5 * L + 2:
            run = [int(c - max(b, st[i - 1, 2] if i else a)) for i, (a, b, c) in enumerate(st)]
            gu = [run[3 + 5 * l] for l in range(L)]
            gu_us = sum(gu) / len(gu) / 1e3
            head_us = run[-2] / 1e3
            gu_bytes = 2 * CFG8B["hidden"] * CFG8B["dim"] * 5 // 8
            head_bytes = CFG8B["vocab"] * CFG8B["dim"] * 4
            in_graph = {"source": "q_b200_profile_step: %globaltimer stamps of one decode step",
                        "gate_up_us": round(gu_us, 2), "gate_up_gbs": round(gu_bytes / (gu_us * 1e-6) / 1e9, 1),
                        "lm_head_us": round(head_us, 1), "lm_head_gbs": round(head_bytes / (head_us * 1e-6) / 1e9, 1),
                        "step_us": round((st[-1, 2] - st[0, 0]) / 1e3, 1)}
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("hbm_gbs", 6650.0))
    roof = gemv_roofline(Q, torch, peak)
    if not peaks:
        roof["peak_source"] = "of fallback"
    ctx_mid = t_pos + args.steps // 2  # mean context of the timed steps
    step_bytes = token_bytes(CFG8B, ctx_mid)
    step_gbs = step_bytes / (ms * 1e-3 / args.steps) / 1e9

    sweep = gemv_sweep(Q, torch, peak, host=not args.no_cpu_baseline) if world == 1 else None
    prefill = None
    if world == 1 and not args.no_prefill:
        prefill = prefill_measure(Q, m, torch, float(peaks.get("bf16_tflops", 1590.0)))
    batch = None
    if world == 1 and not args.no_batch:
        batch = batch_measure(Q, torch, peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        m.close()
        # upstream as shipped: one thread (the reference has no threading)
        kind, times = cpu_reference_decode(path, cfg, 3, 1)
        cpu = {"value": round(len(times) / sum(times), 4), "unit": "tok/s", "cores": 1,
               "kind": kind, "sample": f"{len(times)} full decode steps of the same 8B-shaped "
               "model and KV image at context 2049+ (upstream AVX2 kernels, one thread)"}
        threads = os.cpu_count() or 1
        kind, times = cpu_reference_decode(path, cfg, 4, threads)
        times = times[1:]
        cpu["threaded"] = {"value": round(len(times) / sum(times), 3), "unit": "tok/s",
                           "cores": threads, "kind": kind,
                           "sample": f"{len(times)} decode steps after one warm-up, the upstream "
                           "kernels row-parallel over all host threads (the --impl reference arm's setup)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "f32 (q4_0 weights)", "data": "synthetic",
            "config": CONFIG,
            "parallelism": f"tp{world}" if world > 1 else "single",
            "roofline": roof,
            "in_graph": in_graph,
            # the token's bytes over all ranks' HBM (each rank streams its shard)
            "step_roofline": {"bytes_per_token": step_bytes, "achieved": round(step_gbs, 1),
                              "peak": round(peak * world, 1), "unit": "GB/s",
                              "frac": round(step_gbs / (peak * world), 4)},
            "cpu_baseline": cpu,
            "sweep": sweep,
            "prefill": prefill,
            "batch_decode": batch,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 + 16,
                    "d2h_bytes_per_step": CFG8B["vocab"] * 4},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "load_s": round(t_load, 1),
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
