#!/usr/bin/env python
"""Decode benchmark: Llama-3-8B-shaped q4 decoder, batch 1, context 4096.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (the 8B configuration of the q4 decode metric): dim 4096, 32 layers,
32 query / 8 KV heads (head_dim 128), SwiGLU 14336, vocab 128256, RoPE theta
5e5, RMSNorm eps 1e-5; weights N(0, 0.02) quantised to q4 (group 32) by the
reference rule, generated on the device from a seed (synthetic data, no
checkpoint). A 512-token random prompt is fed, greedy decode fills the
context, and the timed steps decode at context ~4096. One step = one token
for every sequence of the batch.

value: tokens/s from CUDA events around K device-side steps (weights and KV
are 5.8 GB per step, far above the 126 MB L2, so no flush is needed).
e2e:   tokens/s through att1_infer_decode_token (token id in from the host,
       next token id and the error word back each step), CUDA events around
       the loop on the library's stream.
roofline: the dominant kernel (the q4 GEMV at the gate/up shape, 28672x4096)
       timed alone with CUDA events over rotating weight copies (294 MB, so
       every launch streams from HBM), algorithmic bytes / time vs the
       measured HBM copy bandwidth.
cpu_baseline: the reference CPU implementation (compiled from its sources,
       oracle/_ref) on a bounded sample of the same workload, all host cores
       for its matmuls.

--impl reference runs only that reference CPU measurement (rank 0).
Under torchrun (N>1) ranks run tensor-parallel shards when the build
supports it; the JSON line reports whole-job tokens/s (max time over ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "att-1_b200"))

SHAPE = dict(vocab=128256, n_layers=32, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
             theta=500000.0, eps=1e-5)
METRIC = "q4 decode tokens/s (Llama-3-8B shape, batch 1, ctx 4096)"
WORKLOAD = "llama3-8b-shape q4 decode"
# the Llama-70B-shaped workload: 8-way tensor parallel, batch 64 at context 8192
SHAPE_70B = dict(vocab=128256, n_layers=80, n_heads=64, n_kv_heads=8, d_model=8192, d_ff=28672,
                 theta=500000.0, eps=1e-5)
METRIC_70B = "q4 decode tokens/s (Llama-70B shape, batch 64, ctx 8192)"


def q4_bytes(r, c):
    return r * c // 2 + r * (c // 32) * 4


def step_bytes(ctx, batch=1, s=SHAPE):
    d, H, Hkv, F, V, L = s["d_model"], s["n_heads"], s["n_kv_heads"], s["d_ff"], s["vocab"], s["n_layers"]
    hd = d // H
    w = L * (q4_bytes(H * hd, d) + 2 * q4_bytes(Hkv * hd, d) + q4_bytes(d, H * hd) + 2 * q4_bytes(F, d) +
             q4_bytes(d, F)) + q4_bytes(V, d)
    kv = batch * L * 2 * ctx * Hkv * hd * 4
    app = batch * (L * 2 * Hkv * hd * 4 + d * 4)
    return w + kv + app


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------
# reference CPU path (oracle/_ref: the ATT-1 sources compiled as they are)
# ---------------------------------------------------------------------------------------------

REF_SHIPPED = "libatt1ref_shipped.so"   # the reference Makefile's flags (no -O)


def reference_cpu_sample(ctx, steps=2, warmup=1, threads=None, lib=None):
    """Time the reference decode (oracle/_ref: the ATT-1 sources compiled as
    they are, driven through its own block functions) on a bounded sample of
    the 8B workload: full-width layers with GQA expanded to the reference's
    MHA layout, KV filled to the context, a 4096-entry lm_head; a 1- and a
    2-layer model separate the per-layer and the per-token parts, which are
    extrapolated to 32 layers and the 128256-entry vocabulary. `steps` decode
    steps are timed on each sample model after `warmup` untimed ones.
    threads: host threads for the matmuls (row slices; None = all cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    threads = cores if threads is None else threads
    ref = O.Reference(O.REF_SO if lib is None else os.path.join(os.path.dirname(O.REF_SO), lib))
    times = {}
    timed = 0.0
    vs = 4096
    for layers in (1, 2):
        cfg = O.Config.make(vocab=vs, n_layers=layers, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
                            max_seq=ctx, dtype=O.Q4, eps=1e-5, theta=500000.0)
        m = ref.model(cfg, 11, threads=cores)
        m.set_threads(threads)
        m.fill(ctx - 1 - steps - warmup)
        for i in range(warmup):
            m.decode(5 + i)
        t0 = time.perf_counter()
        for i in range(steps):
            m.decode(7 + i)
        dt = time.perf_counter() - t0
        timed += dt
        times[layers] = dt / steps
        m.close()
    t_layer = max(times[2] - times[1], 1e-9)
    t_head = max(times[1] - t_layer, 0.0)
    t_tok = SHAPE["n_layers"] * t_layer + t_head * SHAPE["vocab"] / vs
    sample = (f"reference att1 decode at ctx {ctx}: 1- and 2-layer full-width models (GQA expanded to MHA), "
              f"lm_head 4096 rows, {steps} timed steps each after {warmup} untimed; {t_layer * 1e3:.1f} ms/layer, "
              f"extrapolated to 32 layers + 128256-row lm_head")
    return {"value": 1.0 / t_tok, "cores": threads, "host_cores": cores, "sample": sample, "timed_region_s": timed,
            "ms_per_layer": t_layer * 1e3}


def reference_single_core_rows(ctx):
    """The reference as its own Makefile builds it (no -O) and at -O2, on one
    host core each (its math is single-threaded): one timed step per sample
    model, extrapolated like reference_cpu_sample."""
    rows = []
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    for build, lib in (("as shipped (no -O, reference Makefile:10)", REF_SHIPPED), ("-O2", None)):
        path = os.path.join(os.path.dirname(O.REF_SO), lib) if lib else O.REF_SO
        if not os.path.exists(path):
            rows.append({"build": build, "unavailable": f"{os.path.basename(path)} not built"})
            continue
        r = reference_cpu_sample(ctx, steps=1, warmup=0, threads=1, lib=lib)
        rows.append({"build": build, "value": r["value"], "unit": "tokens/s",
                     "cores": f"1 of {r['host_cores']} host cores", "ms_per_layer": r["ms_per_layer"],
                     "timed_region_s": r["timed_region_s"], "extrapolated": True})
    return rows


# ---------------------------------------------------------------------------------------------
# B200 path
# ---------------------------------------------------------------------------------------------

def time_dominant_gemv(b2, torch, reps=30):
    """q4 GEMV at the gate/up shape on 4 rotating weight copies (294 MB)."""
    import ctypes as C
    L = b2.lib()
    rows, cols = 2 * SHAPE["d_ff"], SHAPE["d_model"]
    nbuf = 4
    bufs = [torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda") for _ in range(nbuf)]
    for i, b in enumerate(bufs):
        assert L.b2_q4_synth(b.data_ptr(), 0, rows, cols, 5, 100 + 2 * i, 101 + 2 * i, 0.02, b2.ROWS_GATEUP,
                             None) == 0
    x = torch.randn(cols, device="cuda")
    g = torch.ones(cols, device="cuda")
    out = torch.zeros(SHAPE["d_ff"], device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = []
    for b in bufs:
        a = b2.GemvArgs()
        a.w = b2.QWeight(b.data_ptr(), None, 4, rows, cols, rows // 16, cols // 64)
        a.batch = 1
        a.x = x.data_ptr()
        a.x_stride = cols
        a.norm_w = g.data_ptr()
        a.eps = 1e-5
        a.epilogue = b2.EPI_SWIGLU
        a.out = out.data_ptr()
        a.out_stride = SHAPE["d_ff"]
        a.err = err.data_ptr()
        args.append(a)
    need = L.b2_gemv_scratch_bytes(C.byref(args[0]))
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(L.b2_gemv_counters_len(C.byref(args[0])), dtype=torch.int32, device="cuda")
    for a in args:
        a.scratch = scratch.data_ptr()
        a.scratch_bytes = need
        a.counters = counters.data_ptr()
        a.counters_len = counters.numel()
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(8):
            assert L.b2_gemv(C.byref(args[i % nbuf]), C.c_void_p(sp)) == 0
        # back-to-back launches on one stream (each streams a different 73 MB
        # copy from HBM); the average is the per-launch device time
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            L.b2_gemv(C.byref(args[i % nbuf]), C.c_void_p(sp))
        e1.record(stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ms = e0.elapsed_time(e1) / reps
    algo = q4_bytes(rows, cols) + cols * 4 * 2 + SHAPE["d_ff"] * 4
    del bufs
    return algo, ms


def time_attention(b2, torch, reps=30, ctx=4096, layers=8):
    """Single-query attention of the 8B shape at context `ctx`: 8 layers of KV
    pools (268 MB at 4096, larger than L2) used in turn, back-to-back launches."""
    import ctypes as C
    L = b2.lib()
    H, HKV = SHAPE["n_heads"], SHAPE["n_kv_heads"]
    hd = SHAPE["d_model"] // H
    pt = 64
    pages = (ctx + pt - 1) // pt
    kp = [torch.randn(pages * HKV * pt * hd, device="cuda") * 0.1 for _ in range(layers)]
    vp = [torch.randn(pages * HKV * pt * hd, device="cuda") for _ in range(layers)]
    ptab = torch.arange(pages, dtype=torch.int32, device="cuda")
    q = torch.randn(H * hd, device="cuda")
    out = torch.zeros(H * hd, device="cuda")
    pos = torch.tensor([ctx - 1], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = []
    for layer in range(layers):
        a = b2.AttnArgs()
        a.batch, a.n_heads, a.n_kv_heads, a.head_dim = 1, H, HKV, hd
        a.q, a.ctx, a.positions, a.max_ctx, a.err = q.data_ptr(), out.data_ptr(), pos.data_ptr(), ctx, err.data_ptr()
        a.kv = b2.KVLayout(kp[layer].data_ptr(), vp[layer].data_ptr(), ptab.data_ptr(), pt, pages, HKV, hd)
        args.append(a)
    need, ncnt = L.b2_attn_scratch_bytes(C.byref(args[0])), L.b2_attn_counters_len(C.byref(args[0]))
    scr = torch.zeros(need, dtype=torch.uint8, device="cuda")
    cnt = torch.zeros(ncnt, dtype=torch.int32, device="cuda")
    for a in args:
        a.scratch, a.scratch_bytes, a.counters, a.counters_len = scr.data_ptr(), need, cnt.data_ptr(), ncnt
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(8):
            assert L.b2_attn(C.byref(args[i % layers]), sp) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            L.b2_attn(C.byref(args[i % layers]), sp)
        e1.record(stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ms = e0.elapsed_time(e1) / reps
    algo = 2 * HKV * ctx * hd * 4 + 2 * H * hd * 4
    return algo, ms


def time_prefill(b2, torch, n=512, seed=3):
    """Prompt prefill of the 8B shape: n tokens through att1_b200_infer_prefill
    (tcgen05 dequant-GEMM for every projection, causal attention) on a fresh
    context, CUDA events on the context's stream."""
    import numpy as np
    cfg = b2.Config.make(SHAPE["vocab"], SHAPE["n_layers"], SHAPE["n_heads"], SHAPE["n_kv_heads"], SHAPE["d_model"],
                         SHAPE["d_ff"], 4096, dtype=4, eps=SHAPE["eps"], theta=SHAPE["theta"])
    inf = b2.Infer.synth(cfg, seed)
    toks = np.random.default_rng(seed).integers(0, SHAPE["vocab"], size=n)
    inf.prefill(toks[:64])           # warm-up (plans, first launches)
    inf.seek(0)
    st = torch.cuda.ExternalStream(inf.stream())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    inf.prefill(toks)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    inf.close()
    d, F, V, L = SHAPE["d_model"], SHAPE["d_ff"], SHAPE["vocab"], SHAPE["n_layers"]
    hd = d // SHAPE["n_heads"]
    params = L * (d * (SHAPE["n_heads"] + 2 * SHAPE["n_kv_heads"]) * hd + d * d + 3 * F * d) + V * d
    flops = 2.0 * n * params                        # the products of the reference's f32 matmuls
    return {"tokens": n, "ms": ms, "tokens_per_s": n / (ms * 1e-3), "useful_tflops": flops / (ms * 1e-3) / 1e12,
            "note": "useful = 2 * tokens * weights (f32-equivalent products); the GEMM issues 2 bf16 MMAs "
                    "per product (x hi/lo as one operand, w hi/lo) for q4"}


def time_batch_decode(b2, torch, batch=32, ctx=1024, steps=10, seed=4):
    """Decode of `batch` sequences at context ~ctx through the tensor-core
    route (batches above what the GEMVs hold), device-loop steps timed with
    CUDA events. The KV of positions before ctx is the context's own
    (zero-initialised) pages: the attention reads ctx positions per sequence
    either way."""
    cfg = b2.Config.make(SHAPE["vocab"], SHAPE["n_layers"], SHAPE["n_heads"], SHAPE["n_kv_heads"], SHAPE["d_model"],
                         SHAPE["d_ff"], ctx + 64, dtype=4, eps=SHAPE["eps"], theta=SHAPE["theta"])
    inf = b2.Infer.synth(cfg, seed, batch=batch)
    inf.decode_batch(list(range(1, batch + 1)))
    inf.seek(ctx - steps - 3)
    inf.run_steps(3)
    inf.sync()
    st = torch.cuda.ExternalStream(inf.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    inf.run_steps(steps)
    e1.record(st)
    inf.sync()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    inf.close()
    by = step_bytes(ctx - steps // 2, batch)
    peak, _ = measured_peak()
    return {"batch": batch, "ctx": ctx, "ms_per_step": ms, "tokens_per_s": batch * 1000.0 / ms,
            "hbm_frac": by / (ms * 1e-3) / (peak * 1e9), "step_bytes": by}


def time_decode_config(b2, torch, shape, dtype, batch, ctx, steps=20, seed=6):
    """Decode of another named configuration: `batch` sequences of a synthetic
    model of `shape` (dtype 4 = q4, 8 = q8) at context ~ctx (reached by seeking;
    the attention reads every position either way), device-loop steps timed
    with CUDA events after 3 warm-up steps."""
    cfg = b2.Config.make(shape["vocab"], shape["n_layers"], shape["n_heads"], shape["n_kv_heads"], shape["d_model"],
                         shape["d_ff"], shape["max_seq"], dtype=dtype, eps=shape["eps"], theta=shape["theta"])
    inf = b2.Infer.synth(cfg, seed, batch=batch)
    inf.decode_batch(list(range(1, batch + 1)))
    inf.seek(max(1, ctx - steps - 3))
    inf.run_steps(3)
    inf.sync()
    st = torch.cuda.ExternalStream(inf.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    inf.run_steps(steps)
    e1.record(st)
    inf.sync()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    inf.close()
    return {"batch": batch, "ctx": ctx, "dtype": "q4" if dtype == 4 else "q8", "ms_per_step": ms,
            "tokens_per_s": batch * 1000.0 / ms}


def time_matvec(b2, torch, rows, cols, batch, reps=40):
    """The q4 matvec microbenchmark: W [rows x cols] (seeded N(0, 0.02), packed
    by the reference q4 rule on the device) times `batch` vectors x ~ N(0, 1),
    no norm, plain epilogue; weights rotated over copies covering more than L2,
    back-to-back launches timed with CUDA events. Returns HBM GB/s of the
    algorithmic bytes (weights + x + out) and the fraction of the measured peak."""
    import ctypes as C
    L = b2.lib()
    wbytes = L.b2_q4_bytes(rows, cols)
    nbuf = max(2, -(-300_000_000 // wbytes))
    bufs = [torch.zeros(wbytes, dtype=torch.uint8, device="cuda") for _ in range(nbuf)]
    for i, b in enumerate(bufs):
        assert L.b2_q4_synth(b.data_ptr(), 0, rows, cols, 7, 200 + i, 0, 0.02, b2.ROWS_PLAIN, None) == 0
    x = torch.randn(batch * cols, device="cuda")
    out = torch.zeros(batch * rows, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = []
    for b in bufs:
        a = b2.GemvArgs()
        a.w = b2.QWeight(b.data_ptr(), None, 4, rows, cols, rows // 16, cols // 64)
        a.batch, a.x, a.x_stride = batch, x.data_ptr(), cols
        a.epilogue, a.out, a.out_stride, a.err = 0, out.data_ptr(), rows, err.data_ptr()
        args.append(a)
    need = L.b2_gemv_scratch_bytes(C.byref(args[0]))
    scratch = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    counters = torch.zeros(max(1, L.b2_gemv_counters_len(C.byref(args[0]))), dtype=torch.int32, device="cuda")
    for a in args:
        a.scratch, a.scratch_bytes = scratch.data_ptr(), need
        a.counters, a.counters_len = counters.data_ptr(), counters.numel()
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(2 * nbuf):
            assert L.b2_gemv(C.byref(args[i % nbuf]), sp) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            L.b2_gemv(C.byref(args[i % nbuf]), sp)
        e1.record(stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ms = e0.elapsed_time(e1) / reps
    algo = q4_bytes(rows, cols) + 4 * batch * (cols + rows)
    peak, _ = measured_peak()
    gbs = algo / (ms * 1e-3) / 1e9
    return {"rows": rows, "cols": cols, "batch": batch, "launch_us": ms * 1e3, "GB/s": gbs, "frac": gbs / peak}


SMALL_GQA = {"vocab": 49152, "n_layers": 30, "n_heads": 9, "n_kv_heads": 3, "d_model": 576, "d_ff": 1536,
             "max_seq": 2048, "eps": 1e-5, "theta": 10000.0}
TINY_Q8 = {"vocab": 32000, "n_layers": 6, "n_heads": 6, "n_kv_heads": 6, "d_model": 288, "d_ff": 768,
           "max_seq": 256, "eps": 1e-5, "theta": 10000.0}


def other_configs(b2, torch):
    """One line per other named workload (synthetic weights of that shape)."""
    out = {}
    # tiny q8 decoder: 16-token prompt + 128 greedy tokens, timed at the end of the run
    out["tiny_q8_b1"] = time_decode_config(b2, torch, TINY_Q8, 8, 1, 16 + 128)
    # small GQA q4 decoder near the end of its 2048 context, batch 1 and 16
    out["small_gqa_b1"] = time_decode_config(b2, torch, SMALL_GQA, 4, 1, 2040)
    out["small_gqa_b16"] = time_decode_config(b2, torch, SMALL_GQA, 4, 16, 2040)
    # q4 matvec microbenchmark
    for rows in (4096, 14336):
        for batch in (1, 8):
            out[f"matvec_q4_{rows}x4096_b{batch}"] = time_matvec(b2, torch, rows, 4096, batch)
    return out


def time_gemm(b2, torch, m=512, rows=14336 * 2, cols=4096, reps=10):
    """The tcgen05 dequant GEMM alone: m rows of x (prefill tokens or decode
    sequences) against a q4 [rows x cols] matrix in the unit layout (the
    gate/up shape by default), x prepared once; back-to-back launches timed
    with CUDA events. Returns useful flops (2 m rows cols) and bf16 MMA flops
    (two bf16 MMAs per product for q4: x hi/lo stacked against w hi, and w lo
    against x hi)."""
    import ctypes as C
    L = b2.lib()
    w = torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(w.data_ptr(), 0, rows, cols, 5, 100, 101, 0.02, b2.ROWS_GATEUP, None) == 0
    x = torch.randn(m * cols, device="cuda")
    xs = torch.zeros(L.b2_gemm_xs_bytes(m, cols), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.b2_gemm_prep(x.data_ptr(), cols, m, cols, None, 1e-5, xs.data_ptr(), err.data_ptr(), None) == 0
    out = torch.zeros(m * rows, device="cuda")
    a = b2.GemmArgs()
    a.w = b2.QWeight(w.data_ptr(), None, 4, rows, cols, rows // 16, cols // 64)
    a.xs, a.m, a.epilogue, a.out, a.out_stride, a.err = xs.data_ptr(), m, 0, out.data_ptr(), rows, err.data_ptr()
    need = L.b2_gemm_scratch_bytes(C.byref(a))
    scratch = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")
    a.scratch, a.scratch_bytes = scratch.data_ptr(), need
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(3):
            assert L.b2_gemm(C.byref(a), sp) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            L.b2_gemm(C.byref(a), sp)
        e1.record(stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * m * rows * cols
    return {"m": m, "rows": rows, "cols": cols, "launch_ms": ms, "useful_tflops": flops / (ms * 1e-3) / 1e12,
            "bf16_mma_tflops": 2 * flops / (ms * 1e-3) / 1e12, "weight_GBps": q4_bytes(rows, cols) / (ms * 1e-3) / 1e9}


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch

    import att1_b200 as b2

    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    ctx = args.ctx
    e2e_steps = max(args.steps, 8)
    cfg = b2.Config.make(SHAPE["vocab"], args.layers, SHAPE["n_heads"], SHAPE["n_kv_heads"],
                         SHAPE["d_model"], SHAPE["d_ff"], ctx, dtype=4, eps=SHAPE["eps"], theta=SHAPE["theta"])
    if world > 1 and not args.replicas:
        # tensor parallel: this rank's shard; ranks exchange their exchange-region
        # handles (CUDA IPC) over the process group, then connect
        inf = b2.Infer.synth_tp(cfg, args.seed, rank, world, batch=args.batch, device=local_rank)
        if args.tp_exchange == "nccl":
            # comparison arm: the exchange as NCCL collectives on the step's stream
            ids = [b2.Infer.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(ids, src=0)
            inf.tp_connect_nccl(ids[0])
        else:
            handles = [None] * world
            dist.all_gather_object(handles, inf.tp_handle())
            inf.tp_connect(handles)
    else:
        b2.lib().att1_b200_set_device(local_rank)
        inf = b2.Infer.synth(cfg, args.seed, batch=args.batch)
    if args.no_graph:
        inf.set_options(graph=False, pdl=False)
    persistent = args.persistent
    if persistent:
        inf.set_options(persistent=True)
    rng = np.random.default_rng(args.seed + rank)
    prompt = rng.integers(0, SHAPE["vocab"], size=(args.prompt, args.batch), dtype=np.int64)
    for t in prompt:
        tok = inf.decode_batch(t)
    fill = ctx - args.warmup - args.steps - e2e_steps - args.prompt
    if fill > 0 and args.seek_fill:
        # jump to the timed context without decoding the positions in between
        # (their K/V rows stay zero; the attention reads them all the same)
        inf.seek(inf.position() + fill)
    elif fill > 0:
        inf.run_steps(fill)
    inf.sync()
    st = torch.cuda.ExternalStream(inf.stream())

    # warm-up
    inf.run_steps(args.warmup)
    inf.sync()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local_rank)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    inf.run_steps(args.steps)
    e1.record(st)
    inf.sync()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1) / args.steps
    pos_timed = inf.position()
    graph_ops = inf.step_launches()  # operations in one step of the captured graph (0 without graphs)

    # end to end through att1_infer_decode_token / att1_b200_infer_decode_batch
    toks = inf.decode_batch(np.asarray(tok))
    if dist:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(st)
    t0 = time.perf_counter()
    for _ in range(e2e_steps - 1):
        if args.batch == 1:
            toks = [inf.decode(int(toks[0]))]
        else:
            toks = inf.decode_batch(toks)
    f1.record(st)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / (e2e_steps - 1)
    e2e_ms = max(f0.elapsed_time(f1) / (e2e_steps - 1), wall * 1e3)

    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])

    if dist and not args.replicas:
        inf.tp_disconnect()  # unmap the peers' regions before any rank frees its own
        dist.barrier()
    inf.close()
    algo, kms = time_dominant_gemv(b2, torch, reps=4 if args.no_graph else 30)
    extras = {}
    if world == 1 and not args.no_extras:
        extras["prefill_8b"] = time_prefill(b2, torch)
        extras["decode_8b_batch32"] = time_batch_decode(b2, torch)
        extras.update(other_configs(b2, torch))
    peak, peak_kind = measured_peak()
    achieved = algo / (kms * 1e-3) / 1e9
    traffics = load_traffic()
    bytes_step = step_bytes(pos_timed - args.steps // 2, args.batch, dict(SHAPE, n_layers=args.layers))
    gemv_line = {"kernel": f"gemv_q4 gate/up {2 * SHAPE['d_ff']}x{SHAPE['d_model']} (RMSNorm+SwiGLU fused), "
                           "standalone launches",
                 "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                 "traffic": traffics.get(f"gemv_q4_gateup_{2 * SHAPE['d_ff']}x{SHAPE['d_model']}"),
                 "algorithmic_bytes": algo, "launch_ms": kms}
    if persistent:
        # the step is one launch of the decode kernel: its algorithmic bytes are the step's
        step_achieved = bytes_step / (ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": "decode_kernel (whole step, one launch)", "achieved": step_achieved,
                    "peak": peak, "unit": "GB/s", "frac": step_achieved / peak, "peak_kind": peak_kind,
                    "traffic": traffics.get("decode_kernel_8b_step"), "algorithmic_bytes": bytes_step,
                    "launch_ms": ms, "gemv": gemv_line}
    else:
        roofline = dict(gemv_line, bound="hbm", peak_kind=peak_kind)
    out = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            r = reference_cpu_sample(ctx)
            cpu = {"value": r["value"], "unit": "tokens/s", "cores": r["cores"], "kind": "reference",
                   "sample": r["sample"], "extrapolated": True}
        value = args.batch * 1000.0 / ms * (world if args.replicas else 1)
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak" if args.replicas else "strong", "vs_baseline": None, "dtype": "q4xf32",
            "data": (f"synthetic (seeded N(0,0.02) weights quantised on device; random {args.prompt}-token prompt"
                     + ("; context reached by seeking)" if args.seek_fill else ")")),
            "config": {"workload": WORKLOAD, "global_batch": args.batch * (world if args.replicas else 1),
                       "seq_len": ctx, "context_at_timed_steps": pos_timed,
                       "parallelism": (f"replicas{world}" if args.replicas else f"tp{world}"),
                       "tp_exchange": None if world == 1 or args.replicas else args.tp_exchange,
                       "step_launch": "one persistent kernel" if persistent else "kernel sequence (CUDA graph)",
                       "l2": f"inputs larger than L2 ({bytes_step / 1e9:.1f} GB streamed per step)",
                       "step_bytes": bytes_step,
                       "step_hbm_frac": bytes_step / (ms * 1e-3) / (peak * 1e9 * (1 if args.replicas else world))},
            "e2e": {"value": args.batch * 1000.0 / e2e_ms * (world if args.replicas else 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * args.batch, "d2h_bytes_per_step": 4 * args.batch + 4},
            "gpu_launches": args.steps * (1 if persistent else (graph_ops or 3 + 5 * args.layers)),
            "roofline": roofline,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "extras": extras,
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return out


def run_reference(args, rank):
    """The reference CPU arm: the ATT-1 decode compiled from its sources,
    timed on this host on a bounded sample of the 8B workload (the full
    model decodes at seconds per token on the CPU) and extrapolated; the
    steps reported are the steps timed on each sample model."""
    if rank != 0:
        return None
    steps = max(1, args.steps)
    r = reference_cpu_sample(args.ctx, steps=steps, warmup=max(0, args.warmup))
    v = r["value"]
    single = reference_single_core_rows(args.ctx) if not args.no_cpu else []
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": 1000.0 / v, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4xf32", "data": "synthetic",
        "extrapolated": True,
        "timed_region_s": r["timed_region_s"],
        "config": {"workload": "llama3-8b-shape q4 decode", "global_batch": 1, "seq_len": args.ctx,
                   "parallelism": "cpu", "sample": "1- and 2-layer full-width models, lm_head 4096 rows; "
                   "steps are timed on each and extrapolated to 32 layers and 128256 rows"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": r["cores"], "kind": "reference",
                         "sample": r["sample"], "extrapolated": True, "single_core": single},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true", help="skip the reference CPU baseline leg")
    ap.add_argument("--shape", default="8b", choices=["8b", "70b"],
                    help="70b: the Llama-70B-shaped workload (batch 64, context 8192, tensor parallel over the "
                         "launched ranks, context reached by seeking, no CPU leg or side measurements)")
    ap.add_argument("--no-extras", action="store_true", help="skip the prefill and batch-32 side measurements")
    ap.add_argument("--seek-fill", action="store_true",
                    help="reach the timed context by seeking instead of decoding (short runs, e.g. under ncu)")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch kernels one by one without graph or PDL (for ncu launch lists)")
    ap.add_argument("--tp-exchange", default="fused", choices=["fused", "nccl"],
                    help="tensor parallel: partial sums exchanged by the step's kernels over peer memory (fused, "
                         "the default) or by NCCL all-reduce / all-gather (the comparison arm)")
    ap.add_argument("--replicas", action="store_true",
                    help="with several GPUs: independent replicas instead of one tensor-parallel model")
    ap.add_argument("--persistent", action="store_true",
                    help="run each step as one persistent launch instead of the per-operation kernel sequence")
    ap.add_argument("--kernel-only", nargs="?", const="gemv", choices=["gemv", "attn", "gemm"],
                    help="time only one kernel and print it (for ncu captures): the gate/up GEMV (default), the "
                         "attention at context 4096, or the tcgen05 GEMM at the gate/up shape for --batch rows")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder depth (profiling and functional runs only; the metric is defined at the shape's "
                         "depth: 32 for 8b, 80 for 70b)")
    args = ap.parse_args()
    if args.shape == "70b":
        global METRIC, WORKLOAD
        SHAPE.update(SHAPE_70B)
        METRIC, WORKLOAD = METRIC_70B, "llama-70b-shape q4 decode"
        args.batch, args.ctx, args.prompt = 64, 8192, 8
        args.seek_fill, args.no_cpu, args.no_extras = True, True, True
    if args.layers is None:
        args.layers = SHAPE["n_layers"]
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    args.replicas = args.replicas and world > 1
    if args.kernel_only:
        import torch
        import att1_b200 as b2
        torch.cuda.set_device(local_rank)
        if args.kernel_only == "gemm":
            r = time_gemm(b2, torch, m=args.batch, reps=args.steps)
            print(json.dumps(dict(r, kernel="att1_qgemm_kernel q4 gate/up 28672x4096")), flush=True)
            return
        if args.kernel_only == "attn":
            algo, kms = time_attention(b2, torch, reps=args.steps)
            name = "attention 8B shape, context 4096 (32 query / 8 KV heads, hd 128)"
        else:
            algo, kms = time_dominant_gemv(b2, torch, reps=args.steps)
            name = "gemv_q4 gate/up 28672x4096"
        print(json.dumps({"kernel": name, "launch_ms": kms,
                          "algorithmic_bytes": algo, "GB/s": algo / (kms * 1e-3) / 1e9}), flush=True)
        return
    out = run_reference(args, rank) if args.impl == "reference" else run_b200(args, rank, world, local_rank)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
