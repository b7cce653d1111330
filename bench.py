#!/usr/bin/env python
"""bench.py — CQ LUT GEMV HBM GB/s on B200 (BASELINE.json's metric).

Workload (configs[1], the mixed 2/4-bit sweep): batch-1 GEMVs on packed CQ
matrices, group 32, {512x512, 512 out x 2048 in, 2048x512, 16384x512} x
{2-bit, 4-bit}, 1000 calls each. One step runs all 8 x 1000 calls. Each
call reads its own weights: the calls cycle through distinct copies that
total >= 4x the L2 size per shape, so the weights stream from HBM (inputs
larger than L2; no flush needed). The 1000 calls of a shape share their
input x and run as cq.GEMMs (internal/cq/kernel.go:134) through the C ABI,
captured once in a CUDA graph and replayed per step.

value = algorithmic bytes of all calls (B = Out*RowBytes +
2*Out*Groups + 4*In + 4*Out + 4*2^bits per GEMV) / device time, summed over
ranks (weak scaling: every rank runs the full sweep on its own GPU).

`--impl reference` times the reference's algorithm on the host cores (the
oracle's C restatement of the lut kernel with the reference's work split;
the reference is Go and cannot be built in this image).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

GROUP = 32
# (out, in, bits)
SWEEP = [(512, 512, 2), (512, 512, 4), (512, 2048, 2), (512, 2048, 4), (2048, 512, 2), (2048, 512, 4),
         (16384, 512, 2), (16384, 512, 4)]
METRIC = "CQ LUT GEMV HBM GB/s"
UNIT = "GB/s"
WORKLOAD = "configs[1]: CQ LUT GEMV sweep, batch 1, G32, {512x512, 512x2048(in), 2048x512, 16384x512} x {2,4}-bit"


def gemv_bytes(out, in_, bits, group=GROUP):
    groups = (in_ + group - 1) // group
    return out * groups * group * bits // 8 + 2 * out * groups + 4 * in_ + 4 * out + 4 * (1 << bits)


def weight_bytes(out, in_, bits, group=GROUP):
    groups = (in_ + group - 1) // group
    return out * groups * group * bits // 8 + 2 * out * groups


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ----------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi samples of this GPU's clocks during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 7]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                smax = float(r[1])
            except ValueError:
                continue
            for name, v in zip(names, r[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------- reference ----

def run_reference(args, world, rank):
    """The reference's lut path on the host cores (oracle port), same metric."""
    if rank != 0:
        return
    import oracle

    pkg = __import__("importlib").import_module("go-whistle_b200")
    oracle.build()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1001)
    preps = []
    for out, in_, bits in SWEEP:
        p = pkg.synth.random_packed(rng, out, in_, GROUP, bits)
        om = oracle.OracleMatrix.of(p)
        preps.append((oracle.PreparedLUT(om), om, rng.normal(size=in_).astype(np.float32),
                      np.zeros(out, np.float32), gemv_bytes(out, in_, bits)))
    # The GPU line's weighting: the same number of calls of every shape
    # (args.calls, 1000), so the two arms time the same mix of bytes.
    reps = [args.calls] * len(preps)

    def step():
        for (prep, om, x, y, b), r in zip(preps, reps):
            for _ in range(r):
                prep.gemm(x, 1, y, threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    total = sum(b * r for (_, _, _, _, b), r in zip(preps, reps)) * args.steps
    value = total / dt / 1e9
    # Per shape, for ratios against the GPU line's per_shape figures.
    per_shape = {}
    for (prep, om, x, y, b), (out, in_, bits) in zip(preps, SWEEP):
        t0 = time.perf_counter()
        for _ in range(args.calls // 4):
            prep.gemm(x, 1, y, threads)
        per_shape[f"{out}x{in_}/{bits}b"] = round(b * (args.calls // 4) / (time.perf_counter() - t0) / 1e9, 3)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 index, int32 sums, f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "calls_per_shape": args.calls, "group": GROUP,
                                        "per_shape_gbs": per_shape},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{args.calls} GEMV calls of each of the 8 sweep shapes per step (the GPU line's "
                                   f"mix), one matrix per shape (cache-warm, as the reference's own benchmarks run), "
                                   f"the reference's amd64 lut path restated in C (oracle/: AVX2 lookup, tables and "
                                   f"FWHT of lut_amd64.s) with its work split on a persistent thread pool"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_decode:
        line["decode"] = decode_cpu_baseline(pkg)
    print(json.dumps(line), flush=True)


def cpu_baseline(seconds_per_shape=0.6, one_core_seconds=0.25):
    """Bounded CPU sample: the oracle's lut path (reference split) on all
    cores, and on one core, with the GPU line's weighting (equal calls of
    every shape: each shape's time per call measured, the sweep's GB/s
    formed from them)."""
    import oracle

    pkg = __import__("importlib").import_module("go-whistle_b200")
    oracle.build()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1002)
    res = {}
    for nthr, secs in ((threads, seconds_per_shape), (1, one_core_seconds)):
        total_b, total_t, calls = 0, 0.0, 0
        for out, in_, bits in SWEEP:
            p = pkg.synth.random_packed(rng, out, in_, GROUP, bits)
            prep = oracle.PreparedLUT(oracle.OracleMatrix.of(p))
            x = rng.normal(size=in_).astype(np.float32)
            y = np.zeros(out, np.float32)
            prep.gemm(x, 1, y, nthr)
            t0 = time.perf_counter()
            n = 0
            while True:
                prep.gemm(x, 1, y, nthr)
                n += 1
                dt = time.perf_counter() - t0
                if dt >= secs and n >= 3:
                    break
            total_b += gemv_bytes(out, in_, bits)  # one call of each shape
            total_t += dt / n
            calls += n
        res[nthr] = (total_b / total_t / 1e9, calls)
    return {"value": round(res[threads][0], 3), "unit": UNIT, "cores": threads, "kind": "port",
            "one_core": round(res[1][0], 3), "cpu_model": cpu_model(),
            "sample": f"{res[threads][1]} GEMV calls over the 8 sweep shapes (~{seconds_per_shape}s each; "
                      f"{res[1][1]} more on one core), one matrix per shape (cache-warm), weighted as the GPU line "
                      f"(equal calls of every shape); the reference's amd64 lut path restated in C (AVX2 lookup, "
                      f"tables and FWHT of lut_amd64.s) with its work split on a persistent thread pool"}


# ------------------------------------------------------------------ b200 ----

class Shape:
    """One sweep shape: distinct weight copies as Rows views of one matrix."""

    def __init__(self, pkg, torch, out, in_, bits, calls, l2_bytes, rng):
        self.out, self.in_, self.bits, self.calls = out, in_, bits, calls
        wb = weight_bytes(out, in_, bits)
        self.copies = min(calls, max(1, math.ceil(4 * l2_bytes / wb)))
        groups = (in_ + GROUP - 1) // GROUP
        row_bytes = groups * GROUP * bits // 8
        rows = self.copies * out
        base = rng.integers(0, 256, size=min(rows * row_bytes, 1 << 26), dtype=np.uint8)
        index = np.resize(base, rows * row_bytes)
        norms = np.resize(pkg.synth.random_norms16(rng, min(rows * groups, 1 << 22)).astype("<u2").view(np.uint8),
                          2 * rows * groups)
        cb = np.sort(rng.normal(0.0, 0.02, size=1 << bits)).astype(np.float32)
        p = pkg.cq.Packed(Out=rows, In=in_, Group=GROUP, Bits=bits, Width=bits, Codebook=cb, Index=index,
                          Norms=norms)
        self.big = pkg.cq.New(p)
        del index, norms, base
        self.views = [self.big.Rows(k * out, (k + 1) * out) for k in range(self.copies)]
        self.handles = (ctypes.c_void_p * calls)(*[self.views[c % self.copies].handle.value for c in range(calls)])
        self.hot = (ctypes.c_void_p * calls)(*[self.views[0].handle.value] * calls)
        self.x = torch.randn(in_, device="cuda", dtype=torch.float32)
        self.y = torch.empty(calls, out, device="cuda", dtype=torch.float32)
        self.ys = (ctypes.c_void_p * calls)(*[self.y.data_ptr() + 4 * out * c for c in range(calls)])
        self.bytes = calls * gemv_bytes(out, in_, bits)
        self.x_host = torch.empty(in_, dtype=torch.float32).pin_memory()
        self.x_host.copy_(self.x.cpu())
        self.y_host = torch.empty(calls, out, dtype=torch.float32).pin_memory()
        self.ys_host = (ctypes.c_void_p * calls)(*[self.y_host.data_ptr() + 4 * out * c for c in range(calls)])
        self.y_lens = (ctypes.c_size_t * calls)(*[out] * calls)

    def run_host(self, lib):
        st = lib.wc_cq_gemms_host(self.handles, self.calls, ctypes.c_void_p(self.x_host.data_ptr()), self.in_,
                                  self.ys_host, self.y_lens, 1)
        if st != 0:
            raise RuntimeError(self._err())

    def run(self, lib, stream, hot=False):
        st = lib.wc_cq_gemms(self.hot if hot else self.handles, self.calls, ctypes.c_void_p(self.x.data_ptr()),
                             self.ys, 1, stream)
        if st != 0:
            raise RuntimeError(self._err())

    def _err(self):
        pkg = __import__("importlib").import_module("go-whistle_b200")
        return pkg._lib.last_error()


def attention_component(pkg, torch, lib, stream, streams=256, layers=8, reps=5, flags=3):
    """one decode step's int8 attention for `streams` streams over
    `layers` layers, each layer with its own caches (self: 8 query heads over
    2 KV heads, qk 48, v 64, 224 positions; cross: 8 heads over 375 frames),
    as two wc_attend_int8_streams launches per layer, in a CUDA graph."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(3000)
    geo = {"self": (8, 2, 48, 64, 224), "cross": (8, 8, 48, 64, 375)}
    bufs, algo = [], 0
    for _layer in range(layers):
        for name, (heads, kvh, qk, vd, cap) in geo.items():
            k8 = torch.randint(-127, 128, (streams * cap * kvh * qk,), dtype=torch.int8, device=dev)
            v8 = torch.randint(-127, 128, (streams * cap * kvh * vd,), dtype=torch.int8, device=dev)
            ks = torch.empty(streams * cap * kvh, device=dev).uniform_(0.01, 0.05)
            vs = torch.empty(streams * cap * kvh, device=dev).uniform_(0.01, 0.05)
            q = torch.randn(streams * heads * qk, device=dev)
            nk = torch.full((streams,), cap, dtype=torch.int32, device=dev)
            out = torch.empty(streams * heads * vd, device=dev)
            bufs.append((name, heads, kvh, qk, vd, cap, q, k8, ks, v8, vs, nk, out))
            algo += streams * (cap * kvh * (qk + vd) + cap * kvh * 8 + heads * qk * 4 + heads * vd * 4)
    P = lambda t: ctypes.c_void_p(t.data_ptr())

    def step():
        for (name, heads, kvh, qk, vd, cap, q, k8, ks, v8, vs, nk, out) in bufs:
            st = lib.wc_attend_int8_streams(streams, P(q), heads, P(k8), P(ks), P(v8), P(vs), cap, P(nk), kvh, qk,
                                            vd, float(np.sqrt(qk)), flags, P(out), stream)
            if st != 0:
                raise RuntimeError(pkg._lib.last_error())

    s = torch.cuda.Stream()
    sptr = ctypes.c_void_p(s.cuda_stream)
    stream = sptr
    with torch.cuda.stream(s):
        step()
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="relaxed"):
            step()
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    mode = "any-order float sums (1e-5 rel)" if flags & 2 else "exact reference order"
    return {"workload": f"configs[3]: {streams} streams x {layers} layers, self 8/2 heads qk48 v64 x224 + "
                        f"cross 8 heads x375 frames, int8 KV, quant_q, {mode}",
            "gbs": round(algo / (ms / 1e3) / 1e9, 1), "us_per_decode_step": round(ms * 1e3, 2),
            "attention_tokens_per_s": round(streams / (ms / 1e3), 1), "algorithmic_bytes": algo,
            "launches": 2 * layers}


def exact_rows(m) -> np.ndarray:
    """The matrix's exact float32 rows (matrix.go:161 Row), as float64."""
    w = np.empty((m.Out(), m.In()), np.float32)
    for r in range(m.Out()):
        m.Row(w[r], r)
    return w.astype(np.float64)


def check_sample(torch, x, pairs, rows=8, seed=0):
    """A sample of a product's output rows against the float64 product with
    the exact weights: the reference's accept, cosine >= 0.99999 per row
    (internal/cq/cq_test.go:196-254). pairs: (exact weights, output tensor).
    Raises if a sampled row falls short; returns the smallest cosine."""
    n = x.shape[0]
    pick = np.random.default_rng(seed).choice(n, size=min(rows, n), replace=False)
    xs = x[torch.from_numpy(pick).to(x.device)].double().cpu().numpy()
    worst = 1.0
    for w, y in pairs:
        want = xs @ w.T
        got = y[torch.from_numpy(pick).to(y.device)].double().cpu().numpy()
        cos = np.sum(got * want, axis=1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
        worst = min(worst, float(cos.min()))
    if not worst >= 0.99999:
        raise RuntimeError(f"sampled output rows fall short of cosine 0.99999: {worst}")
    return worst


def prefill_component(pkg, torch, lib, frames=24000, reps=5):
    """encoder prefill GEMMs, X = 64 streams x 375 frames = 24,000
    rows x 512 fp32 ~N(0,1) times 4-bit G32 CQ weights 512->2048 (up),
    2048->512 (down), 512->1536 (QKV), and Whistle's qkvg set (384+96+128+512
    rows x 512, 2-bit G128) as one more point, on the tensor cores
    (wc_cq_gemm_ex, WC_GEMM_TENSOR_CORES), each in a CUDA graph."""
    rng = np.random.default_rng(2000)
    peaks_gbs, _ = peaks()
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tflops_peak = float(pk.get("bf16_tflops", 1590.0))
    shapes = [("up 512->2048 CQ4 G32", 2048, 512, 32, 4), ("down 2048->512 CQ4 G32", 512, 2048, 32, 4),
              ("qkv 512->1536 CQ4 G32", 1536, 512, 32, 4), ("whistle qkvg 1120x512 CQ2 G128", 1120, 512, 128, 2)]
    res = {}
    st = torch.cuda.Stream()
    sptr = ctypes.c_void_p(st.cuda_stream)
    for name, out, in_, group, bits in shapes:
        p = pkg.synth.random_packed(rng, out, in_, group, bits)
        m = pkg.cq.New(p)
        pkg._lib.check(lib.wc_cq_prepare_tc(m.handle))
        x = torch.randn(frames, in_, device="cuda", dtype=torch.float32)
        y = torch.empty(frames, out, device="cuda", dtype=torch.float32)
        args = (m.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), frames, 1, sptr)
        with torch.cuda.stream(st):
            pkg._lib.check(lib.wc_cq_gemm_ex(*args))
            st.synchronize()
            cos = check_sample(torch, x, [(exact_rows(m), y)])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
                pkg._lib.check(lib.wc_cq_gemm_ex(*args))
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                g.replay()
            e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        del g
        groups = (in_ + group - 1) // group
        wbytes = out * groups * group * bits // 8 + 2 * out * groups
        algo = wbytes + 4 * frames * in_ + 4 * frames * out
        flops = 2.0 * frames * out * in_
        t_roof = max(algo / (peaks_gbs * 1e9), flops / (tflops_peak * 1e12))
        res[name] = {"us": round(ms * 1e3, 2), "gbs": round(algo / (ms / 1e3) / 1e9, 1),
                     "tflops": round(flops / (ms / 1e3) / 1e12, 1), "roofline_frac": round(t_roof / (ms / 1e3), 3),
                     "algorithmic_bytes": algo, "sample_min_cosine": round(cos, 8)}
    return {"workload": f"configs[2]: {frames} x in fp32 ~N(0,1) prefill rows, tensor cores (fp16 operands in the "
                        f"rotated domain, fp32 accumulate)", "per_matrix": res,
            "roofline": "max(algorithmic bytes / measured HBM, flops / measured bf16 peak)"}


ENCODER_CLIPS, ENCODER_FRAMES = 64, 375  # configs[2]: 64 streams x 375 frames = 24,000 rows


def encoder_flops_per_frame(w) -> float:
    """The stack's CQ product flops per frame (2 per multiply-add): per
    layer the φ products (24 rows x 2048), q, k, v and gate (x 512),
    out_proj, pw1 (1024 x 512) and pw2 (512 x 512)."""
    D, n = w.dim, w.lanes
    macs = (2 * n + n * n) * n * D
    macs += D * (w.heads * w.qk + w.kv_heads * w.qk + w.kv_heads * w.vd + w.heads * w.vd)
    macs += w.heads * w.vd * D + 2 * D * D + D * D
    return 2.0 * macs * len(w.layers)


def encoder_component(pkg, torch, lib, clips=ENCODER_CLIPS, frames=ENCODER_FRAMES, reps=3):
    """f2: the encoder stack (wc_encoder_stack: encoder.go:167 Stack, 8
    mHC-wrapped macaron blocks and the final norm) over configs[2]'s 64
    clips x 375 frames of synthetic stem output ~N(0, 1), synthetic
    Whistle-shaped weights. Two modes: the production one (products on the
    tensor cores, attention in any order) and the exact one (lut products,
    the attention's exact order). Each checks one clip against the CPU
    restatement before timing."""
    import oracle

    w = pkg.synth.EncoderWeights(seed=5300, layers=8)
    oe = oracle.OracleEncoder(w)
    x = pkg.synth.stem_output(np.random.default_rng(5301), clips, frames)
    dx = torch.from_numpy(x).cuda()
    want_f = oe.stack(x[:1], oracle.ENC_ATTEND_FLOAT)[0]
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tflops_peak = float(pk.get("bf16_tflops", 1590.0))
    flops = encoder_flops_per_frame(w) * clips * frames
    res = {}
    for name, flags in (("tensor cores, attention any order", 3), ("lut products, attention exact order", 0)):
        enc = pkg.encoder.Encoder(w, max_clips=clips, max_frames=frames, flags=flags)
        out = enc.Stack(dx)
        torch.cuda.synchronize()
        got = out[0].cpu().numpy()
        cos = float(((got * want_f).sum(-1) / np.linalg.norm(got, axis=-1) / np.linalg.norm(want_f, axis=-1)).min())
        if not cos >= 0.99999:
            raise RuntimeError(f"encoder ({name}): clip 0 falls short of cosine 0.99999 against the oracle: {cos}")
        n0 = lib.wc_launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            enc.Stack(dx, out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms_per_stack": round(ms, 3), "frames_per_s": round(clips * frames / (ms / 1e3)),
                     "clips_per_s": round(clips / (ms / 1e3), 1), "launches_per_stack": (lib.wc_launch_count() - n0)
                     // reps, "product_tflops": round(flops / (ms / 1e3) / 1e12, 1),
                     "products_at_peak_ms": round(flops / (tflops_peak * 1e12) * 1e3, 3),
                     "clip0_min_cosine_vs_reference_form": round(cos, 8)}
        del enc
    # The whole encoder (encoder.go:108 Embed): 30 s of 16 kHz audio per
    # clip through the log-mel front end, the conv stem and the stack.
    from oracle import frontend as fe

    n = frames * 8 * 160
    audio = pkg.synth.audio(np.random.default_rng(5302), clips, n)
    daudio = torch.from_numpy(audio).cuda()
    want_e = oe.stack(fe.stem(fe.logmel(audio[0], w.mel_filters), w, oracle), oracle.ENC_ATTEND_FLOAT)
    enc = pkg.encoder.Encoder(w, max_clips=clips, max_frames=frames, flags=3)
    out = enc.Embed(daudio)
    torch.cuda.synchronize()
    got = out[0].cpu().numpy()
    cos = float(((got * want_e).sum(-1) / np.linalg.norm(got, axis=-1) / np.linalg.norm(want_e, axis=-1)).min())
    if not cos >= 0.99999:
        raise RuntimeError(f"encoder embed: clip 0 falls short of cosine 0.99999 against the oracle: {cos}")
    parts = {}
    mel = torch.empty(clips, n // 160, 80, device="cuda")
    xs = torch.empty(clips, frames, w.dim, device="cuda")
    for part, call in (("logmel", lambda: enc.LogMel(daudio, mel)), ("stem", lambda: enc.Stem(mel, xs)),
                       ("embed", lambda: enc.Embed(daudio, out))):
        call()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            call()
        e1.record()
        torch.cuda.synchronize()
        parts[part] = round(e0.elapsed_time(e1) / reps, 3)
    res["embed: front end + stem + stack, tensor cores, attention any order"] = {
        "ms_per_embed": parts["embed"], "ms_logmel": parts["logmel"], "ms_stem": parts["stem"],
        "audio_seconds_per_s": round(clips * n / 16000 / (parts["embed"] / 1e3)),
        "clips_per_s": round(clips / (parts["embed"] / 1e3), 1), "clip0_min_cosine_vs_reference_form": round(cos, 8)}
    del enc
    return {"workload": f"configs[2]: encoder (8 layers, width 512, 4 mHC lanes, int8 attention over each clip's "
                        f"frames) on {clips} clips x {frames} frames: the stack on synthetic stem output, and "
                        f"Embed on {clips} clips of {n // 16000} s of synthetic 16 kHz audio",
            "data": "synthetic weights (Whistle's shapes, a triangular mel bank) and inputs", "per_mode": res,
            "product_flops": flops, "cpu_baseline": encoder_cpu_baseline(pkg)}


def transcribe_component(pkg, torch, lib, clips=64, check_clips=4, max_tok=None):
    """The full synthetic forward, whistle.Transcribe's greedy path: 30 s of
    16 kHz audio per clip through the device encoder (encoder.go:108 Embed:
    front end, stem, stack on the tensor cores with any-order attention)
    and the device decoder (decoder.go:157 Memory, greedy.go:40
    GreedyMemory on the bit-exact lut kernels), one stream per clip; timed
    from the samples in HBM to the tokens in HBM. Before that, check_clips
    clips run with every product on the lut kernels and the attention in
    its exact order, and their tokens are compared with the CPU
    restatement's whole chain (the reference's float attention in the
    encoder)."""
    import oracle
    from oracle import frontend as fe

    max_tok = max_tok or DECODE_TOKENS
    S_ = pkg.synth
    dw = S_.DecoderWeights(seed=4000, vocab=DECODE_VOCAB)
    ew = S_.EncoderWeights(seed=5300)
    n = ENCODER_FRAMES * 8 * 160
    audio = S_.audio(np.random.default_rng(5304), clips, n)
    da = torch.from_numpy(audio).cuda()
    args = (S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, max_tok)

    enc_x = pkg.encoder.Encoder(ew, max_clips=check_clips, max_frames=ENCODER_FRAMES)
    dec_x = pkg.decoder.Decoder(dw, max_streams=check_clips, max_frames=ENCODER_FRAMES, max_positions=max_tok + 1)
    dec_x.Memory(enc_x.Embed(da[:check_clips].contiguous()))
    tok, cnt, lang, _ = (t.cpu().numpy() for t in dec_x.GreedyMemory(*args))
    del enc_x, dec_x
    oe, od = oracle.OracleEncoder(ew), oracle.OracleDecoder(dw)
    xs = np.stack([fe.stem(fe.logmel(a, ew.mel_filters), ew, oracle) for a in audio[:check_clips]])
    enc_o = oe.stack(xs, oracle.ENC_ATTEND_FLOAT, threads=check_clips)
    otok, ocnt, olang, _ = od.greedy_streams(enc_o, *args, threads=check_clips)
    same = sum(int(lang[b] == olang[b] and cnt[b] == ocnt[b] and np.array_equal(tok[b], otok[b, :max_tok - 1]))
               for b in range(check_clips))

    enc = pkg.encoder.Encoder(ew, max_clips=clips, max_frames=ENCODER_FRAMES,
                              flags=pkg.encoder.WC_ENCODER_TENSOR_CORES | pkg.encoder.WC_ENCODER_ANY_ORDER)
    dec = pkg.decoder.Decoder(dw, max_streams=clips, max_frames=ENCODER_FRAMES, max_positions=max_tok + 1)
    out = torch.empty(clips, ENCODER_FRAMES, ew.dim, device="cuda")

    def run():
        enc.Embed(da, out)
        dec.Memory(out)
        return dec.GreedyMemory(*args)

    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    _, cnt, _, eh = run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    ntok = int(clips + cnt.sum().item() + eh.sum().item())
    return {"workload": f"{clips} clips of {n // 16000} s of synthetic 16 kHz audio -> encoder (tensor cores, any-order "
                        f"attention) -> decoder (lut kernels), greedy {max_tok} tokens per clip (language + text)",
            "ms": round(ms, 2), "audio_seconds_per_s": round(clips * n / 16000 / (ms / 1e3)),
            "tokens_per_s": round(ntok / (ms / 1e3)), "tokens": ntok,
            "exact_chain_vs_cpu_restatement": f"{same} of {check_clips} clips with the CPU restatement's tokens "
                                              f"(lut products, exact attention order on the device)"}


def single_call_component(pkg, torch, lib, calls=20, reps=10):
    """Batch-1 latency: one GEMV call at a time (configs[0]'s 2048 x 512
    CQ4 G32, and the 16384 x 512 CQ4 vocabulary head), `calls` calls in a row
    captured in a CUDA graph; hot = the same weights each call (L2-resident,
    as a decode loop's weights are), cold = a distinct copy per call."""
    rng = np.random.default_rng(5000)
    st = torch.cuda.Stream()
    sptr = ctypes.c_void_p(st.cuda_stream)
    res = {}
    for name, out, in_, group, bits in (("configs[0] 2048x512 CQ4 G32", 2048, 512, 32, 4),
                                        ("head 16384x512 CQ4 G32", 16384, 512, 32, 4)):
        mats = [pkg.cq.New(pkg.synth.random_packed(rng, out, in_, group, bits)) for _ in range(calls)]
        x = torch.randn(in_, device="cuda", dtype=torch.float32)
        y = torch.empty(out, device="cuda", dtype=torch.float32)
        row = {}
        for mode in ("hot", "cold"):
            def run():
                for i in range(calls):
                    m = mats[0] if mode == "hot" else mats[i]
                    pkg._lib.check(lib.wc_cq_gemm(m.handle, ctypes.c_void_p(x.data_ptr()),
                                                  ctypes.c_void_p(y.data_ptr()), 1, sptr))

            with torch.cuda.stream(st):
                run()
                st.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
                    run()
                g.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(reps):
                    g.replay()
                e1.record(st)
            torch.cuda.synchronize()
            row[f"us_per_call_{mode}"] = round(e0.elapsed_time(e1) * 1e3 / (reps * calls), 2)
            del g
        row["algorithmic_bytes"] = pkg.synth.algorithmic_bytes_gemv(out, in_, group, bits)
        res[name] = row
    return {"workload": "batch-1 GEMV latency, calls back to back in a CUDA graph (launch gaps included)",
            "per_shape": res}


def decode_gemm_component(pkg, torch, lib, streams=256, reps=20):
    """Multi-stream decode GEMMs: `streams` activation rows (one per stream)
    through Whistle's self-attention projections (q 384, k 96, v 128, gate
    512 from x 512; CQ2 G128, one GEMMs call) and the 16384 x 512 CQ4 G32
    vocabulary head, with WC_GEMM_AUTO (tensor cores at this batch), each
    call captured in a CUDA graph; and the head followed by the greedy step's
    argmax (wc_head_argmax: one token id per stream)."""
    rng = np.random.default_rng(4000)
    peaks_gbs, _ = peaks()
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    tflops_peak = float(pk.get("bf16_tflops", 1590.0))
    sets = [("qkvg 384+96+128+512 x512 CQ2 G128", [384, 96, 128, 512], 512, 128, 2, False),
            ("head 16384x512 CQ4 G32", [16384], 512, 32, 4, False),
            ("head 16384x512 CQ4 G32 + argmax", [16384], 512, 32, 4, True)]
    st = torch.cuda.Stream()
    sptr = ctypes.c_void_p(st.cuda_stream)
    res = {}
    for name, outs, in_, group, bits, argmax in sets:
        ps, ms = [], []
        for o in outs:
            p = pkg.synth.random_packed(rng, o, in_, group, bits)
            if ps:
                p.Codebook = ps[0].Codebook
            ps.append(p)
            ms.append(pkg.cq.New(p))
            pkg._lib.check(lib.wc_cq_prepare_tc(ms[-1].handle))
        x = torch.randn(streams, in_, device="cuda", dtype=torch.float32)
        ys = [torch.empty(streams, o, device="cuda", dtype=torch.float32) for o in outs]
        hs = (ctypes.c_void_p * len(ms))(*[m.handle.value for m in ms])
        yp = (ctypes.c_void_p * len(ms))(*[y.data_ptr() for y in ys])
        idx = torch.empty(streams, device="cuda", dtype=torch.int32)
        n0 = lib.wc_launch_count()

        def call():
            pkg._lib.check(lib.wc_cq_gemms_ex(hs, len(ms), ctypes.c_void_p(x.data_ptr()), yp, streams, 2, sptr))
            if argmax:
                pkg._lib.check(lib.wc_head_argmax(ctypes.c_void_p(ys[0].data_ptr()), streams, outs[0], 1.0, None,
                                                  ctypes.c_void_p(idx.data_ptr()), sptr))

        with torch.cuda.stream(st):
            call()
            st.synchronize()
            launches = lib.wc_launch_count() - n0
            cos = check_sample(torch, x, [(exact_rows(m), y) for m, y in zip(ms, ys)])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
                call()
            g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(reps):
                g.replay()
            e1.record(st)
        torch.cuda.synchronize()
        ms_call = e0.elapsed_time(e1) / reps
        del g
        algo = sum(pkg.synth.algorithmic_bytes_gemv(o, in_, group, bits) - 4 * in_ - 4 * o for o in outs)
        algo += 4 * streams * in_ + 4 * streams * sum(outs) + (4 * streams if argmax else 0)
        flops = 2.0 * streams * in_ * sum(outs)
        t_roof = max(algo / (peaks_gbs * 1e9), flops / (tflops_peak * 1e12))
        res[name] = {"us": round(ms_call * 1e3, 2), "gbs": round(algo / (ms_call / 1e3) / 1e9, 1),
                     "tflops": round(flops / (ms_call / 1e3) / 1e12, 1),
                     "roofline_frac": round(t_roof / (ms_call / 1e3), 3), "algorithmic_bytes": algo,
                     "launches": launches, "sample_min_cosine": round(cos, 8)}
    return {"workload": f"{streams} decode streams: one activation row each, WC_GEMM_AUTO (tensor cores, fp16 "
                        f"operands, fp32 accumulate)", "per_set": res,
            "roofline": "max(algorithmic bytes / measured HBM, flops / measured bf16 peak); launch-bound at "
                        "this size"}


def rows_sweep_component(pkg, torch, lib, reps=20, rows_list=(1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 256)):
    """The lut kernels against the tensor cores by activation rows: each
    row count through wc_cq_gemms_ex with flags 0 (the bit-exact lut path
    run_lut picks) and WC_GEMM_TENSOR_CORES, `reps` calls in a CUDA graph on
    the same weights (L2-warm, as a decode loop's are), µs per call. The
    crossover this shows is WC_GEMM_AUTO's row threshold."""
    rng = np.random.default_rng(4100)
    sets = [("qkvg 384+96+128+512 x512 CQ2 G128", [384, 96, 128, 512], 512, 128, 2),
            ("2048x512 CQ4 G32", [2048], 512, 32, 4),
            ("head 16384x512 CQ4 G32", [16384], 512, 32, 4)]
    st = torch.cuda.Stream()
    sptr = ctypes.c_void_p(st.cuda_stream)
    out = {}
    for name, outs, in_, group, bits in sets:
        ps, ms = [], []
        for o in outs:
            p = pkg.synth.random_packed(rng, o, in_, group, bits)
            if ps:
                p.Codebook = ps[0].Codebook
            ps.append(p)
            ms.append(pkg.cq.New(p))
            pkg._lib.check(lib.wc_cq_prepare_tc(ms[-1].handle))
        hs = (ctypes.c_void_p * len(ms))(*[m.handle.value for m in ms])
        rows_res = {}
        for rows in rows_list:
            x = torch.randn(rows, in_, device="cuda", dtype=torch.float32)
            ys = [torch.empty(rows, o, device="cuda", dtype=torch.float32) for o in outs]
            yp = (ctypes.c_void_p * len(ms))(*[y.data_ptr() for y in ys])
            point = {}
            for label, flags in (("lut", 0), ("tc", 1)):
                def call():
                    pkg._lib.check(lib.wc_cq_gemms_ex(hs, len(ms), ctypes.c_void_p(x.data_ptr()), yp, rows,
                                                      flags, sptr))

                with torch.cuda.stream(st):
                    call()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
                        for _ in range(reps):
                            call()
                    g.replay()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    g.replay()
                    g.replay()
                    e1.record(st)
                torch.cuda.synchronize()
                point[label + "_us"] = round(e0.elapsed_time(e1) * 1e3 / (2 * reps), 2)
                del g
            point["faster"] = "lut" if point["lut_us"] <= point["tc_us"] else "tc"
            rows_res[rows] = point
        out[name] = rows_res
    return {"workload": "rows sweep: lut (bit-exact) against tensor cores per call, L2-warm weights, CUDA graph of "
                        f"{reps} calls", "per_set": out}


DECODE_STREAMS = 1024   # configs[4]: streams sharded over the GPUs (stream s -> rank s mod N)
DECODE_FRAMES = 375     # 30 s of audio at 12.5 encoder frames/s
DECODE_TOKENS = 65      # the language token and 64 greedy text tokens
DECODE_VOCAB = 16384


def decode_streams_of(rank, world, total=DECODE_STREAMS):
    """The streams a rank decodes (go-whistle_b200/dp.py's shard: s mod N)."""
    return [s for s in range(total) if s % world == rank]


def decode_component(pkg, torch, lib, world, rank, pg, dev, total=DECODE_STREAMS, frames=DECODE_FRAMES,
                     max_tok=DECODE_TOKENS, flags=0, keep=None):
    """configs[4]'s decoder: greedy decoding of `total` independent streams
    of the synthetic Whistle decoder (8 layers, 4 mHC lanes, int8 self and
    cross attention over 375 frames, engram, vocab 16384), sharded over the
    ranks with no collective. Each rank projects its streams' memories
    (untimed, the prefill), then runs GreedyMemory for all of them on the
    device; tokens/s = every token the ranks decoded (the language token,
    the text tokens, the EOS that ends a stream) / the slowest rank's
    device time of the decode."""
    S_ = pkg.synth
    mine = decode_streams_of(rank, world, total)
    w = S_.DecoderWeights(seed=4000, vocab=DECODE_VOCAB)
    enc = np.stack([S_.encoder_output(np.random.default_rng(5000 + s), 1, frames)[0] for s in mine])
    denc = torch.from_numpy(enc).to(dev)
    dec = pkg.decoder.Decoder(w, max_streams=len(mine), max_frames=frames, max_positions=max_tok + 1, flags=flags)
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record(stream)
    dec.Memory(denc)
    ev[1].record(stream)
    # Warm-up run: captures the step graph.
    dec.GreedyMemory(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, 4)
    dec.Memory(denc)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    n0 = lib.wc_launch_count()
    ev[2].record(stream)
    tokens, counts, lang, eos = dec.GreedyMemory(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, max_tok)
    ev[3].record(stream)
    torch.cuda.synchronize()
    launches = lib.wc_launch_count() - n0
    ms = ev[2].elapsed_time(ev[3])
    mem_ms = ev[0].elapsed_time(ev[1])
    counts_h, eos_h = counts.cpu().numpy(), eos.cpu().numpy()
    if keep is not None:
        keep["tokens"], keep["counts"], keep["lang"] = tokens.cpu().numpy(), counts_h, lang.cpu().numpy()
    ntok = int(len(mine) + counts_h.sum() + eos_h.sum())
    if pg:
        t = torch.tensor([ms, float(ntok)], device=dev, dtype=torch.float64)
        tmax = t.clone()
        pg.all_reduce(tmax, op=pg.ReduceOp.MAX)
        pg.all_reduce(t, op=pg.ReduceOp.SUM)
        ms, ntok = float(tmax[0].item()), int(t[1].item())
    # Algorithmic bytes of one step on this rank (the decode's roofline):
    # the int8 cross memory of every layer and stream, the self caches, and
    # the CQ weights once.
    L, S = len(w.layers), len(mine)
    cross = S * L * (frames * w.x_heads * (w.x_qk + w.x_vd) + frames * w.x_heads * 2 * 4)
    ctx = max_tok / 2
    self_b = S * L * (ctx * w.kv_heads * (w.qk + w.vd) + ctx * w.kv_heads * 2 * 4)
    def wb_(p):
        return p.Index.size + p.Norms.size
    wbytes = wb_(w.embedding) + wb_(w.phi_pre) + wb_(w.phi_post) + wb_(w.phi_res) + sum(
        wb_(Ld[k]) for Ld in w.layers for k in ("q_proj", "k_proj", "v_proj", "gate_proj", "out_proj", "x_q_proj",
                                                "x_gate_proj", "x_out_proj"))
    step_bytes = cross + self_b + wbytes
    steps = max_tok
    peak, peak_kind = peaks()
    return {"workload": f"configs[4] decoder: {total} streams sharded stream mod {world}, greedy {max_tok} tokens "
                        f"(language + 64 text) per stream, synthetic Whistle decoder (8 layers, vocab {DECODE_VOCAB}, "
                        f"int8 KV, cross memory of {frames} frames), every CQ product on the bit-exact lut kernels",
            "metric": "decode tokens/s", "value": round(ntok / (ms / 1e3), 1), "unit": "tokens/s",
            "scaling": "strong", "streams_total": total, "streams_this_rank": S, "tokens": ntok,
            "ms_decode": round(ms, 3), "ms_per_step": round(ms / steps, 4), "ms_memory_prefill": round(mem_ms, 2),
            "gpu_launches_per_step": round(launches / steps, 1),
            "roofline": {"bound": "hbm", "bytes_per_step_per_rank": int(step_bytes),
                         "achieved_gbs": round(step_bytes / (ms / steps / 1e3) / 1e9, 1), "peak": peak,
                         "frac": round(step_bytes / (ms / steps / 1e3) / 1e9 / peak, 4), "peak_kind": peak_kind},
            "parity": "token ids identical to the CPU restatement (tests/test_decoder_step_gpu.py)"}


BEAM_CLIPS = 256  # clips searched at once, 5 beams each (1280 decoder streams)


def beam_component(pkg, torch, lib, clips=BEAM_CLIPS, beams=5, frames=DECODE_FRAMES, max_tok=DECODE_TOKENS,
                   cpu_clips=1):
    """Beam search (search/beam.go with options.go Default: 5 beams, Whisper's
    StopK rule) on the device decoder for `clips` clips of the synthetic
    Whistle decoder: every live hypothesis is a decoder stream, the beams of
    a clip share its cross memory, forks copy stream states on the device,
    the search's bookkeeping runs on the host each step. The EOS id the
    synthetic weights never reach keeps every search to the token limit
    (the language token and 64 text steps), the longest case. Timed by CUDA
    events on the stream around wc_decoder_beam (host gaps included); the
    CPU figure is the oracle's restatement of the same search on the same
    weights, one clip on one host thread."""
    import time

    S_ = pkg.synth
    w = S_.DecoderWeights(seed=4000, vocab=DECODE_VOCAB)
    enc = np.stack([S_.encoder_output(np.random.default_rng(7000 + c), 1, frames)[0] for c in range(clips)])
    denc = torch.from_numpy(enc).cuda()
    dec = pkg.decoder.Decoder(w, max_streams=clips * beams, max_frames=frames, max_positions=max_tok + 1)
    opts = pkg.decoder.DefaultBeam(beams=beams, max_tokens=max_tok)
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    dec.MemoryBeams(denc, beams)  # warm-up search: captures the step graph
    dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, pkg.decoder.DefaultBeam(beams=beams, max_tokens=4))
    ev[0].record(stream)
    dec.MemoryBeams(denc, beams)
    ev[1].record(stream)
    n0 = lib.wc_launch_count()
    ev[2].record(stream)
    tok, cnt, lang, eos_hit, score, _, _ = dec.Beam(S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, opts)
    ev[3].record(stream)
    torch.cuda.synchronize()
    launches = lib.wc_launch_count() - n0
    ms = ev[2].elapsed_time(ev[3])
    steps = max_tok
    hyp_tokens = clips * (1 + beams * (steps - 1))  # tokens fed to live hypotheses
    # The CPU restatement on one clip (same weights, same options).
    import oracle
    from oracle import beam as bm

    od = oracle.OracleDecoder(w)
    t0 = time.perf_counter()
    same = True
    for c in range(cpu_clips):
        st = od.state(max_tok + 1, frames)
        st.memory(enc[c])
        r = bm.search(st, S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, bm.Options(beams=beams), max_tok)
        same &= r.tokens == tok[c, :cnt[c]].tolist() and r.lang == int(lang[c])
    cpu_s = (time.perf_counter() - t0) / cpu_clips
    return {"workload": f"beam search: {clips} clips x {beams} beams (options.go Default, StopK), synthetic Whistle "
                        f"decoder (vocab {DECODE_VOCAB}, {frames} frames of cross memory shared by a clip's beams), "
                        f"{steps} positions per clip (the language token and {steps - 1} text steps)",
            "metric": "beam search clips/s", "value": round(clips / (ms / 1e3), 2), "unit": "clips/s",
            "hypothesis_tokens_per_s": round(hyp_tokens / (ms / 1e3), 1), "ms_search": round(ms, 2),
            "ms_per_step": round(ms / steps, 3), "ms_memory_prefill": round(ev[0].elapsed_time(ev[1]), 2),
            "gpu_launches": launches,
            "cpu_baseline": {"value": round(1.0 / cpu_s, 4), "unit": "clips/s", "cores": 1, "kind": "port",
                             "sample": f"{cpu_clips} clip(s) through the oracle's restatement of beam.go over its "
                                       f"decoder, one host thread"},
            "parity": "the CPU restatement's best hypothesis for the sampled clip(s): " + ("identical" if same
                                                                                          else "DIFFERENT")}


def decode_cpu_baseline(pkg, streams=16, max_tok=DECODE_TOKENS, frames=DECODE_FRAMES):
    """The decoder's CPU baseline: the oracle's restatement of the
    reference's greedy decode (internal/decoder, int8 numerics, the lut
    kernels) for a sample of streams, one stream per host thread; memories
    untimed, the decodes timed by the wall clock."""
    import oracle

    oracle.build()
    S_ = pkg.synth
    w = S_.DecoderWeights(seed=4000, vocab=DECODE_VOCAB)
    od = oracle.OracleDecoder(w)
    enc = np.stack([S_.encoder_output(np.random.default_rng(5000 + s), 1, frames)[0] for s in range(streams)])
    threads = min(streams, os.cpu_count() or 1)
    secs, tok, cnt, lang, eh = oracle.timed_greedy(od, enc, S_.WHISTLE_BOS, S_.WHISTLE_LANGS, S_.WHISTLE_EOS, max_tok,
                                                   threads)
    ntok = int(streams + cnt.sum() + eh.sum())
    return {"value": round(ntok / secs, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{streams} streams x {max_tok} greedy tokens of the same synthetic decoder, one stream per "
                      f"thread (memories untimed)", "cpu_model": cpu_model()}


def encoder_cpu_baseline(pkg, clips=16, frames=ENCODER_FRAMES):
    """The encoder stack's CPU baseline: the oracle's restatement of the
    reference's Stack (encoder.go:167, int8 numerics, the lut products,
    attendGEMM's float attention) on a sample of clips, one clip per host
    thread, timed by the wall clock."""
    import time

    import oracle

    oracle.build()
    w = pkg.synth.EncoderWeights(seed=5300, layers=8)
    oe = oracle.OracleEncoder(w)
    x = pkg.synth.stem_output(np.random.default_rng(5303), clips, frames)
    threads = min(clips, os.cpu_count() or 1)
    t0 = time.perf_counter()
    oe.stack(x, oracle.ENC_ATTEND_FLOAT, threads=threads)
    secs = time.perf_counter() - t0
    return {"value": round(clips * frames / secs), "unit": "frames/s", "cores": threads, "kind": "port",
            "sample": f"{clips} clips x {frames} frames through the 8-layer stack, one clip per thread",
            "cpu_model": cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_b200(args, world, rank, local):
    import torch

    pkg = __import__("importlib").import_module("go-whistle_b200")
    lib = pkg._lib.lib()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 1024 * 1024) or 126 * 1024 * 1024
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist

    rng = np.random.default_rng(1000 + rank)
    sweep = SWEEP
    if args.only:
        o, i, b = (int(v) for v in args.only.split("x"))
        sweep = [(o, i, b)]
    shapes = [Shape(pkg, torch, o, i, b, args.calls, l2, rng) for o, i, b in sweep]
    stream = torch.cuda.Stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    bytes_per_step = sum(s.bytes for s in shapes)

    def step():
        for s in shapes:
            s.run(lib, sptr)

    # Per-shape device GB/s for the breakdown, cold (distinct weights) and
    # hot (one weight copy, L2-resident), each shape's calls in its own CUDA
    # graph so host work stays outside the timing.
    per_shape = {}
    distinct_ms = 0.0
    with torch.cuda.stream(stream):
        for s in shapes:
            res = {}
            for hot in (False, True):
                s.run(lib, sptr, hot=hot)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
                    s.run(lib, sptr, hot=hot)
                g.replay()
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 5
                ev0.record(stream)
                for _ in range(reps):
                    g.replay()
                ev1.record(stream)
                ev1.synchronize()
                res[hot] = s.bytes * reps / (ev0.elapsed_time(ev1) / 1e3) / 1e9
                del g
            # The calls as a decode step issues them: each GEMV its own
            # launch on its own activation (wc_cq_gemm, batch 1), the
            # weights cycling through the copies, in one CUDA graph.
            if args.no_distinct:
                per_shape[f"{s.out}x{s.in_}/{s.bits}b"] = {
                    "cold_hbm_gbs": round(res[False], 1), "hot_l2_gbs": round(res[True], 1),
                    "weight_copies": s.copies,
                    "l2_multiple": round(s.copies * weight_bytes(s.out, s.in_, s.bits) / l2, 2)}
                continue
            xs = torch.randn(s.calls, s.in_, device="cuda", dtype=torch.float32)

            def run_distinct(s=s, xs=xs):
                for c in range(s.calls):
                    st = lib.wc_cq_gemm(s.handles[c], ctypes.c_void_p(xs.data_ptr() + 4 * s.in_ * c),
                                        ctypes.c_void_p(s.ys[c]), 1, sptr)
                    if st != 0:
                        raise RuntimeError(s._err())

            run_distinct()
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
                run_distinct()
            g.replay()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            for _ in range(3):
                g.replay()
            ev1.record(stream)
            ev1.synchronize()
            d_ms = ev0.elapsed_time(ev1) / 3
            distinct_ms += d_ms
            del g, xs
            per_shape[f"{s.out}x{s.in_}/{s.bits}b"] = {
                "cold_hbm_gbs": round(res[False], 1), "hot_l2_gbs": round(res[True], 1),
                "distinct_x_gbs": round(s.bytes / (d_ms / 1e3) / 1e9, 1),
                "distinct_x_us_per_call": round(d_ms * 1e3 / s.calls, 2),
                "weight_copies": s.copies,
                # Distinct weight bytes the calls cycle through, in L2 sizes:
                # below 4 the copies are capped by the 1000 calls and part of
                # the "cold" figure is L2-resident.
                "l2_multiple": round(s.copies * weight_bytes(s.out, s.in_, s.bits) / l2, 2)}

    # Capture one step in a CUDA graph.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step()  # warm the launch path before capture
        stream.synchronize()
        n0 = lib.wc_launch_count()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
            step()
        launches_per_step = lib.wc_launch_count() - n0
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local)
    sampler = ClockSampler(gpu_id)
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    if pg:
        pg.barrier()
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * bytes_per_step * args.steps / (ms / 1e3) / 1e9

    # End to end through the C ABI's host-slice call (wc_cq_gemms_host, the
    # reference's GEMMs on Go slices): x from pinned host memory in, every
    # output back to pinned host memory, each step; wall-clock time, since
    # the call is synchronous and its copies run on the library's streams.
    h2d = sum(4 * s.in_ for s in shapes)
    d2h = sum(4 * s.calls * s.out for s in shapes)
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        for s in shapes:
            s.run_host(lib)

    e2e_step()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) * 1e3
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * bytes_per_step * e2e_steps / (e2e_ms / 1e3) / 1e9

    peak, peak_kind = peaks()
    avg_launch_ms = ms_per_step / max(launches_per_step, 1)
    bytes_per_launch = bytes_per_step / max(launches_per_step, 1)
    achieved = bytes_per_launch / (avg_launch_ms / 1e3) / 1e9
    # DRAM traffic per launch from the committed ncu summary (a smaller
    # launch of the same kernel, scaled by the bytes it covers).
    traffic = None
    tf = ROOT / "profiles" / "cq_lut_stream_2048x512x4_traffic.md"
    if tf.exists():
        for line in tf.read_text().splitlines():
            if line.startswith("traffic_over_algorithmic:"):
                traffic = int(float(line.split(":")[1]) * bytes_per_launch)

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8 index, int32 table sums, f32 epilogue", "data": "synthetic",
        "config": {"workload": WORKLOAD, "calls_per_shape": args.calls, "group": GROUP,
                   "cache": "inputs larger than L2: each shape's weights cycle through distinct copies, >= 4x L2 "
                            "where the 1000 calls allow it (per_shape.l2_multiple); the step's 9.6 GB is 76x L2",
                   "launch": "cq.GEMMs over the calls of a shape (shared x), CUDA graph of one step",
                   "bytes_per_step": bytes_per_step, "parallelism": f"replicas x{world} (no collectives)",
                   "per_shape": per_shape},
        # The same step with every GEMV on its own activation, one launch a
        # call (as a decode step issues them, each waiting for the last):
        # the batch-1 latency figure, beside the shared-x `value`.
        "distinct_x": None if args.no_distinct else {"gbs": round(bytes_per_step / (distinct_ms / 1e3) / 1e9, 1),
                       "ms_per_step": round(distinct_ms, 3),
                       "launch": "wc_cq_gemm per call (batch 1, its own x), every call of a shape in one CUDA graph",
                       "scope": "rank 0's own step (per GPU)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                     "kernel": "cq_lut_stream_kernel", "bytes_per_launch": int(bytes_per_launch)},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "call": "wc_cq_gemms_host per shape (pinned host x and outputs), wall clock", "steps": e2e_steps,
                "d2h": "the kernels store the results into the page-locked host outputs over PCIe"},
        "gpu_launches": int(launches_per_step * args.steps), "gpu_launches_scope": "per rank",
        "clocks": clocks,
    }
    if not args.only and not args.no_decode:
        exact, tc = {}, {}
        line["decode"] = decode_component(pkg, torch, lib, world, rank, pg, dev, keep=exact)
        # The same decode with every CQ product on the tensor cores (fp16
        # operands within the stated bound, not the reference's lut bits):
        # its speed, and how many streams decode the same tokens.
        r = decode_component(pkg, torch, lib, world, rank, pg, dev, flags=pkg.decoder.WC_DECODER_TENSOR_CORES,
                             keep=tc)
        same = np.all(exact["tokens"] == tc["tokens"], axis=1) & (exact["counts"] == tc["counts"]) & (
            exact["lang"] == tc["lang"])
        agree = [int(same.sum()), int(same.size)]
        if pg:
            t = torch.tensor(agree, device=dev, dtype=torch.int64)
            pg.all_reduce(t, op=pg.ReduceOp.SUM)
            agree = [int(v) for v in t.tolist()]
        line["decode"]["tensor_cores"] = {
            "value": r["value"], "unit": r["unit"], "ms_per_step": r["ms_per_step"],
            "streams_with_the_exact_tokens": f"{agree[0]} of {agree[1]}",
            "numerics": "WC_DECODER_TENSOR_CORES: fp16 operands, fp32 accumulate, within the header's bound"}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            line["decode"]["cpu_baseline"] = decode_cpu_baseline(pkg)
    if args.only:
        line["config"]["workload"] = f"one shape {args.only} (profiling run, not the headline workload)"
    elif not args.no_components and world == 1:
        line["components"] = {"int8_attention": attention_component(pkg, torch, lib, None, flags=3),
                              "int8_attention_exact_order": attention_component(pkg, torch, lib, None, flags=1),
                              "cq_gemm_prefill": prefill_component(pkg, torch, lib),
                              "cq_gemm_decode_streams": decode_gemm_component(pkg, torch, lib),
                              "cq_gemv_single_call": single_call_component(pkg, torch, lib),
                              "beam_search": beam_component(pkg, torch, lib),
                              "encoder_stack": encoder_component(pkg, torch, lib)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.only:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--calls", type=int, default=1000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", default="", help="one shape OUTxINxBITS (profiling runs)")
    ap.add_argument("--no-components", action="store_true", help="skip the attention component")
    ap.add_argument("--attention-only", action="store_true", help="only the attention component (profiling)")
    ap.add_argument("--prefill-only", action="store_true", help="only the prefill GEMM component (profiling)")
    ap.add_argument("--decode-gemm-only", action="store_true", help="only the multi-stream decode GEMM component")
    ap.add_argument("--no-decode", action="store_true", help="skip the greedy decoder component")
    ap.add_argument("--decode-only", action="store_true", help="only the greedy decoder component")
    ap.add_argument("--rows-sweep", action="store_true", help="only the lut / tensor-core rows sweep")
    ap.add_argument("--beam-only", action="store_true", help="only the beam search component")
    ap.add_argument("--encoder-only", action="store_true", help="only the encoder stack component")
    ap.add_argument("--transcribe-only", action="store_true", help="only the audio-to-tokens forward (not in the default run)")
    ap.add_argument("--encoder-clips", type=int, default=ENCODER_CLIPS, help="--encoder-only: clips of 375 frames")
    ap.add_argument("--no-distinct", action="store_true",
                    help="skip the distinct-activation figure (its 8000 launches a step; profiling runs)")
    ap.add_argument("--decode-streams", type=int, default=DECODE_STREAMS, help="--decode-only: total streams")
    ap.add_argument("--decode-tokens", type=int, default=DECODE_TOKENS, help="--decode-only: tokens per stream")
    ap.add_argument("--decode-eager", action="store_true", help="--decode-only: steps as eager launches (profiling)")
    ap.add_argument("--decode-tc", action="store_true", help="--decode-only: CQ products on the tensor cores")
    args = ap.parse_args()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.prefill_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(prefill_component(pkg, torch, pkg._lib.lib())), flush=True)
        return
    if args.decode_gemm_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(decode_gemm_component(pkg, torch, pkg._lib.lib())), flush=True)
        return
    if args.encoder_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(encoder_component(pkg, torch, pkg._lib.lib(), clips=args.encoder_clips)), flush=True)
        return
    if args.transcribe_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(transcribe_component(pkg, torch, pkg._lib.lib())), flush=True)
        return
    if args.beam_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(beam_component(pkg, torch, pkg._lib.lib())), flush=True)
        return
    if args.rows_sweep:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        print(json.dumps(rows_sweep_component(pkg, torch, pkg._lib.lib())), flush=True)
        return
    if args.decode_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        pg = None
        if world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            pg = dist
        res = decode_component(pkg, torch, pkg._lib.lib(), world, rank, pg, torch.device("cuda", local),
                               total=args.decode_streams, max_tok=args.decode_tokens,
                               flags=(pkg.decoder.WC_DECODER_NO_GRAPH if args.decode_eager else 0) |
                               (pkg.decoder.WC_DECODER_TENSOR_CORES if args.decode_tc else 0))
        if rank == 0:
            print(json.dumps(res), flush=True)
        if pg:
            pg.barrier()
            pg.destroy_process_group()
        return
    if args.attention_only:
        import torch

        pkg = __import__("importlib").import_module("go-whistle_b200")
        torch.cuda.set_device(local)
        for flags in (3, 1):
            print(json.dumps(attention_component(pkg, torch, pkg._lib.lib(), None, flags=flags)), flush=True)
        return
    run_b200(args, world, rank, local)


if __name__ == "__main__":
    main()
