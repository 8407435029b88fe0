#!/usr/bin/env python
"""Headline benchmark of the GGUF K-quant linear path on B200.

Workload (the largest single-GPU configuration of
the Q4_K_M dequant-GEMM metric): the linear stack of a Z-Image-style 6B
single-stream DiT -- hidden 3840, 30 layers, per layer qkv [11520, 3840],
out [3840, 3840], w1 / w3 [10240, 3840] (SwiGLU), w2 [3840, 10240]; M = 8448
tokens (1024x1024 image: 4096 image + 128 text tokens, CFG 2).  Q4_K_M mix:
every tensor Q4_K except w2 (ffn_down), which is Q6_K in even layers.
Weights ~ N(0, 0.02), activations ~ N(0, 1) bf16, all synthetic.

A step is one pass of the hot path over the batch: every layer's qkv, out,
w1 / w3 and w2 projections (the FLOPs of 150 quantised linears), fp16
activations in and fp16 outputs out (the reference's GGUF execution runs fp16
activations, and its projection returns X's dtype).  By default
(--ffn swiglu) w1 and w3 run as one interleaved weight whose GEMM epilogue
computes the FFN's silu(w1 x) * w3 x, as the model does; --ffn separate runs
them as two plain linears without the SwiGLU.  With --gpus N each weight is
N-column sharded across the ranks (one process per GPU) and every output is
all-gathered over NVLink, by default by copy-engine peer pushes on a side
stream beside the next GEMM (--gather copy), with --gather fused inside the
GEMM epilogue (peer stores), with --gather nccl by NCCL after each GEMM.
After timing, sampled rows of the last outputs are checked against the CPU
oracle (dequant + fp64 matmul) on every rank, and at N > 1 every rank's
gathered Y is checked to equal the shards the other ranks computed.
Prints one JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q4_K_M dequant-GEMM TFLOPS (% bf16 TC peak); small-M GEMV GB/s (% HBM)"
HIDDEN, FFN, LAYERS, M_TOKENS = 3840, 10240, 30, 8448
Q4_K, Q6_K = 12, 14
DISTINCT_LAYERS = 2     # weight contents cycle over 2 seeds; every layer has its own HBM buffers


def layer_linears(layer: int):
    """(name, N, K, ggml_type) of one layer's linears in the Q4_K_M mix."""
    return [("qkv", 3 * HIDDEN, HIDDEN, Q4_K), ("out", HIDDEN, HIDDEN, Q4_K), ("w1", FFN, HIDDEN, Q4_K),
            ("w3", FFN, HIDDEN, Q4_K), ("w2", HIDDEN, FFN, Q6_K if layer % 2 == 0 else Q4_K)]


def step_flops(layers: int, m: int = M_TOKENS) -> float:
    return float(sum(2.0 * m * n * k for l in range(layers) for _, n, k, _ in layer_linears(l)))


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons of the job's GPUs every 50 ms.
    Started when the run starts (nvidia-smi needs up to a second before its
    first row, longer with several instances); stop(window) keeps the samples
    taken inside the timed region's host-time window -- or, for a region
    shorter than the sampling period, the first samples after it began --
    over every sampled GPU (median clock, union of the throttle reasons)."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = [devices] if isinstance(devices, int) else list(devices)
        self.proc, self.path = None, None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", ",".join(map(str, self.devices)),
                                          f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50", "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            import atexit
            atexit.register(self._kill)   # never outlive the bench, whatever ends it
        except OSError:
            self.proc = None

    def _kill(self):
        if self.proc and self.proc.poll() is None:
            self.proc.kill()

    @staticmethod
    def _when(stamp: str):
        import datetime
        try:
            return datetime.datetime.strptime(stamp, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self, window=None):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        os.unlink(self.path)
        if window and rows:
            t0, t1 = window
            stamped = [(self._when(r[0]), r) for r in rows]
            inside = [r for t, r in stamped if t is not None and t0 <= t <= t1]
            after = [r for t, r in stamped if t is not None and t >= t0]
            n = len(self.devices)
            rows = inside or after[:2 * n] or rows[-2 * n:]
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- CPU path
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def workload_config(layers: int) -> dict:
    """The workload both arms measure."""
    return {"workload": "config5_zimage_6b_linear_stack", "layers": layers, "m_tokens": M_TOKENS,
            "hidden": HIDDEN, "ffn": FFN, "mix": "Q4_K_M (w2 Q6_K in even layers)",
            "weights": "N(0, 0.02) quantised to the mix; X ~ N(0, 1)"}


def cpu_reference_sample(m_sample: int, linears, threads: int, x=None):
    """The reference's CPU path on a bounded sample: decode_cpu_into -> f32
    (the reference decoder built from its sources, row-split over `threads`
    as its RowDecodePool does, native/runtime/streaming/gguf_packed_bank.cpp:48-100)
    then an fp32 matmul with torch on `threads` host threads (the reference
    has no CPU GEMM).  Returns (seconds, flops, kind)."""
    import torch
    from oracle import oracle
    kind = "reference" if oracle.ref() is not None else "port"
    torch.set_num_threads(threads)
    if x is None:
        x = torch.randn(m_sample, FFN, generator=torch.Generator().manual_seed(5))
    t0 = time.perf_counter()
    flops = 0.0
    for name, n, k, typ, raw in linears:
        w = oracle.decode_parallel(raw, typ, n, k, 0, which="ref" if kind == "reference" else "port", threads=threads)
        y = x[:m_sample, :k] @ torch.from_numpy(w).T
        flops += 2.0 * m_sample * n * k
        del y, w
    return time.perf_counter() - t0, flops, kind


def make_cpu_linears(layer: int = 0):
    """Raw GGUF blocks of one layer's linears, quantised by the numpy
    restatement of the backend's quantiser (oracle/kq_quantize.py, same bytes
    as tc_quantize), so the CPU arm never loads the backend library."""
    from oracle import kq_quantize
    out = []
    for i, (name, n, k, typ) in enumerate(layer_linears(layer)):
        w = (np.random.default_rng(1000 * layer + i).standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        out.append((name, n, k, typ, kq_quantize.quantize(typ, w)))
    return out


def run_reference(args):
    """The reference arm: the reference's own CPU path for the workload (its
    decoder from oracle/_ref, all host threads) on rank 0; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch
    threads = os.cpu_count() or 1
    linears = make_cpu_linears(0)
    m_sample = args.cpu_rows or M_TOKENS
    x = torch.randn(m_sample, FFN, generator=torch.Generator().manual_seed(5))
    for _ in range(args.warmup):
        cpu_reference_sample(m_sample, linears, threads, x)
    times, flops, kind = [], 0.0, "port"
    for _ in range(args.steps):
        t, flops, kind = cpu_reference_sample(m_sample, linears, threads, x)
        times.append(t)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    sample = (f"layer 0 of the stack (qkv, out, w1, w3, w2 Q6_K) per step: the reference's decode_cpu_into -> f32 "
              f"of the 5 weights + fp32 matmul at {m_sample} of {M_TOKENS} rows")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(args.layers),
            "parallelism": "CPU, rank 0 only",
            "cpu_baseline": {"value": round(value, 4), "unit": "TFLOPS", "cores": threads, "cpu": cpu_model(),
                             "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
def build_weights(ctx, rank, world, layers, device, ffn: str = "separate"):
    """Upload every layer's weight shard (turbocider_b200.shard.shard_rows) to HBM.
    ffn "swiglu": w1 and w3 go up as one interleaved weight "w13" whose GEMM
    epilogue computes silu(w1 x) * w3 x (tc_cuda_weight_upload_glu).
    Returns (weights per layer, {(seed layer, name): (raw shard, rows, K, type)})."""
    import torch
    from turbocider_b200 import cuda as tcc
    from turbocider_b200 import shard
    threads = max(1, (os.cpu_count() or 8) // max(1, world))
    raw_cache = {}
    for d in range(min(DISTINCT_LAYERS, layers)):
        for i, (name, n, k, typ) in enumerate(layer_linears(d)):
            g = torch.Generator(device=device).manual_seed(1000 * d + i)
            b, rows = shard.shard_rows(n, world, rank)
            w = torch.randn(n, k, generator=g, device=device)[b:b + rows].mul_(0.02)
            raw_cache[(d, name)] = (tcc.quantize(typ, w.cpu().numpy(), threads=threads), rows, k, typ)
            del w
    weights = []
    for layer in range(layers):
        lw = {}
        for name, n, k, typ in layer_linears(layer):
            raw, rows, kk, t = raw_cache[(layer % DISTINCT_LAYERS, name)]
            assert t == typ
            if ffn == "swiglu" and name in ("w1", "w3"):
                if name == "w1":
                    up = raw_cache[(layer % DISTINCT_LAYERS, "w3")]
                    lw["w13"] = tcc.Weight.upload_glu(ctx, typ, rows, kk, raw, up[0])
                continue
            lw[name] = tcc.Weight.upload(ctx, typ, rows, kk, raw)
        weights.append(lw)
    return weights, raw_cache


def gemv_measure(ctx, device, hbm_peak):
    """Config 2: Q6_K GEMV, K=12288, N=3072, M in {1, 4, 16}; 10 weight copies
    (310 MB > L2) cycled inside a CUDA graph so every call streams HBM."""
    import torch
    from turbocider_b200 import cuda as tcc
    n, k, copies, calls = 3072, 12288, 10, 40
    w = (np.random.default_rng(2).standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
    raw = tcc.quantize(Q6_K, w)
    ws = [tcc.Weight.upload(ctx, Q6_K, n, k, raw) for _ in range(copies)]
    out = {}
    stream = torch.cuda.Stream(device)
    for m in (1, 4, 16):
        x = torch.randn(m, k, device=device).to(torch.bfloat16)
        y = torch.empty(m, n, device=device, dtype=torch.bfloat16)
        with torch.cuda.stream(stream):
            for i in range(copies):
                tcc.qlinear(ctx, ws[i], x, out=y, stream=stream)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(calls):
                    tcc.qlinear(ctx, ws[i % copies], x, out=y, stream=stream)
            for _ in range(3):
                graph.replay()
            stream.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 10
            ev0.record(stream)
            for _ in range(reps):
                graph.replay()
            ev1.record(stream)
            ev1.synchronize()
        sec = ev0.elapsed_time(ev1) / 1e3 / (reps * calls)
        nbytes = len(raw) + m * k * 2 + m * n * 2
        gbs = nbytes / sec / 1e9
        out[str(m)] = {"us_per_call": round(sec * 1e6, 3), "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4),
                       "bytes_per_call": nbytes}
        del graph
        # Batched: the 10 weights (e.g. 10 blocks' modulation linears, all fed
        # the same timestep embedding) in one launch per call.
        ys = [torch.empty(m, n, device=device, dtype=torch.bfloat16) for _ in range(copies)]
        bcalls = 8
        with torch.cuda.stream(stream):
            tcc.qlinear_batched(ctx, ws, x, outs=ys, stream=stream)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(bcalls):
                    tcc.qlinear_batched(ctx, ws, x, outs=ys, stream=stream)
            for _ in range(3):
                graph.replay()
            stream.synchronize()
            ev0.record(stream)
            for _ in range(reps):
                graph.replay()
            ev1.record(stream)
            ev1.synchronize()
        bsec = ev0.elapsed_time(ev1) / 1e3 / (reps * bcalls)
        bbytes = copies * len(raw) + m * k * 2 + copies * m * n * 2
        bgbs = bbytes / bsec / 1e9
        out[str(m)]["batched"] = {"weights_per_launch": copies, "us_per_call": round(bsec * 1e6, 3),
                                  "gbs": round(bgbs, 1), "frac": round(bgbs / hbm_peak, 4), "bytes_per_call": bbytes}
        del graph
    assert ctx.status() == 0
    for wt in ws:
        wt.free()
    return {"config": "configs[1]: Q6_K W[3072, 12288], X bf16 [M, 12288]; 10 weight copies cycled (> L2), "
                      "40 calls per CUDA graph; 'batched': the 10 weights in one tc_cuda_qlinear_batched launch "
                      "(310 MB per call), 8 calls per graph", "peak_gbs": hbm_peak, "m": out}


# ---------------------------------------------------------------- config 4
C4_HIDDEN, C4_FFN, C4_BLOCKS = 3072, 12288, 60
C4_REQUESTS = [(256, 256), (1024, 256), (2304, 256), (2304, 256)]   # (image, text) tokens, CFG 2 each


def config4_linears(block: int):
    """(name, N, K, type) of one Qwen-Image-style dual-stream block's linears
    (same for the image and the text stream): qkv/out/ffn_up Q4_K, attn_v Q6_K,
    ffn_down Q6_K in even blocks; AdaLN modulation [6 * hidden, hidden]."""
    h, f = C4_HIDDEN, C4_FFN
    return [("q", h, h, Q4_K), ("k", h, h, Q4_K), ("v", h, h, Q6_K), ("out", h, h, Q4_K),
            ("up", f, h, Q4_K), ("down", h, f, Q6_K if block % 2 == 0 else Q4_K), ("mod", 6 * h, h, Q4_K)]


def config4_stream(ctx, device, passes: int = 2):
    """4 ragged requests packed along M (8 segments,
    image / text weights chosen per segment), 60 blocks, every block's weights
    streamed from pinned host memory through two HBM slots while the previous
    block computes.  Contents cycle over 2 seeds (2 pinned blocks); the bytes
    moved over PCIe per pass are those of 60 blocks."""
    import torch
    from turbocider_b200 import cuda as tcc
    from turbocider_b200.stream import LayerStream
    threads = os.cpu_count() or 1
    seg, sw, m = [0], [], 0
    for img, txt in C4_REQUESTS:
        for rows, which in ((2 * img, 0), (2 * txt, 1)):
            m += rows
            seg.append(m)
            sw.append(which)
    raws = {}
    for d in range(2):
        for i, (name, n, k, typ) in enumerate(config4_linears(d)):
            for stream_id in range(2):
                g = torch.Generator(device=device).manual_seed(50000 + 100 * d + 10 * i + stream_id)
                w = torch.randn(n, k, generator=g, device=device).mul_(0.02).cpu().numpy()
                raws[(d, name, stream_id)] = tcc.quantize(typ, w, threads=threads)
    layers = []
    for b in range(C4_BLOCKS):
        layers.append({f"{name}.{sid}": (typ, n, k, raws[(b % 2, name, sid)])
                       for name, n, k, typ in config4_linears(b) for sid in range(2)})
    st = LayerStream(ctx, layers, device, threads=threads)
    g = torch.Generator(device=device).manual_seed(9)
    x_h = torch.randn(m, C4_HIDDEN, generator=g, device=device).to(torch.float16)
    x_f = torch.randn(m, C4_FFN, generator=g, device=device).to(torch.float16)
    x_mod = torch.randn(2 * len(C4_REQUESTS), C4_HIDDEN, generator=g, device=device).to(torch.bfloat16)
    y = {n: torch.empty(m, n, device=device, dtype=torch.bfloat16) for n in (C4_HIDDEN, C4_FFN)}
    y_mod = torch.empty(2 * len(C4_REQUESTS), 6 * C4_HIDDEN, device=device, dtype=torch.bfloat16)
    compute = torch.cuda.Stream(device)
    flops = 0.0

    def one_pass():
        nonlocal flops
        flops = 0.0
        st.begin(compute)
        for b in range(C4_BLOCKS):
            w = st.acquire(b, compute)
            for name, n, k, typ in config4_linears(b):
                pair = [w[f"{name}.0"], w[f"{name}.1"]]
                if name == "mod":   # per-request modulation rows, image and text stream
                    for sid in range(2):
                        tcc.qlinear(ctx, pair[sid], x_mod, out=y_mod, stream=compute)
                        flops += 2.0 * x_mod.shape[0] * n * k
                    continue
                x = x_f if name == "down" else x_h
                tcc.qlinear(ctx, pair, x, seg_offsets=seg, seg_weight=sw, out=y[n], stage=tcc.STAGE_F16_X16,
                            stream=compute)
                flops += 2.0 * m * n * k
            st.release(b, compute)

    with torch.cuda.stream(compute):
        one_pass()
        compute.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        for _ in range(passes):
            one_pass()
        e1.record(compute)
        e1.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / passes
    moved = sum(st.bytes_per_layer)
    assert ctx.status() == 0
    st.close()
    return {"config": "configs[3]: 60 dual-stream blocks (hidden 3072, FFN 12288), 4 ragged requests "
                      "(256/1024/2304/2304 image + 256 text tokens, CFG 2) packed along M = 13824 in 8 segments; "
                      "weights streamed per block from pinned host memory (2 HBM slots)",
            "tflops": round(flops / sec / 1e12, 2), "ms_per_pass": round(sec * 1e3, 2),
            "h2d_gb_per_pass": round(moved / 1e9, 2), "h2d_gbs": round(moved / sec / 1e9, 1),
            "passes": passes}


def epilogue_measure(ctx, device):
    """Fused epilogues on config-5 shapes (M = 8448, K = 3840, fp16 activations
    and staging, bf16 out): the qkv weight plain, with a bias, with bias + GELU;
    a 20480-row weight plain and as the SwiGLU pair w1 / w3 (one output per
    gate / up row pair).  Each timed over 10 calls with CUDA events."""
    import torch
    from turbocider_b200 import cuda as tcc
    threads = os.cpu_count() or 1
    m = M_TOKENS

    def raw(n, seed):
        g = torch.Generator(device=device).manual_seed(seed)
        w = torch.randn(n, HIDDEN, generator=g, device=device).mul_(0.02)
        return tcc.quantize(Q4_K, w.cpu().numpy(), threads=threads)
    w_qkv = tcc.Weight.upload(ctx, Q4_K, 3 * HIDDEN, HIDDEN, raw(3 * HIDDEN, 71))
    r1, r3 = raw(FFN, 72), raw(FFN, 73)
    w_glu = tcc.Weight.upload_glu(ctx, Q4_K, FFN, HIDDEN, r1, r3)
    w_2f = tcc.Weight.upload(ctx, Q4_K, 2 * FFN, HIDDEN, raw(2 * FFN, 74))
    g = torch.Generator(device=device).manual_seed(75)
    x = torch.randn(m, HIDDEN, generator=g, device=device).to(torch.float16)
    b_qkv = torch.randn(3 * HIDDEN, generator=g, device=device) * 0.1
    b_glu = torch.randn(2 * FFN, generator=g, device=device) * 0.1
    s = torch.cuda.Stream(device)

    def tflops(w, xin=None, stage=tcc.STAGE_F16_X16, **kw):
        out = torch.empty(m, w.n_out, dtype=torch.bfloat16, device=device)
        xx = x if xin is None else xin
        call = lambda: tcc.qlinear(ctx, w, xx, out=out, stage=stage, stream=s, **kw)
        with torch.cuda.stream(s):
            for _ in range(3):
                call()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(10):
                call()
            e1.record(s)
            e1.synchronize()
        return round(2.0 * m * w.n * w.k * 10 / (e0.elapsed_time(e1) / 1e3) / 1e12, 1)
    x_b = x.to(torch.bfloat16)
    res = {"config": "config-5 shapes, M = 8448, K = 3840, X fp16, bf16 out; TFLOP/s of 2 M N K",
           "qkv_plain": tflops(w_qkv), "qkv_bias": tflops(w_qkv, bias=b_qkv),
           "qkv_bf16_x_stage_f16": tflops(w_qkv, xin=x_b, stage=tcc.STAGE_F16),
           "qkv_bf16_x_stage_bf16": tflops(w_qkv, xin=x_b, stage=tcc.STAGE_BF16),
           "qkv_bias_gelu_tanh": tflops(w_qkv, bias=b_qkv, activation="gelu_tanh"),
           "rows20480_plain": tflops(w_2f), "w1_w3_swiglu_bias": tflops(w_glu, bias=b_glu)}
    assert ctx.status() == 0
    for w in (w_qkv, w_glu, w_2f):
        w.free()
    return res


# ---------------------------------------------------------------- GGUF loader
def write_gguf(path, tensors, alignment: int = 32):
    """Minimal GGUF v3 container: no metadata; tensors = [(name, ggml type,
    rows, columns, raw uint8 blocks)], payloads back to back at `alignment`
    (the layout read_directory accepts, gguf_directory.hpp:199-271)."""
    import struct
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), 0)
    offset = 0
    for name, typ, rows, cols, raw in tensors:
        nb = name.encode()
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", 2) + struct.pack("<QQ", cols, rows)
        head += struct.pack("<IQ", typ, offset)
        offset = (offset + raw.nbytes + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head + bytes((-len(head)) % alignment))
        for *_, raw in tensors:
            f.write(raw.tobytes())
            f.write(bytes((-raw.nbytes) % alignment))


def loader_measure(ctx, raw_cache, reps: int = 3):
    """File -> HBM streaming load (tc_cuda_weight_load_gguf: pread read-ahead
    into pinned slots, copy to HBM, device re-layout) of one stack layer's
    five weights (about 100 MB) from a GGUF file written to a temporary
    directory just before, i.e. from the page cache.  GB/s of raw blocks."""
    from turbocider_b200 import cuda as tcc
    tensors = [(f"blk.0.{name}.weight", typ, rows, k, raw_cache[(0, name)][0])
               for name, _, _, typ in layer_linears(0) for rows, k in [raw_cache[(0, name)][1:3]]]
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "layer0.gguf"
        write_gguf(path, tensors)
        f = tcc.GGUFFile(path)
        best = None
        for _ in range(reps):
            tot = {"bytes": 0, "seconds": 0.0, "read_seconds": 0.0, "wait_seconds": 0.0, "chunks": 0}
            for name, *_ in tensors:
                w, st = tcc.Weight.load_gguf(ctx, f, name)
                w.free()
                for key in tot:
                    tot[key] += st[key]
            if best is None or tot["seconds"] < best["seconds"]:
                best = tot
        f.close()
    return {"config": "one stack layer's 5 weights (qkv, out, w1, w3, w2 Q6_K) from a GGUF file in the page cache, "
                      "8 MiB chunks (whole 128-row panels), best of 3",
            "gb": round(best["bytes"] / 1e9, 4), "gbs": round(best["bytes"] / best["seconds"] / 1e9, 2),
            "chunks": best["chunks"], "read_seconds": round(best["read_seconds"], 4),
            "wait_seconds": round(best["wait_seconds"], 4), "seconds": round(best["seconds"], 4)}


# ---------------------------------------------------------------- configs 1 and 3
def config1_measure(ctx, device, tc_burst):
    """BASELINE configs[0] on the GPU: one Q4_K linear, W [3072, 3072], X bf16
    [256, 3072] (converted to fp16 for fp16 staging, TC_STAGE_F16), bf16 out.
    32 weight copies (170 MB > L2) cycled inside a CUDA graph of 64 calls."""
    import torch
    from turbocider_b200 import cuda as tcc
    n = k = 3072
    m, copies, calls, reps = 256, 32, 64, 10
    g = torch.Generator(device=device).manual_seed(11)
    raw = tcc.quantize(Q4_K, (torch.randn(n, k, generator=g, device=device) * 0.02).cpu().numpy())
    ws = [tcc.Weight.upload(ctx, Q4_K, n, k, raw) for _ in range(copies)]
    x = torch.randn(m, k, generator=g, device=device).to(torch.bfloat16)
    y = torch.empty(m, n, device=device, dtype=torch.bfloat16)
    stream = torch.cuda.Stream(device)
    res = {"config": "configs[0]: Q4_K W[3072, 3072], X bf16 [256, 3072] -> fp16 staging (TC_STAGE_F16, "
                     "conversion included), bf16 Y; 32 weight copies cycled (> L2), 64 calls per CUDA graph"}
    with torch.cuda.stream(stream):
        for i in range(copies):
            tcc.qlinear(ctx, ws[i], x, out=y, stage=tcc.STAGE_F16, stream=stream)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(calls):
                tcc.qlinear(ctx, ws[i % copies], x, out=y, stage=tcc.STAGE_F16, stream=stream)
        for _ in range(3):
            graph.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / (reps * calls)
    tflops = 2.0 * m * n * k / sec / 1e12
    res.update({"us_per_call": round(sec * 1e6, 2), "tflops": round(tflops, 1),
                "frac": round(tflops / tc_burst, 4), "peak": "measured burst bf16",
                "tiles": "12 pair tiles (256 weight rows x 256 tokens) of 4.8 GFLOP in total"})
    del graph
    assert ctx.status() == 0
    for w in ws:
        w.free()
    return res


C3_HIDDEN, C3_FFN, C3_IMG, C3_TXT = 3072, 12288, 2048, 512


def config3_linears(block: int):
    """(name, N, K, type, activation) of one Qwen-Image-style dual-stream
    MMDiT block, per stream (reference call sites
    native/models/qwen21/transformer.cpp:857-859 to_q/k/v, :953 to_out,
    :971-978 the FFN): q, k, out, ffn_up Q4_K; v Q6_K; ffn_down Q6_K in even
    blocks and Q4_K in odd ones; ffn_up carries the GELU (tanh form)."""
    h, f = C3_HIDDEN, C3_FFN
    return [("q", h, h, Q4_K, None), ("k", h, h, Q4_K, None), ("v", h, h, Q6_K, None),
            ("out", h, h, Q4_K, None), ("up", f, h, Q4_K, "gelu_tanh"),
            ("down", h, f, Q6_K if block % 2 == 0 else Q4_K, None)]


def config3_measure(ctx, device, tc_sustained):
    """one dual-stream MMDiT block's linears, image stream
    M = 2048 and text stream M = 512 packed as two ragged segments of one call
    per projection (separate image / text weights), X bf16 -> fp16 staging,
    bf16 out, GELU fused into ffn_up; plus the AdaLN modulation linears
    [6 * 3072, 3072] of both streams at M = 2 (the CFG pair's timestep
    embedding, reference transformer.cpp:368-369, :420-421) in one batched
    GEMV.  Two blocks per iteration (ffn_down Q6_K, then Q4_K)."""
    import torch
    from turbocider_b200 import cuda as tcc
    threads = os.cpu_count() or 1
    h, f, m = C3_HIDDEN, C3_FFN, C3_IMG + C3_TXT
    seg, sw = [0, C3_IMG, m], [0, 1]
    blocks = []
    seed = 300
    for b in range(2):
        lw = {}
        for name, n, k, typ, act in config3_linears(b):
            pair = []
            for stream_id in range(2):
                seed += 1
                g = torch.Generator(device=device).manual_seed(seed)
                raw = tcc.quantize(typ, (torch.randn(n, k, generator=g, device=device) * 0.02).cpu().numpy(),
                                   threads=threads)
                pair.append(tcc.Weight.upload(ctx, typ, n, k, raw))
            lw[name] = pair
        mods = []
        for stream_id in range(2):
            seed += 1
            g = torch.Generator(device=device).manual_seed(seed)
            raw = tcc.quantize(Q4_K, (torch.randn(6 * h, h, generator=g, device=device) * 0.02).cpu().numpy(),
                               threads=threads)
            mods.append(tcc.Weight.upload(ctx, Q4_K, 6 * h, h, raw))
        lw["mod"] = mods
        blocks.append(lw)
    g = torch.Generator(device=device).manual_seed(399)
    x_h = torch.randn(m, h, generator=g, device=device).to(torch.bfloat16)
    x_f = torch.randn(m, f, generator=g, device=device).to(torch.bfloat16)
    temb = torch.randn(2, h, generator=g, device=device).to(torch.bfloat16)
    y_h = torch.empty(m, h, device=device, dtype=torch.bfloat16)
    y_f = torch.empty(m, f, device=device, dtype=torch.bfloat16)
    y_mod = [torch.empty(2, 6 * h, device=device, dtype=torch.bfloat16) for _ in range(2)]
    stream = torch.cuda.Stream(device)
    flops = 0.0

    def one_iter():
        nonlocal flops
        flops = 0.0
        for b, lw in enumerate(blocks):
            tcc.qlinear_batched(ctx, lw["mod"], temb, outs=y_mod, stream=stream)
            flops += 2 * 2.0 * 2 * 6 * h * h
            for name, n, k, typ, act in config3_linears(b):
                x = x_f if name == "down" else x_h
                out = y_f if n == f else y_h
                tcc.qlinear(ctx, lw[name], x, seg_offsets=seg, seg_weight=sw, out=out, stage=tcc.STAGE_F16,
                            activation=act, stream=stream)
                flops += 2.0 * m * n * k

    reps = 10
    with torch.cuda.stream(stream):
        for _ in range(3):
            one_iter()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            one_iter()
        e1.record(stream)
        e1.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    tflops = flops / sec / 1e12
    assert ctx.status() == 0
    for lw in blocks:
        for pair in lw.values():
            for w in pair:
                w.free()
    return {"config": "configs[2]: 2 dual-stream MMDiT blocks (hidden 3072, FFN 12288 GELU; ffn_down Q6_K then "
                      "Q4_K), image M = 2048 + text M = 512 as two ragged segments per call, X bf16 -> fp16 "
                      "staging, bf16 Y, + AdaLN modulation [18432, 3072] x 2 streams at M = 2 (batched GEMV)",
            "ms_per_block": round(sec * 1e3 / 2, 3), "gflop_per_block": round(flops / 2 / 1e9, 2),
            "tflops": round(tflops, 1), "frac": round(tflops / tc_sustained, 4), "peak": "measured sustained bf16"}


# ---------------------------------------------------------------- multi-GPU
def push_engine(args) -> str:
    """How --gather copy moves each output shard to the peers (for the JSON line)."""
    if args.push_kernel:
        return f"a peer-push kernel ({args.push_kernel} blocks of SM stores over NVLink, on a side stream"
    if args.push_streams >= 2:
        return f"copy-engine peer pushes (over {args.push_streams} side streams"
    return "copy-engine peer pushes (back to back on a side stream"


def gather_measure(ctx, device, world, rank, m, width):
    """The all-gather alone (no GEMM running): one rank's shard of `m` rows x
    `width` fp16 columns goes to every other rank, by copy-engine pushes back
    to back on one stream or spread over 2, 4 or world - 1 side streams, and
    by NCCL all_gather_into_tensor.  GB/s = bytes each GPU
    receives ((world - 1) shards) / time, max over ranks."""
    import torch
    import torch.distributed as dist
    from turbocider_b200.peer import PeerGroup
    pg = PeerGroup(ctx, timeout_us=20_000_000)
    shard = m * width * 2
    buf = pg.alloc(world * shard)
    s = torch.cuda.Stream(device)
    out = {"shard_mb": round(shard / 1e6, 2)}

    def timed(fn, reps=5):
        for _ in range(2):
            fn()
        torch.cuda.synchronize(device)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            fn()
        e1.record(s)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3 / reps], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def push():
        pg.push(buf, rank * shard, shard, stream=s)
        pg.barrier(s)

    for streams in sorted({1, 2, 4, world - 1}):
        if streams > world - 1:
            continue
        ctx.set_push_fanout(streams)
        t = timed(push)
        out["push_serial" if streams == 1 else f"push_{streams}_streams"] = {
            "ms": round(t * 1e3, 3), "gbs_in_per_gpu": round((world - 1) * shard / t / 1e9, 1)}
    ctx.set_push_fanout(0)
    for ctas in (37, 74, 148, 296):
        ctx.set_push_kernel(ctas)
        t = timed(push)
        out[f"push_kernel_{ctas}_blocks"] = {
            "ms": round(t * 1e3, 3), "gbs_in_per_gpu": round((world - 1) * shard / t / 1e9, 1)}
    ctx.set_push_kernel(0)
    src = torch.zeros(m, width, device=device, dtype=torch.float16)
    dst = torch.empty(world * m, width, device=device, dtype=torch.float16)

    def nccl():
        with torch.cuda.stream(s):
            dist.all_gather_into_tensor(dst, src)

    t = timed(nccl)
    out["nccl_all_gather"] = {"ms": round(t * 1e3, 3), "gbs_in_per_gpu": round((world - 1) * shard / t / 1e9, 1),
                              "bus_gbs": round((world - 1) * shard / t / 1e9, 1)}
    assert ctx.status() == 0
    del src, dst
    pg.close()
    return out


def parity_check(raw_cache, names, layers, y_loc, y_all, x_h, x_f, world, rank, nloc, mode, n_out):
    """Sampled rows of the last outputs against the CPU oracle, and the
    gathered Y of every rank against the shards the ranks computed.

    Oracle: the reference's decode (decode_cpu_into to f32, oracle/ port) and
    an fp64 matmul of the same fp16 X rows (oracle.qlinear_ref), with the
    SwiGLU silu(w1 x) * w3 x applied in fp64 (oracle.epilogue_ref); bar
    rel-L2 <= 1e-3 on the fp16 outputs.  Both buffers of each linear are
    checked: they hold the last two layers (w2 Q6_K and Q4_K).
    Gather: every rank checksums each rank-slot of its gathered buffers; all
    ranks must agree, i.e. each rank's copy of slot r equals what rank r
    wrote (its own slot, whose rows were checked against the oracle)."""
    import torch
    import torch.distributed as dist
    from oracle import oracle
    rows = np.sort(np.random.default_rng(123).choice(M_TOKENS, 16, replace=False))
    idx = torch.from_numpy(rows).to(x_h.device)
    xs = {"h": x_h.index_select(0, idx).view(torch.int16).cpu().numpy().view(np.uint16),
          "f": x_f.index_select(0, idx).view(torch.int16).cpu().numpy().view(np.uint16)}
    worst, checked = 0.0, []
    for b in (0, 1):
        layer = layers - 1 if ((layers - 1) & 1) == b else layers - 2
        if layer < 0:
            continue
        d = layer % DISTINCT_LAYERS
        for name in names:
            raw, cols, k, typ = raw_cache[(d, "w1" if name == "w13" else name)]
            if not cols:
                continue   # this rank holds no columns of the weight
            got = y_loc[(name, b)].index_select(0, idx).float().cpu().numpy().astype(np.float64)
            x = xs["f"] if name == "w2" else xs["h"]
            if name == "w13":
                u_raw = raw_cache[(d, "w3")][0]
                acc = np.concatenate([oracle.qlinear_ref(x, raw, typ, cols, k, "f32", x_dtype="f16"),
                                      oracle.qlinear_ref(x, u_raw, typ, cols, k, "f32", x_dtype="f16")], axis=1)
                ref = oracle.epilogue_ref(acc, glu=True)
            else:
                ref = oracle.qlinear_ref(x, raw, typ, cols, k, "f32", x_dtype="f16")
            err = oracle.rel_l2(got[:, :ref.shape[1]], ref)
            worst = max(worst, err)
            checked.append(f"layer{layer}.{name}")
    consistent = None
    if world > 1:
        sums = []
        for key in sorted(y_all):
            name = key[0]
            buf = y_all[key]
            if mode == "fused":
                slots = [buf[:, r * nloc[name]:(r + 1) * nloc[name]] for r in range(world)]
            else:
                slots = list(buf.reshape(world, M_TOKENS, nloc[name]).unbind(0))
            for sl in slots:
                v = sl.contiguous().view(torch.int16).to(torch.int64).flatten()
                w = torch.arange(v.numel(), device=v.device, dtype=torch.int64) % 65521 + 1
                sums.append((v * w).sum())
        mine = torch.stack(sums)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        consistent = all(bool(torch.equal(e, every[0])) for e in every)
        t = torch.tensor([worst, 0.0 if consistent else 1.0], device=x_h.device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        worst, consistent = float(t[0]), float(t[1]) == 0.0
    return {"rel_l2_max": float(f"{worst:.3e}"), "bar": 1e-3, "ok": bool(worst <= 1e-3 and consistent is not False),
            "rows_sampled": int(len(rows)), "linears_checked_per_rank": len(checked),
            "oracle": "decode_cpu_into(f32) + fp64 matmul of the same fp16 X rows; SwiGLU in fp64",
            "gathered_y_consistent_on_all_ranks": consistent}


def run_leg(args):
    """One measurement leg alone on GPU 0 (the unit a profiler captures)."""
    import torch
    from turbocider_b200 import cuda as tcc
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    hbm_peak, tc_burst, tc_sustained, _ = peaks()
    ctx = tcc.Context(0)
    if args.leg == "gemv":
        out = gemv_measure(ctx, device, hbm_peak)
    elif args.leg == "config1":
        out = config1_measure(ctx, device, tc_burst)
    elif args.leg == "config3":
        out = config3_measure(ctx, device, tc_sustained)
    elif args.leg == "config4":
        out = config4_stream(ctx, device)
    elif args.leg == "epilogues":
        out = epilogue_measure(ctx, device)
    else:
        weights, raw_cache = build_weights(ctx, 0, 1, 1, device, args.ffn)
        out = loader_measure(ctx, raw_cache)
        for lw in weights:
            for wt in lw.values():
                wt.free()
    ctx.close()
    print(json.dumps({"leg": args.leg, **out}), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from turbocider_b200 import cuda as tcc

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    # rank 0 samples the clocks of every GPU of the job (device i = local rank i)
    clocks = ClockSampler(list(range(world)) if world > 1 else local)
    if rank == 0:
        clocks.start()
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    hbm_peak, tc_burst, tc_sustained, peak_src = peaks()
    layers = args.layers
    ctx = tcc.Context(local)
    reserve = args.reserve_sms or 0
    if reserve:
        # leave SMs free for the NCCL all-gather that runs beside each GEMM
        ctx.set_sm_limit(torch.cuda.get_device_properties(device).multi_processor_count - reserve)
    weights, raw_cache = build_weights(ctx, rank, world, layers, device, args.ffn)

    m = M_TOKENS
    g = torch.Generator(device=device).manual_seed(7)
    # fp16 activations, W staged fp16 (TC_STAGE_F16_X16), fp16 outputs: the
    # precision that meets rel-L2 <= 1e-3 against dequant + fp32 matmul, and
    # the activation type of the reference's own GGUF execution.
    x_h = torch.randn(m, HIDDEN, generator=g, device=device).to(torch.float16)
    x_f = torch.randn(m, FFN, generator=g, device=device).to(torch.float16)
    compute = torch.cuda.Stream(device)
    comm = torch.cuda.Stream(device)
    sync = torch.cuda.Stream(device)   # per-layer completion barriers, off the push stream
    names = [l[0] for l in layer_linears(0)]
    if args.ffn == "swiglu":
        names = ["w13" if nm == "w1" else nm for nm in names if nm != "w3"]
    from turbocider_b200 import shard
    nloc = {name: shard.rows_per_rank(n, world) for name, n, _, _ in layer_linears(0)}
    nloc["w13"] = nloc["w1"]   # SwiGLU: one output column per gate / up row pair
    fused = world > 1 and args.gather == "fused"
    ce = world > 1 and args.gather == "copy"
    pg = None
    f16 = torch.float16
    if ce:
        # All-gather by the copy engines: every rank's gathered Y is
        # shard-major [g, M, N/g] (an NCCL all-gather's layout) in a buffer all
        # ranks can write (CUDA IPC).  The GEMM stores only this rank's slot;
        # a side stream then pushes the slot into every peer's buffer
        # (tc_cuda_peer_push) while the next linear runs, and one device flag
        # barrier per layer on that stream marks every rank's Y complete.
        from turbocider_b200.peer import PeerGroup
        pg = PeerGroup(ctx, timeout_us=20_000_000)
        ctx.set_push_fanout(args.push_streams)
        ctx.set_push_kernel(args.push_kernel)
        y_sym = {(name, b): pg.alloc(world * m * nloc[name] * 2) for name in names for b in (0, 1)}
        y_all = {key: buf.tensor((world, m, nloc[key[0]]), f16) for key, buf in y_sym.items()}
        y_loc = {key: y_all[key][rank][:, :weights[0][key[0]].n_out] for key in y_all}
    elif fused:
        # All-gather fused into the GEMM epilogue: every rank's Y[M, g * N/g]
        # lives in a buffer all ranks can store into (CUDA IPC); each GEMM
        # writes its column shard into all of them over NVLink, then a device
        # flag barrier marks every Y complete (turbocider_b200.peer).
        from turbocider_b200.peer import PeerGroup
        pg = PeerGroup(ctx, timeout_us=20_000_000)
        y_sym = {(name, b): pg.alloc(m * world * nloc[name] * 2) for name in names for b in (0, 1)}
        y_all = {key: buf.tensor((m, world * nloc[key[0]]), f16) for key, buf in y_sym.items()}
        y_loc = {key: y_all[key][:, rank * nloc[key[0]]:rank * nloc[key[0]] + weights[0][key[0]].n_out]
                 for key in y_all}
        y_peers = {key: pg.peers_of(buf, rank * nloc[key[0]] * 2) for key, buf in y_sym.items()}
    else:
        # double-buffered local outputs and gathered outputs per linear
        y_loc = {(name, b): torch.empty(m, nloc[name], device=device, dtype=f16)
                 for name in names for b in (0, 1)}
        y_all = ({(name, b): torch.empty(world * m, nloc[name], device=device, dtype=f16)
                  for name in names for b in (0, 1)} if world > 1 else {})
    gathered = {(name, b): None for name in names for b in (0, 1)}

    def one_step(timing=None, dependent=False):
        """One pass of the stack.  dependent=True: every linear waits (on the
        compute stream) until the previous linear's output has been gathered
        on every rank, as a chain of layers that consume the gathered Y must."""
        prev = None
        for layer in range(layers):
            b = layer & 1
            for name in names:
                x = x_f if name == "w2" else x_h
                if world > 1 and not fused and gathered[(name, b)] is not None:
                    compute.wait_event(gathered[(name, b)])     # buffer reuse after its gather / push
                if dependent and prev is not None:
                    compute.wait_event(prev)
                if timing is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(compute)
                tcc.qlinear(ctx, weights[layer][name], x, out=y_loc[(name, b)], out_dtype=tcc.F16,
                            stage=tcc.STAGE_F16_X16, stream=compute, peers=y_peers[(name, b)] if fused else None)
                if timing is not None:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(compute)
                    timing.append((e0, e1, 2.0 * m * weights[layer][name].n * weights[layer][name].k))
                if fused:
                    pg.barrier(compute)
                elif ce:
                    done = torch.cuda.Event()
                    done.record(compute)
                    comm.wait_event(done)
                    nb = m * nloc[name] * 2
                    pg.push(y_sym[(name, b)], rank * nb, nb, stream=comm)
                    if dependent:
                        pg.barrier(comm)    # this linear's Y complete on every rank
                    ev = torch.cuda.Event()
                    ev.record(comm)
                    gathered[(name, b)] = ev
                    prev = ev
                elif world > 1:
                    done = torch.cuda.Event()
                    done.record(compute)
                    comm.wait_event(done)
                    with torch.cuda.stream(comm):
                        dist.all_gather_into_tensor(y_all[(name, b)], y_loc[(name, b)])
                    ev = torch.cuda.Event()
                    ev.record(comm)
                    gathered[(name, b)] = ev
                    prev = ev
            if ce and not dependent:
                # every rank's outputs of this layer complete: a flag barrier
                # ordered after this rank's pushes, on its own stream so that
                # the next layer's pushes do not queue behind the slowest rank
                pushed = torch.cuda.Event()
                pushed.record(comm)
                sync.wait_event(pushed)
                pg.barrier(sync)
        if world > 1 and not fused:
            compute.wait_stream(comm)
            compute.wait_stream(sync)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(sec):
        if world == 1:
            return sec
        tt = torch.tensor([sec], device=device, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    with torch.cuda.stream(compute):
        for _ in range(args.warmup):
            one_step()
    barrier()
    if ctx.status(clear=True):
        raise SystemExit("device status word set during warm-up")

    timing = []
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host_t0 = time.time()
    t0.record(compute)
    for i in range(args.steps):
        # per-launch events only in the last step: events between kernels would
        # otherwise cancel the programmatic-dependent-launch overlap everywhere
        one_step(timing if i == args.steps - 1 else None)
    t1.record(compute)
    barrier()
    clock_info = clocks.stop((host_t0, time.time()))
    elapsed = max_over_ranks(t0.elapsed_time(t1) / 1e3)
    flops = step_flops(layers) * args.steps
    value = flops / elapsed / 1e12
    gemm_time = sum(a.elapsed_time(b) for a, b, _ in timing) / 1e3
    gemm_flops = sum(f for _, _, f in timing)
    achieved = gemm_flops / gemm_time / 1e12
    status = ctx.status(clear=True)

    # the same stack as a dependent chain (N > 1: each linear waits for the
    # previous linear's gathered output)
    dependent = None
    if world > 1:
        dep_steps = max(1, min(args.steps, 3))
        with torch.cuda.stream(compute):
            one_step(dependent=True)
        barrier()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(compute)
        with torch.cuda.stream(compute):
            for _ in range(dep_steps):
                one_step(dependent=True)
        d1.record(compute)
        barrier()
        dsec = max_over_ranks(d0.elapsed_time(d1) / 1e3)
        dependent = {"value": round(step_flops(layers) * dep_steps / dsec / 1e12, 2), "unit": "TFLOPS",
                     "ms_per_step": round(1e3 * dsec / dep_steps, 3), "steps": dep_steps,
                     "note": "every linear waits until the previous linear's output is gathered on every rank "
                             "(no overlap of a transfer with the next linear)"}

    # end to end: pinned host inputs -> HBM, the stack, result -> pinned host
    h_xh = x_h.cpu().pin_memory()
    h_xf = x_f.cpu().pin_memory()
    last = y_all[("w2", (layers - 1) & 1)] if world > 1 else y_loc[("w2", (layers - 1) & 1)]
    h_y = torch.empty(last.shape, dtype=last.dtype, pin_memory=True)
    e2e_steps = max(1, min(args.steps, 3))
    barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(compute)
    with torch.cuda.stream(compute):
        for _ in range(e2e_steps):
            x_h.copy_(h_xh, non_blocking=True)
            x_f.copy_(h_xf, non_blocking=True)
            one_step()
            h_y.copy_(last, non_blocking=True)
    s1.record(compute)
    barrier()
    e2e_sec = max_over_ranks(s0.elapsed_time(s1) / 1e3)
    e2e_value = step_flops(layers) * e2e_steps / e2e_sec / 1e12

    parity = parity_check(raw_cache, names, layers, y_loc, y_all, x_h, x_f, world, rank, nloc,
                          "fused" if fused else "copy" if ce else "nccl", None)

    gather = None
    if world > 1 and not args.no_extras:
        gather = gather_measure(ctx, device, world, rank, m, nloc["w13"])
        ctx.set_push_fanout(args.push_streams)
        ctx.set_push_kernel(args.push_kernel)

    extras = {}
    cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        extras["gemv"] = gemv_measure(ctx, device, hbm_peak)
        extras["config1"] = config1_measure(ctx, device, tc_burst)
        extras["config3"] = config3_measure(ctx, device, tc_sustained)
        extras["config4_streamed"] = config4_stream(ctx, device)
        extras["epilogues"] = epilogue_measure(ctx, device)
        extras["loader"] = loader_measure(ctx, raw_cache)
        # bounded CPU sample: layer 0 at cpu_rows rows, repeated until >= 10 s of work
        linears, threads = make_cpu_linears(0), os.cpu_count() or 1
        cpu_rows = args.cpu_rows or M_TOKENS
        t = f = 0.0
        reps = 0
        while t < 10.0 and reps < 20:
            dt, df, kind = cpu_reference_sample(cpu_rows, linears, threads)
            t, f, reps = t + dt, f + df, reps + 1
        cpu = {"value": round(f / t / 1e12, 4), "unit": "TFLOPS", "cores": threads, "cpu": cpu_model(),
               "kind": kind,
               "sample": f"layer 0 of the stack (5 linears): the reference's decode_cpu_into->f32 + fp32 torch "
                         f"matmul at {cpu_rows} of {M_TOKENS} rows, {reps} repetitions, {t:.1f} s"}

    # DRAM bytes per GEMM launch from the committed ncu summary (mean over one layer)
    traffic = None
    tfile = ROOT / "profiles" / "gemm_pair_config5_layer.md"
    if tfile.exists():
        import re
        mt = re.search(r"traffic_bytes_per_launch_mean: (\d+)", tfile.read_text())
        traffic = int(mt.group(1)) if mt else None
    if rank == 0:
        peak = tc_sustained
        parallelism = ("single GPU" if world == 1 else
                       f"N-shard x{world}, all-gather fused into the GEMM epilogue (NVLink peer stores) + device "
                       f"flag barrier per linear" if fused else
                       f"N-shard x{world}, all-gather by " + push_engine(args)
                       + ", shard-major Y) beside the next GEMM + device flag barrier per layer" if ce else
                       f"N-shard x{world} + NCCL all-gather" + (f" ({reserve} SMs left to it)" if reserve else ""))
        cfg = workload_config(layers)
        cfg.update({"operands": "X fp16, W dequantised to fp16 in TMEM, fp32 accumulate, fp16 Y",
                    "ffn_form": ("SwiGLU: w1 / w3 as one weight, silu(w1 x) * w3 x in the GEMM epilogue"
                                 if args.ffn == "swiglu" else "w1, w3 as separate linears (no SwiGLU op)"),
                    "l2": "inputs larger than L2 (3 GB of packed weights streamed per step)",
                    "weight_buffers": f"{layers} distinct HBM buffers per tensor, contents cycle over "
                                      f"{DISTINCT_LAYERS} seeds"})
        line = {"metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(1e3 * elapsed / args.steps, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic", "config": cfg, "parallelism": parallelism,
                "headline_form": ("independent linears: each output's transfer overlaps the next linear"
                                  if world > 1 else "single GPU"),
                "gpu_launches": (len(timing) * (2 if fused else 1) + (layers if ce else 0)) * args.steps,
                "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                             "frac": round(achieved / peak, 4), "traffic": traffic,
                             "traffic_source": "ncu dram bytes per launch, mean over one layer's linears, from "
                                               "the committed capture profiles/gemm_pair_config5_layer.md",
                             "kernel": "pair_gemm_kernel (tcgen05 cta_group::2, A in TMEM)",
                             "peak_source": f"{peak_src} sustained"},
                "e2e": {"value": round(e2e_value, 2), "unit": "TFLOPS",
                        "h2d_bytes_per_step": int(h_xh.numel() * 2 + h_xf.numel() * 2),
                        "d2h_bytes_per_step": int(h_y.numel() * 2), "steps": e2e_steps},
                "parity": parity, "clocks": clock_info, "status_word": status}
        if dependent:
            line["dependent_chain"] = dependent
        if gather:
            line["gather_alone"] = gather
        if cpu:
            line["cpu_baseline"] = cpu
        line.update(extras)
        print(json.dumps(line), flush=True)
    for lw in weights:
        for wt in lw.values():
            wt.free()
    if pg is not None:
        del y_loc, y_all
        pg.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-rows", type=int, default=None,
                    help="rows of X in the CPU sample (default: 2048 per reference-arm step, all rows for cpu_baseline)")
    ap.add_argument("--no-extras", action="store_true", help="skip the GEMV and CPU-baseline legs")
    ap.add_argument("--gather", choices=["fused", "copy", "nccl"], default="copy",
                    help="N>1: all-gather fused into the GEMM epilogue (peer stores), pushed by the copy "
                         "engines beside the next GEMM, or NCCL after each GEMM")
    ap.add_argument("--ffn", choices=["swiglu", "separate"], default="swiglu",
                    help="FFN input projections: one SwiGLU-fused weight (silu(w1 x) * w3 x) or two plain linears")
    ap.add_argument("--leg", choices=["gemv", "config1", "config3", "config4", "epilogues", "loader"],
                    default=None, help="run only this measurement leg on GPU 0 and print its JSON (profiling)")
    ap.add_argument("--push-streams", type=int, default=0,
                    help="--gather copy: spread each output's peer copies over this many side streams "
                         "(0 / 1: back to back, the default)")
    ap.add_argument("--push-kernel", type=int, default=None,
                    help="--gather copy: push each output with a kernel of this many 128-thread blocks (SM stores "
                         "over NVLink) instead of the copy engines (0).  Default: 296 blocks at 8 GPUs, the copy "
                         "engines below (measured stack, TFLOP/s: 2 GPUs 1798 copy / 1617 kernel, 4 GPUs 3248 / "
                         "2466, 8 GPUs 2745 / 3078-3094 with 148 blocks, 3156 with 296)")
    ap.add_argument("--reserve-sms", type=int, default=None,
                    help="SMs kept free of the GEMM for the all-gather (default 0: measured no gain at N=2)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.push_kernel is None:
        args.push_kernel = 296 if args.gpus >= 8 else 0
    if args.leg:
        return run_leg(args)
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
