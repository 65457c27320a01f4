#!/usr/bin/env python
"""Benchmark of the quantized-matmul hot path on B200 (one JSON line).

Headline workload (the shape the reference's own CPU
kernel runs): the Llama-7B decode projection x f32 [1,4096] -> per-tensor
INT8 quantization -> W int8 [N=11008, K=4096] per-channel GEMV -> f32
[1,11008].  metric = weight GB/s (45,088,768 int8 weight bytes per call).

  step     = 256 independent decode-projection calls (256 distinct activation
             vectors), replayed from one CUDA graph; weights rotate over 16
             device copies (721 MB, 5.7x the 126 MB L2) so every call streams
             its weights from HBM.
  value    = weight bytes of all calls on all ranks / max-over-ranks time.
  e2e      = the same calls through the host-buffer C-ABI drop-in
             (mri_host_matmul_int8_from_f32): pinned x H2D, kernel, out D2H,
             stream sync, per call.
  roofline = algorithmic bytes per launch (weights + scales + x_q + out) /
             mean launch duration, against the measured HBM copy bandwidth.

Multi-GPU (torchrun): each rank runs its own projections (independent units,
no data-path collective; weak scaling).  `--impl reference` times the
reference's CPU path (C++ restatement of proj_int8_par: quantize_symmetric +
matmul_int8_parallel, forward_int8.rs:87-96) on the host cores, rank 0 only.
"""
import argparse
import ctypes
import datetime
import importlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (REPO, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

K_DIM, N_DIM = 4096, 11008
WEIGHT_BYTES = N_DIM * K_DIM                          # int8 weights per call
ALG_BYTES = WEIGHT_BYTES + 4 * N_DIM + K_DIM * 4 + 4 * N_DIM  # + scales + x f32 + out f32
CALLS_PER_STEP = 256
WEIGHT_COPIES = 16
REF_CALLS_PER_STEP = 4
WORKLOAD = ("decode projection [1,4096]x[4096,11008] int8 per-channel, "
            "per-tensor act quant (BASELINE config 0)")

THROTTLE_BITS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap", 0x2: "applications_clocks",
                 0x1: "gpu_idle", 0x10: "sync_boost"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the Q8_0 / Q4_0 / prefill side measurements")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the timed CPU sample (profiling runs)")
    ap.add_argument("--only", choices=["q8_0", "q4_0", "prefill", "model", "chain", "cpu", "sharded"],
                    help="run one side measurement alone and print it (profiling runs)")
    ap.add_argument("--model-layers", type=int, default=32,
                    help="layers of the Llama-7B-shaped model (profiling runs of its kernels on a "
                         "smaller device footprint; the reported config uses 32)")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def committed_traffic(kernel_key):
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(kernel_key)


class ClockSampler:
    """Polls NVML (SM clock + clock-event reasons) while the timed region runs."""

    def __init__(self, device, period_s=0.002):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - NVML missing: report no clocks
            self._nv = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                self.reasons |= int(self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nv is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return None
        names = [n for b, n in THROTTLE_BITS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": names}


def cpu_baseline_sample(seconds=10.0):
    """The reference's decode projection on the host (C++ restatement of
    proj_int8_par = quantize_symmetric + matmul_int8_parallel), bounded."""
    import oracle
    rng = np.random.default_rng(0)
    w = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    x = rng.normal(0, 1, size=K_DIM).astype(np.float32)
    out = np.empty((1, N_DIM), np.float32)
    threads = oracle.hardware_threads()
    calls, t0 = 0, time.perf_counter()
    while True:
        aq, s = oracle.quantize_symmetric(x)
        oracle.matmul_int8_parallel(aq, s, w, ws, N_DIM, K_DIM, 1, n_threads=threads, out=out)
        calls += 1
        el = time.perf_counter() - t0
        if (el >= seconds and calls >= 2) or el >= 3 * seconds:
            break
    return calls, el


def run_reference(args, rank):
    if rank != 0:
        return
    import oracle
    rng = np.random.default_rng(0)
    w = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    xs = rng.normal(0, 1, size=(REF_CALLS_PER_STEP, K_DIM)).astype(np.float32)
    out = np.empty((1, N_DIM), np.float32)
    threads = oracle.hardware_threads()

    def step():
        for i in range(REF_CALLS_PER_STEP):
            aq, s = oracle.quantize_symmetric(xs[i])
            oracle.matmul_int8_parallel(aq, s, w, ws, N_DIM, K_DIM, 1, n_threads=threads, out=out)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = args.steps * REF_CALLS_PER_STEP * WEIGHT_BYTES / el / 1e9
    sample = (f"{REF_CALLS_PER_STEP} decode projections [1,4096]x[4096,11008] per step; "
              f"matmul_int8_parallel at M=1 runs one row task (parallel.rs:334), so 1 of {threads} "
              f"host threads works")
    line = {
        "impl": "reference", "metric": "decode GEMV weight GB/s", "value": round(gbs, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8->int32->f32", "data": "synthetic (seed 0)",
        "config": {"workload": WORKLOAD,
                   "calls_per_step": REF_CALLS_PER_STEP},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def graph_of(torch, stream, fn):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def time_graph(torch, stream, g, steps, warmup):
    # CUDAGraph.replay() launches on the current stream: make it `stream`,
    # the one the events are recorded on.
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            g.replay()
        e1.record(stream)
        e1.synchronize()
    return e0.elapsed_time(e1)


SIDE_PARTS = ("q8_0", "q4_0", "prefill", "model", "chain", "cpu")


def decode_chain_measurement(torch, mri, lib, device, peak_hbm):
    """The headline decode projection [1,4096]x[4096,11008] in two more forms:
    independent calls with programmatic dependent launch off (each call's
    weight stream starts only after the previous call has finished), and a
    dependent chain, each call's input being the first 4096 outputs of the
    previous call (as consecutive projections of a decode step are), with PDL
    on and off.  Weights rotate over 16 copies as in the headline."""
    s = torch.cuda.Stream(device)
    ctx = mri.Context(device, stream=s)
    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    weights = [mri.QuantizedMatrix(wq, ws, N_DIM, K_DIM, ctx=ctx, keep_host=False) for _ in range(WEIGHT_COPIES)]
    calls = CALLS_PER_STEP
    x = torch.randn(calls, K_DIM, device=f"cuda:{device}")
    out = torch.empty(calls, N_DIM, device=f"cuda:{device}")
    res = {}
    for name, chained, pdl in (("independent_pdl_off", False, 0), ("chain_pdl_on", True, 1),
                               ("chain_pdl_off", True, 0)):
        ctx.set_option(mri.OPT_PDL, pdl)

        def body():
            for i in range(calls):
                src = out[i - 1].data_ptr() if chained and i > 0 else x[i].data_ptr()
                rc = lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(src), 1, K_DIM,
                                                  weights[i % WEIGHT_COPIES].handle,
                                                  ctypes.c_void_p(out[i].data_ptr()))
                if rc != 0:
                    raise RuntimeError(mri._lib.last_error())
        body()
        ctx.synchronize()
        g = graph_of(torch, s, body)
        reps = 10
        ms = time_graph(torch, s, g, reps, 3)
        del g
        t = ms / 1e3 / (reps * calls)
        res[name] = {"us_per_call": round(t * 1e6, 3), "weight_gbs": round(WEIGHT_BYTES / t / 1e9, 1),
                     "roofline_frac_hbm": round(ALG_BYTES / t / 1e9 / peak_hbm, 4)}
    ctx.set_option(mri.OPT_PDL, 1)
    res["note"] = ("value/roofline of the headline: independent calls with PDL on (a call's weight "
                   "prefetch overlaps the previous call's tail)")
    return res


def e2e_breakdown_measurement(torch, mri, lib, device):
    """Where the time of one host-buffer call of the headline projection goes
    (wall clock on the host, per call, weights rotating over 16 copies as in
    the e2e figure): a bare stream synchronisation, the device-pointer call
    plus synchronisation, the same after a pinned host-to-device copy of x,
    and the host-buffer entry point with pageable and with pinned buffers
    (the pinned output is written by a copy kernel instead of a copy)."""
    # The context runs on a stream torch owns: torch's pinned-memory allocator
    # records events on the streams its blocks were used on when they are
    # freed, so that stream must outlive the tensors.
    es = torch.cuda.Stream(device)
    ctx = mri.Context(device, stream=es)
    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    weights = [mri.QuantizedMatrix(wq, ws, N_DIM, K_DIM, ctx=ctx, keep_host=False) for _ in range(WEIGHT_COPIES)]
    x_np = rng.normal(0, 1, size=(1, K_DIM)).astype(np.float32)
    o_np = np.empty((1, N_DIM), np.float32)
    x_pin = torch.from_numpy(x_np).pin_memory()
    o_pin = torch.empty(1, N_DIM).pin_memory()
    x_dev = torch.empty(1, K_DIM, device=f"cuda:{device}")
    o_dev = torch.empty(1, N_DIM, device=f"cuda:{device}")
    state = {"i": 0}

    def w():
        state["i"] += 1
        return weights[state["i"] % WEIGHT_COPIES].handle

    def check(rc):
        if rc != 0:
            raise RuntimeError(mri._lib.last_error())

    def sync():
        check(lib.mri_ctx_synchronize(ctx.handle))

    def dev_call():
        check(lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(x_dev.data_ptr()), 1, K_DIM, w(),
                                           ctypes.c_void_p(o_dev.data_ptr())))

    def h2d_dev_call():
        with torch.cuda.stream(es):
            x_dev.copy_(x_pin, non_blocking=True)
        dev_call()

    def host(xp, op):
        check(lib.mri_host_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(xp), 1, K_DIM, w(), ctypes.c_void_p(op)))

    forms = (("sync_only", sync), ("device_call_sync", lambda: (dev_call(), sync())),
             ("h2d_device_call_sync", lambda: (h2d_dev_call(), sync())),
             ("host_call_pageable", lambda: host(x_np.ctypes.data, o_np.ctypes.data)),
             ("host_call_pinned", lambda: host(x_pin.data_ptr(), o_pin.data_ptr())))
    res = {}
    for name, fn in forms:
        for _ in range(50):
            fn()
        n = 500
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        res[name] = {"us_per_call": round((time.perf_counter() - t0) / n * 1e6, 2)}
    res["note"] = "host wall clock per call; the e2e figure is host_call_pinned over 256 calls per step"
    ctx.synchronize()
    return res


def cpu_side_baselines():
    """The reference's CPU implementations of the secondary configs, timed on
    this host through the C++ restatement (oracle), each a bounded sample:
    matmul_int8_parallel at the prefill shape on all host threads (one row
    task per thread, parallel.rs:308-346), the scalar matmul_q8_0_direct
    (q8_direct.rs:229-289) and matmul_q4_0_dequant (q4_0.rs:94-181) at M = 1
    and 8, and LlamaModelInt8::forward_decode (forward_int8.rs:538-546) at
    the 7B shape with proj_int8_par projections (the 32 layers share one set
    of weight arrays, which still stream from DRAM: 202 MB a layer)."""
    import oracle
    import llama_oracle
    threads = oracle.hardware_threads()
    res = {"cores_available": threads, "kind": "port"}
    rng = np.random.default_rng(1)
    # C3 prefill
    M = 512
    x = rng.normal(0, 1, size=(M, K_DIM)).astype(np.float32)
    wq = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    out = np.empty((M, N_DIM), np.float32)
    t0 = time.perf_counter()
    aq, s = oracle.quantize_symmetric(x)
    oracle.matmul_int8_parallel(aq, s, wq, ws, N_DIM, K_DIM, M, n_threads=threads, out=out)
    el = time.perf_counter() - t0
    res["prefill_m512"] = {"tops": round(2.0 * M * K_DIM * N_DIM / el / 1e12, 4), "s_per_call": round(el, 3),
                           "cores": threads, "sample": "1 call of quantize_symmetric + matmul_int8_parallel"}
    # C2 Q8_0 / Q4_0 (scalar, one thread)
    wf = rng.normal(0, 0.02, size=(N_DIM, K_DIM)).astype(np.float32)
    for fmt in ("q8_0", "q4_0"):
        wb = oracle.quantize_q8_0_matrix(wf, N_DIM, K_DIM) if fmt == "q8_0" else \
            oracle.quantize_q4_0_matrix(wf, N_DIM, K_DIM)
        for m in (1, 8):
            xm = rng.normal(0, 1, size=(m, K_DIM)).astype(np.float32)
            calls, t0 = 0, time.perf_counter()
            while True:
                if fmt == "q8_0":
                    oracle.matmul_q8_0_direct(xm, m, K_DIM, wb, N_DIM, K_DIM)
                else:
                    oracle.matmul_q4_0_dequant(xm, m, K_DIM, wb, N_DIM, K_DIM)
                calls += 1
                el = time.perf_counter() - t0
                if el >= 1.5:
                    break
            t = el / calls
            res[f"{fmt}_m{m}"] = {"weight_gbs": round(wb.size / t / 1e9, 3), "us_per_call": round(t * 1e6, 1),
                                  "cores": 1, "sample": f"{calls} calls (scalar, as the reference)"}
    del wf
    # C4 decode (7B shape)
    L, d, ffn, V, pos = 32, 4096, 11008, 32000, 576
    cfg = dict(n_layers=L, dim=d, n_heads=32, n_kv_heads=32, ffn_dim=ffn, vocab=V, max_seq=pos + 4,
               rope_base=10000.0, rms_eps=1e-5)

    def q(rows, cols):
        return (rng.integers(-127, 128, size=rows * cols, dtype=np.int8),
                rng.uniform(4e-4, 8e-4, size=rows).astype(np.float32))
    layer = dict(wq=q(d, d), wk=q(d, d), wv=q(d, d), wo=q(d, d), wgate=q(ffn, d), wup=q(ffn, d), wdown=q(d, ffn))
    w = dict(token_embd=rng.uniform(-1, 1, size=V * d).astype(np.float32), layers=[layer] * L,
             attn_norm=np.ones(L * d, np.float32), ffn_norm=np.ones(L * d, np.float32),
             output_norm=np.ones(d, np.float32), output=q(V, d))
    # The reference's decode step projects with the scalar proj_int8
    # (forward_int8.rs:333-346, :72-74).
    ref = llama_oracle.LlamaInt8Oracle(cfg, w, proj="scalar")
    ref.kc[:, :pos] = rng.normal(0, 1, size=(pos, d)).astype(np.float32)[None]
    ref.vc[:, :pos] = ref.kc[:, :pos]
    tokens, t0 = 0, time.perf_counter()
    while True:
        ref.forward_decode(7 + tokens, pos + tokens)
        tokens += 1
        el = time.perf_counter() - t0
        if el >= 2.0 or tokens == 3:
            break
    res["llama7b_int8_decode"] = {"tok_s": round(tokens / el, 3), "s_per_token": round(el / tokens, 3),
                                  "cores": 1,
                                  "sample": f"{tokens} decode tokens at position {pos}, scalar proj_int8 "
                                            "projections as the reference's forward_decode; one thread"}
    return res


def secondary_measurements(torch, mri, lib, device, peak_hbm, peak_tc, parts=SIDE_PARTS, model_layers=32):
    """Q8_0 / Q4_0 decode (M=1, M=8), the prefill GEMM and the 7B model, 1 GPU;
    the products from CUDA graphs over rotating weight copies."""
    res = {}
    rng = np.random.default_rng(0)
    wf = rng.normal(0, 0.02, size=(N_DIM, K_DIM)).astype(np.float32)
    s = torch.cuda.Stream(device)
    ctx = mri.Context(device, stream=s)
    for fmt in [f for f in ("q8_0", "q4_0") if f in parts]:
        wb = mri.formats.quantize_q8_0(wf, N_DIM, K_DIM) if fmt == "q8_0" else \
            mri.formats.quantize_q4_0(wf, N_DIM, K_DIM)
        copies = max(3, int(np.ceil(300e6 / wb.size)))
        ws = [mri.Q8_0WeightMatrix.from_raw_bytes(wb, N_DIM, K_DIM, ctx=ctx) if fmt == "q8_0"
              else mri.Q4_0Matrix(wb, N_DIM, K_DIM, ctx=ctx) for _ in range(copies)]
        fn = lib.mri_matmul_q8_0_direct if fmt == "q8_0" else lib.mri_matmul_q4_0_dequant
        for m in (1, 8):
            calls = 32
            x = torch.randn(calls, m, K_DIM, device=f"cuda:{device}", generator=None)
            out = torch.empty(calls, m, N_DIM, device=f"cuda:{device}")

            def body():
                for i in range(calls):
                    rc = fn(ctx.handle, ctypes.c_void_p(x[i].data_ptr()), m, K_DIM,
                            ws[i % copies].handle, ctypes.c_void_p(out[i].data_ptr()))
                    assert rc == 0, mri._lib.last_error()
            body()
            ctx.synchronize()
            g = graph_of(torch, s, body)
            ms = time_graph(torch, s, g, 20, 3)
            per_call_s = ms / 1e3 / (20 * calls)
            alg = wb.size + m * K_DIM * 4 + m * N_DIM * 4
            res[f"{fmt}_m{m}"] = {"weight_gbs": round(wb.size / per_call_s / 1e9, 1),
                                  "us_per_call": round(per_call_s * 1e6, 3),
                                  "roofline_frac_hbm": round(alg / per_call_s / 1e9 / peak_hbm, 4)}
            del g
        del ws
    # Prefill GEMM [512,4096] x [4096,11008]^T
    try:
        if "prefill" not in parts:
            raise LookupError
        M = 512
        wq = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
        wsc = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
        copies = 3
        qms = [mri.QuantizedMatrix(wq, wsc, N_DIM, K_DIM, ctx=ctx, keep_host=False) for _ in range(copies)]
        x = torch.randn(M, K_DIM, device=f"cuda:{device}")
        out = torch.empty(M, N_DIM, device=f"cuda:{device}")
        path = ctx.int8_path(M, N_DIM, K_DIM)

        def body():
            for i in range(copies):
                rc = lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(x.data_ptr()), M, K_DIM,
                                                  qms[i].handle, ctypes.c_void_p(out.data_ptr()))
                assert rc == 0, mri._lib.last_error()
        body()
        ctx.synchronize()
        g = graph_of(torch, s, body)
        ms = time_graph(torch, s, g, 10, 2)
        per_call_s = ms / 1e3 / (10 * copies)
        tops = 2.0 * M * K_DIM * N_DIM / per_call_s / 1e12
        del g
        # The GEMM kernel alone: activations already quantized (device scale).
        xq = torch.randint(-127, 128, (M, K_DIM), dtype=torch.int8, device=f"cuda:{device}")
        sc = torch.tensor([0.01], device=f"cuda:{device}")

        def body_q():
            for i in range(copies):
                rc = lib.mri_matmul_int8_dscale(ctx.handle, ctypes.c_void_p(xq.data_ptr()), M * K_DIM,
                                                ctypes.c_void_p(sc.data_ptr()), 0, qms[i].handle, M,
                                                ctypes.c_void_p(out.data_ptr()), None)
                assert rc == 0, mri._lib.last_error()
        body_q()
        ctx.synchronize()
        g = graph_of(torch, s, body_q)
        ms_k = time_graph(torch, s, g, 10, 2)
        del g
        kern_s = ms_k / 1e3 / (10 * copies)
        kern_tops = 2.0 * M * K_DIM * N_DIM / kern_s / 1e12

        # Per-row activation quantization (BASELINE config 2 names it).
        def body_r():
            for i in range(copies):
                rc = lib.mri_matmul_int8_from_f32_g(ctx.handle, ctypes.c_void_p(x.data_ptr()), M, K_DIM,
                                                    mri.PER_ROW, qms[i].handle, ctypes.c_void_p(out.data_ptr()))
                assert rc == 0, mri._lib.last_error()
        body_r()
        ctx.synchronize()
        g = graph_of(torch, s, body_r)
        ms_r = time_graph(torch, s, g, 10, 2)
        del g
        row_s = ms_r / 1e3 / (10 * copies)
        row_tops = 2.0 * M * K_DIM * N_DIM / row_s / 1e12
        res["prefill_m512"] = {"tops": round(tops, 2), "us_per_call": round(per_call_s * 1e6, 2),
                               "path": {0: "stream-gemv", 1: "generic-gemv", 2: "tcgen05-gemm"}[path],
                               "roofline_frac_int8": round(tops / (2 * peak_tc), 4),
                               "gemm_kernel_tops": round(kern_tops, 2),
                               "gemm_kernel_us": round(kern_s * 1e6, 2),
                               "gemm_kernel_frac_int8": round(kern_tops / (2 * peak_tc), 4),
                               "per_row_tops": round(row_tops, 2), "per_row_us_per_call": round(row_s * 1e6, 2),
                               "per_row_frac_int8": round(row_tops / (2 * peak_tc), 4),
                               "int8_peak_note": "int8 dense peak taken as 2x measured bf16; "
                                                 "tops includes the activation quantizer"}
    except LookupError:
        pass
    except Exception as e:  # noqa: BLE001 - side measurement only
        res["prefill_m512"] = {"error": str(e)[:200]}
    ctx.synchronize()
    if "model" in parts:
        res["llama7b_int8"] = model_measurement(mri, device, peak_hbm, model_layers)
    if "chain" in parts:
        try:
            res["decode_gemv_forms"] = decode_chain_measurement(torch, mri, lib, device, peak_hbm)
        except Exception as e:  # noqa: BLE001 - side measurement only
            res["decode_gemv_forms"] = {"error": str(e)[:200]}
        try:
            res["e2e_breakdown"] = e2e_breakdown_measurement(torch, mri, lib, device)
        except Exception as e:  # noqa: BLE001 - side measurement only
            res["e2e_breakdown"] = {"error": str(e)[:200]}
    if "cpu" in parts:
        try:
            res["cpu_baselines"] = cpu_side_baselines()
        except Exception as e:  # noqa: BLE001 - side measurement only
            res["cpu_baselines"] = {"error": str(e)[:200]}
    return res


def model_measurement(mri, device, peak_hbm, layers=32):
    """Llama-7B-shaped LlamaModelInt8 (32 layers, d=4096,
    32 heads, FFN 11008, vocab 32000), synthetic weights generated on the
    device, 512-token prefill then 128 greedy decode steps (CUDA graph per
    step).  The second of two runs is reported."""
    try:
        L, d, ffn, V = layers, 4096, 11008, 32000
        cfg = mri.LlamaConfig(L, d, 32, ffn, V, 640)
        m = mri.LlamaModelInt8.random(cfg, seed=1, ctx=mri.Context(device))
        prompt = np.random.default_rng(0).integers(0, V, size=512).astype(np.uint32)
        for _ in range(2):
            toks, pre_ms, dec_ms = m.generate_greedy(prompt, 128)
        w_bytes = L * (3 * d * d + d * d + 2 * ffn * d + d * ffn) + V * d
        kv_bytes = L * 2 * (512 + 64) * d * 4  # mean cached positions per step
        step_s = dec_ms / 1e3 / 128
        res = {"prefill_tok_s": round(512 / (pre_ms / 1e3), 1), "decode_tok_s": round(128 / (dec_ms / 1e3), 1),
               "prefill_ms": round(pre_ms, 3), "decode_ms_per_token": round(step_s * 1e3, 4),
               "decode_roofline_frac_hbm": round((w_bytes + kv_bytes) / step_s / 1e9 / peak_hbm, 4),
               "decode_bytes_per_token": w_bytes + kv_bytes,
               "kernels_per_decode_step": m.kernels_per_decode_step(),
               "data": "synthetic weights (device hash RNG), random prompt (seed 0)"}
        del m
        return res
    except Exception as e:  # noqa: BLE001 - side measurement only
        return {"error": str(e)[:300]}


def sharded_measurement(torch, mri, device, world, dist, peak_hbm, peak_tc):
    """Llama-70B FFN projections, W int8 gate/up [28672, 8192]
    and down [8192, 28672] with per-channel scales, N-sharded over the ranks
    (rank r holds rows [r*N/P, (r+1)*N/P)); each call returns the full [M, N]
    f32 product on every rank through mri_sharded_matmul_int8_from_f32
    (per-shard kernels + NCCL all-gather).  M=1 calls are replayed from a CUDA
    graph over rotating weight copies (> 300 MB per rank, so shards stream
    from HBM); M=2048 calls are timed eagerly.  Times are max over ranks."""
    s = torch.cuda.Stream(device)
    ctx = mri.Context(device, stream=s)
    comm = mri.Communicator.from_process_group(ctx=ctx) if world > 1 else \
        mri.Communicator(mri.Communicator.unique_id(), 1, 0, ctx=ctx)
    lib = ctx._lib
    res = {"P": world, "collective": "M = 1: NCCL all-gather of f32 [M, N/P] slices; M = 2048: each "
                                    "rank's GEMM epilogue writes its tiles to every rank over NVLink",
           "data": "synthetic int8 weights, x ~ N(0,1)"}
    rng = np.random.default_rng(comm.rank)

    def max_ms(ms):
        if dist is None:
            return ms
        t = torch.tensor([ms], device=f"cuda:{device}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for name, (N, K) in {"gate_up": (28672, 8192), "down": (8192, 28672)}.items():
        ns = N // world
        shard_bytes = ns * K
        wq = rng.integers(-127, 128, size=shard_bytes, dtype=np.int8)
        ws = rng.uniform(0.001, 0.02, size=ns).astype(np.float32)
        copies = max(2, int(np.ceil(300e6 / shard_bytes)))
        mats = [mri.QuantizedMatrix(wq, ws, ns, K, ctx=ctx, keep_host=False) for _ in range(copies)]
        del wq
        # M = 1 (decode)
        calls = 2 * copies
        x = torch.randn(calls, K, device=f"cuda:{device}")
        out = torch.empty(calls, N, device=f"cuda:{device}")

        def body():
            for i in range(calls):
                rc = lib.mri_sharded_matmul_int8_from_f32(comm.handle, ctypes.c_void_p(x[i].data_ptr()), 1, K,
                                                          mats[i % copies].handle, N,
                                                          ctypes.c_void_p(out[i].data_ptr()))
                if rc != 0:
                    raise RuntimeError(mri._lib.last_error())
        body()
        comm.wait()
        if dist is not None:
            dist.barrier()
        g = graph_of(torch, s, body)
        reps = 10
        ms = max_ms(time_graph(torch, s, g, reps, 3))
        del g
        t = ms / 1e3 / (reps * calls)
        res[f"{name}_m1"] = {"us_per_call": round(t * 1e6, 3),
                             "weight_gbs_aggregate": round(N * K / t / 1e9, 1),
                             "weight_gbs_per_gpu": round(shard_bytes / t / 1e9, 1),
                             "frac_hbm_per_gpu": round(shard_bytes / t / 1e9 / peak_hbm, 4),
                             "gather_bytes_per_rank": 4 * N}
        del x, out
        # M = 2048 (prefill)
        M = 2048
        x = torch.randn(M, K, device=f"cuda:{device}")
        out = torch.empty(M, N, device=f"cuda:{device}")

        def call(i):
            rc = lib.mri_sharded_matmul_int8_from_f32(comm.handle, ctypes.c_void_p(x.data_ptr()), M, K,
                                                      mats[i % copies].handle, N, ctypes.c_void_p(out.data_ptr()))
            if rc != 0:
                raise RuntimeError(mri._lib.last_error())
        call(0)
        comm.wait()
        if dist is not None:
            dist.barrier()
        reps = 6
        with torch.cuda.stream(s):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for i in range(reps):
                call(i)
            e1.record(s)
        comm.wait()
        ms = max_ms(e0.elapsed_time(e1))
        t = ms / 1e3 / reps
        ops = 2.0 * M * N * K
        res[f"{name}_m2048"] = {"ms_per_call": round(t * 1e3, 4),
                                "tops_aggregate": round(ops / t / 1e12, 2),
                                "tops_per_gpu": round(ops / world / t / 1e12, 2),
                                "frac_int8_per_gpu": round(ops / world / t / 1e12 / (2 * peak_tc), 4),
                                "gather_bytes_per_rank": 4 * M * N}
        if world > 1:
            # The same call gathered by NCCL (OPT_SHARD_PEER = 0): the chunked
            # all-gather of f32 slices and the unshard copy.
            ctx.set_option(mri.OPT_SHARD_PEER, 0)
            call(0)
            comm.wait()
            dist.barrier()
            with torch.cuda.stream(s):
                e0.record(s)
                for i in range(reps):
                    call(i)
                e1.record(s)
            comm.wait()
            ctx.set_option(mri.OPT_SHARD_PEER, 2)
            tp = max_ms(e0.elapsed_time(e1)) / 1e3 / reps
            res[f"{name}_m2048"]["nccl_allgather"] = {"ms_per_call": round(tp * 1e3, 4),
                                                      "tops_aggregate": round(ops / tp / 1e12, 2)}
        # Components of one call, each timed alone (max over ranks): the
        # rank's shard product, and an NCCL all-gather of the same f32 bytes.
        if world > 1:
            out_s = torch.empty(M, ns, device=f"cuda:{device}")

            def shard_call(i):
                rc = lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(x.data_ptr()), M, K,
                                                  mats[i % copies].handle, ctypes.c_void_p(out_s.data_ptr()))
                if rc != 0:
                    raise RuntimeError(mri._lib.last_error())
            shard_call(0)
            ctx.synchronize()
            dist.barrier()
            with torch.cuda.stream(s):
                e0.record(s)
                for i in range(reps):
                    shard_call(i)
                e1.record(s)
            ctx.synchronize()
            gemm_ms = max_ms(e0.elapsed_time(e1)) / reps
            flat = out_s.reshape(-1)
            gathered = torch.empty(world * flat.numel(), device=f"cuda:{device}")
            dist.all_gather_into_tensor(gathered, flat)
            torch.cuda.synchronize()
            dist.barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cur = torch.cuda.current_stream(device)
            g0.record(cur)
            for _ in range(reps):
                dist.all_gather_into_tensor(gathered, flat)
            g1.record(cur)
            torch.cuda.synchronize()
            ag_ms = max_ms(g0.elapsed_time(g1)) / reps
            res[f"{name}_m2048"]["components_ms"] = {"shard_gemm": round(gemm_ms, 4),
                                                     "allgather_alone": round(ag_ms, 4)}
            del out_s, gathered
        del x, out, mats
        torch.cuda.empty_cache()
    comm.close()
    return res


def run_ours(args, rank, world, local_rank):
    import torch
    mri = importlib.import_module("mini-rust-inference_b200")
    lib = mri._lib.load()
    device = local_rank
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{device}"))
    peak_hbm, peak_tc, peak_kind = measured_peaks()
    if args.only:
        if args.only == "sharded":
            out = sharded_measurement(torch, mri, device, world, dist, peak_hbm, peak_tc)
        else:
            out = secondary_measurements(torch, mri, lib, device, peak_hbm, peak_tc, parts=(args.only,),
                                         model_layers=args.model_layers)
        if rank == 0:
            print(json.dumps({"only": args.only, "n_gpus": world, "result": out}), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    rng = np.random.default_rng(0)
    wq = rng.integers(-127, 128, size=N_DIM * K_DIM, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=N_DIM).astype(np.float32)
    xs_host = rng.normal(0, 1, size=(CALLS_PER_STEP, K_DIM)).astype(np.float32)

    s = torch.cuda.Stream(device)
    ctx = mri.Context(device, stream=s)
    weights = [mri.QuantizedMatrix(wq, ws, N_DIM, K_DIM, ctx=ctx, keep_host=False)
               for _ in range(WEIGHT_COPIES)]
    x = torch.from_numpy(xs_host).to(f"cuda:{device}")
    out = torch.empty(CALLS_PER_STEP, N_DIM, device=f"cuda:{device}")
    xp, op = x.data_ptr(), out.data_ptr()

    def body():
        for i in range(CALLS_PER_STEP):
            rc = lib.mri_matmul_int8_from_f32(ctx.handle, ctypes.c_void_p(xp + i * K_DIM * 4), 1, K_DIM,
                                              weights[i % WEIGHT_COPIES].handle,
                                              ctypes.c_void_p(op + i * N_DIM * 4))
            if rc != 0:
                raise RuntimeError(mri._lib.last_error())

    body()
    ctx.synchronize()
    ctx.check_device_status()
    n0 = ctx.launch_count
    g = graph_of(torch, s, body)
    launches_per_step = ctx.launch_count - n0

    with torch.cuda.stream(s):  # replay() launches on the current stream
        for _ in range(args.warmup):
            g.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clk, torch.cuda.stream(s):
        e0.record(s)
        for _ in range(args.steps):
            g.replay()
        e1.record(s)
        e1.synchronize()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=f"cuda:{device}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ctx.check_device_status()
    del g

    calls = args.steps * CALLS_PER_STEP
    value = world * calls * WEIGHT_BYTES / (ms / 1e3) / 1e9
    launch_s = ms / 1e3 / calls
    achieved = ALG_BYTES / launch_s / 1e9

    # e2e: host buffers through the synchronous C-ABI drop-in, per call.
    ctx_e2e = mri.Context(device)
    xh = torch.from_numpy(xs_host).pin_memory()
    oh = torch.empty(CALLS_PER_STEP, N_DIM).pin_memory()
    xhp, ohp = xh.data_ptr(), oh.data_ptr()
    e2e_steps = max(1, min(args.steps, 20))

    def e2e_step():
        for i in range(CALLS_PER_STEP):
            rc = lib.mri_host_matmul_int8_from_f32(ctx_e2e.handle, ctypes.c_void_p(xhp + i * K_DIM * 4), 1,
                                                   K_DIM, weights[i % WEIGHT_COPIES].handle,
                                                   ctypes.c_void_p(ohp + i * N_DIM * 4))
            if rc != 0:
                raise RuntimeError(mri._lib.last_error())
    e2e_step()
    es = torch.cuda.ExternalStream(ctx_e2e.stream_handle, device=f"cuda:{device}")
    if dist:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(es)
    for _ in range(e2e_steps):
        e2e_step()
    f1.record(es)
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    if dist:
        t = torch.tensor([e2e_ms], device=f"cuda:{device}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * e2e_steps * CALLS_PER_STEP * WEIGHT_BYTES / (e2e_ms / 1e3) / 1e9

    secondary = None
    if world == 1 and not args.no_secondary:
        parts = tuple(p for p in SIDE_PARTS if p != "cpu" or not args.no_cpu_baseline)
        secondary = secondary_measurements(torch, mri, lib, device, peak_hbm, peak_tc, parts=parts)
    sharded = None
    if not args.no_secondary:
        try:
            sharded = sharded_measurement(torch, mri, device, world, dist, peak_hbm, peak_tc)
        except Exception as e:  # noqa: BLE001 - side measurement only
            sharded = {"error": str(e)[:300]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        calls_c, el = cpu_baseline_sample()
        cpu = {"value": round(calls_c * WEIGHT_BYTES / el / 1e9, 4), "unit": "GB/s", "cores": 1,
               "kind": "port",
               "sample": f"{calls_c} decode projections in {el:.1f}s: quantize_symmetric + "
                         f"matmul_int8_parallel restated in C++ (AVX2 maddubs dot); M=1 gives one "
                         f"row task, so 1 of {oracle.hardware_threads()} host threads works"}

    if rank == 0:
        line = {
            "metric": "decode GEMV weight GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8->int32->f32", "data": "synthetic (seed 0)",
            "config": {"workload": WORKLOAD,
                       "calls_per_step": CALLS_PER_STEP, "parallelism": f"replicas x{world}",
                       "l2": f"weights rotate over {WEIGHT_COPIES} copies "
                             f"({WEIGHT_COPIES * WEIGHT_BYTES / 1e6:.0f} MB > 2x L2)",
                       "graph": "one CUDA graph per step"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_hbm, "unit": "GB/s",
                         "frac": round(achieved / peak_hbm, 4), "peak_kind": peak_kind,
                         "bytes_per_launch": ALG_BYTES,
                         "traffic": committed_traffic("gemv_i8_tma_decode")},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": CALLS_PER_STEP * K_DIM * 4,
                    "d2h_bytes_per_step": CALLS_PER_STEP * N_DIM * 4},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        if secondary is not None:
            line["secondary"] = secondary
        if sharded is not None:
            line["sharded_70b_ffn"] = sharded
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    rank, world, local_rank = dist_env()
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
