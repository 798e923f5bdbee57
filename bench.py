"""Benchmark of the B200 embedding forward and its CPU baseline.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload embed|gemm|search]

Default workload: EmbeddingGemma-300M-shaped Q8_0 forward, 1024 sequences x 512
tokens per GPU (weak scaling: every rank runs its own 1024 sequences, no
collective on the data path), synthetic GGUF weights and seeded token ids.
One JSON line on rank 0. `value` is device-timed (inputs resident in HBM,
CUDA events on the library's stream, max over ranks); `e2e` goes through the
public host API (sem_embed) with pinned host ids and the host copy of the
embeddings inside the timed region.

--impl reference times the CPU restatement of the reference Go path (oracle/,
the reference itself cannot be built here: no Go toolchain) with all host
threads on a bounded sample of the same workload.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "go-semantica_b200"))

import synth  # noqa: E402

METRIC = "embeddings/sec @512 tok"
UNIT = "embeddings/s"
SEQ_LEN = 512
BATCH = 1024
MODEL_DIR = os.environ.get("SEM_BENCH_MODEL_DIR", "/tmp/semantica_b200_bench")
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "roofline_traffic.json")


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": f"EmbeddingGemma-300M Q8_0 forward, {BATCH} seqs x {SEQ_LEN} tokens per GPU (BASELINE config 3), "
                    "768-dim pooled output (512/256/128 are its renormalised prefixes)",
        "model": "synthetic GGUF with EmbeddingGemma-300M shapes (24 layers, hidden 768, FFN 1152, 3q/1kv heads, "
                 "head_dim 256, vocab 262144)",
        "global_batch": BATCH * n_gpus,
        "seq_len": SEQ_LEN,
        "parallelism": f"dp{n_gpus}",
        "l2": "inputs larger than L2: every layer's activations (1.6 GB per fp32 hidden-size tensor) stream through "
              "HBM, about 550 GB of element-wise traffic and 0.4 GB of weight planes per step",
    }


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) < 9:
                    continue
                if self.uuid and p[1] != self.uuid:
                    continue
                rows.append(p)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (C restatement of the reference Go path)
# ---------------------------------------------------------------------------
def cpu_baseline(model_path: str) -> dict:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the CPU baseline leg is one of the places allowed to run the oracle
    threads = max(1, min(os.cpu_count() or 1, 32))
    n_seq = threads
    m = oracle.OracleModel(model_path)
    ids, offs = synth.token_batch(4242, [SEQ_LEN] * n_seq, m.config.vocab_size)
    t0 = time.perf_counter()
    m.forward_batch(ids, offs, 768, nthreads=threads)
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n_seq / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_seq} sequences x {SEQ_LEN} tokens, one per thread ({dt:.1f} s); C restatement of the "
                      "reference Go INT8 forward (oracle/semantica_oracle.c)"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = synth.cached_gguf(MODEL_DIR, seed=1234)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = max(1, min(os.cpu_count() or 1, 64))
    m = oracle.OracleModel(path)
    # bounded sample per step: one 512-token sequence per host thread
    ids, offs = synth.token_batch(4242, [SEQ_LEN] * threads, m.config.vocab_size)
    for _ in range(args.warmup if args.warmup <= 1 else 1):
        m.forward_batch(ids[: offs[1]], offs[:2], 768, nthreads=1)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        m.forward_batch(ids, offs, 768, nthreads=threads)
        times.append(time.perf_counter() - t0)
    m.close()
    per = statistics.median(times)
    value = threads / per
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": workload_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{threads} sequences x {SEQ_LEN} tokens per step, one per thread; C "
                                       "restatement of the reference Go path (Go is not installed)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def stage_roofline(stage: str, total_ms: float, launches: int, T: int, n_seqs: int, peaks: dict) -> dict:
    H, F, nh, hd = 768, 1152, 3, 256
    per_ms = total_ms / max(launches, 1)
    gemm = {"gemm_q8_qkv": (H, nh * hd + 2 * hd, nh * hd + 2 * hd), "gemm_q8_o": (H, H, H),
            "gemm_q8_gate_up": (H, 2 * F, F), "gemm_q8_down": (F, H, H)}
    if stage in gemm:
        K, N, Nout = gemm[stage]
        flops = 2.0 * T * N * K
        achieved = flops / (per_ms * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained") or 1415.9
        return {"kernel": stage, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained (the projections run "
                "kind::f16 MMAs, the bf16 rate; algorithmic FLOPs: the hi and lo planes execute twice that)", "algorithmic_flops_per_launch": flops,
                "launch_ms": per_ms}
    if stage == "attention":
        S = T // n_seqs
        flops = n_seqs * 4.0 * S * S * hd * nh  # scores + P.V of the reference (attention.go:267-310)
        achieved = flops / (per_ms * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained") or 1415.9
        return {"kernel": stage, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained",
                "algorithmic_flops_per_launch": flops, "launch_ms": per_ms}
    # per-launch averages over a forward: quantize runs once on the first
    # attention norm and per layer on the attention output (K = H) and on the
    # MLP product (K = F), fp32 in and fp16 codes out; the residual kernel
    # reads o and hidden, writes hidden, and in all but the last of its 2 L
    # launches also writes the next norm's fp16 codes
    L = 24
    bytes_per_row = {"quantize": 6.0 * ((L + 1) * H + L * F) / (2 * L + 1),
                     "residual_norm": 3 * 4 * H + 2.0 * H * (2 * L - 1) / (2 * L), "row_stats": 4 * H,
                     "qk_norm_rope": 4 * (nh * hd + 2 * hd) + 2 * 2 * (nh * hd + 2 * hd), "embed": 4 * H + H,
                     "pool_l2": 4 * H}.get(stage, 4 * H)
    b = bytes_per_row * T
    achieved = b / (per_ms * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs") or 6650.0
    return {"kernel": stage, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "algorithmic_bytes_per_launch": b, "launch_ms": per_ms}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)

    import _lib
    import runtime

    if world > 1 and local != 0:
        dist.barrier()
    path = synth.cached_gguf(MODEL_DIR, seed=1234)
    if world > 1 and local == 0:
        dist.barrier()

    ctx = _lib.Context(local)
    model = runtime.load_model(path, ctx)
    stream = torch.cuda.ExternalStream(ctx.stream)
    lengths = [SEQ_LEN] * BATCH
    ids_h, offs = synth.token_batch(1000 + rank, lengths, model.config().vocab_size)
    T = int(offs[-1])
    d_ids = torch.from_numpy(ids_h).cuda()
    d_out = torch.empty((BATCH, 768), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step():
        model.embed_device(d_ids.data_ptr(), offs, BATCH, 768, d_out.data_ptr(), ctx.stream)

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-timed value ----
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps

    # ---- per-kernel timing inside the same kind of steps ----
    model.profile(True)
    for _ in range(args.steps):
        step()
    stages = model.profile_read()
    model.profile(False)
    clk = clocks.stop()

    # ---- e2e through the host API (pinned ids in, embeddings out) ----
    pinned = torch.empty(T, dtype=torch.int32, pin_memory=True)
    pinned.numpy()[:] = ids_h
    host_ids = pinned.numpy()
    out_pinned = torch.empty(BATCH * 768, dtype=torch.float32, pin_memory=True).numpy()
    import ctypes as C
    lib = _lib.load()
    dims = np.full(BATCH, 768, dtype=np.int32)
    offs32 = np.ascontiguousarray(offs, dtype=np.int32)

    def e2e_step():
        _lib.check(lib.sem_embed(model.handle, host_ids.ctypes.data, offs32.ctypes.data, BATCH, dims.ctypes.data,
                                 out_pinned.ctypes.data))

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    n_e2e = max(1, min(args.steps, 3))
    for _ in range(n_e2e):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / n_e2e
    barrier()

    # ---- small batch latency (8 x 64 tokens, 768-dim) ----
    # through sem_embed, which replays a CUDA graph of the forward once the
    # shape repeats
    small = None
    if world == 1:
        s_ids, s_offs = synth.token_batch(77, [64] * 8, model.config().vocab_size)
        s_ids = np.ascontiguousarray(s_ids, dtype=np.int32)
        s_offs = np.ascontiguousarray(s_offs, dtype=np.int32)
        s_dims = np.full(8, 768, dtype=np.int32)
        s_out = np.empty(8 * 768, dtype=np.float32)

        def small_call():
            _lib.check(lib.sem_embed(model.handle, s_ids.ctypes.data, s_offs.ctypes.data, 8, s_dims.ctypes.data,
                                     s_out.ctypes.data))

        for _ in range(5):
            small_call()
        n_small = 50
        t0 = time.perf_counter()
        for _ in range(n_small):
            small_call()
        small_ms = (time.perf_counter() - t0) / n_small * 1e3
        small = {"config": "BASELINE config 1: 8 sequences x 64 tokens, 768-dim, host ids in and embeddings out "
                           "through sem_embed (wall clock per call, CUDA graph replay)",
                 "ms_per_call": small_ms, "embeddings_per_s": 8 / (small_ms * 1e-3)}

    # max over ranks
    t = torch.tensor([ms, e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_s = float(t[0]), float(t[1])

    if rank == 0:
        peaks = {}
        if os.path.exists(PEAKS_PATH):
            peaks = json.load(open(PEAKS_PATH))
        dom = max(stages.items(), key=lambda kv: kv[1][0])
        roof = stage_roofline(dom[0], dom[1][0], dom[1][1], T, BATCH, peaks)
        traffic = None
        if os.path.exists(TRAFFIC_PATH):
            tr = json.load(open(TRAFFIC_PATH))
            traffic = tr.get(dom[0])
        roof["traffic"] = traffic
        roof["stages_ms_per_step"] = {k: round(v[0] / args.steps, 3) for k, v in stages.items()}
        launches_per_step = sum(v[1] for v in stages.values()) // max(args.steps, 1)
        line = {
            "metric": METRIC, "value": BATCH * world / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": workload_config(world), "clocks": clk,
            "e2e": {"value": BATCH * world / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(T * 4 + (BATCH + 1) * 4),
                    "d2h_bytes_per_step": int(BATCH * 768 * 4)},
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": roof,
        }
        if small:
            line["small_batch"] = small
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(path)
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# --workload gemm: BASELINE config 2, the isolated Q8_0 x activation projection
# ---------------------------------------------------------------------------
GEMM_SHAPES = [(768, 768, "q/o"), (768, 256, "k/v"), (768, 1152, "gate/up"), (1152, 768, "down"),
               (768, 3072, "dense up"), (3072, 768, "dense down")]
GEMM_M = [1, 64, 512, 4096, 32768]
GEMM_HEAD_M = 32768
GEMM_METRIC = "Q8_0 projection TFLOP/s (kernel on pre-quantised activations, 6 model shapes, M=32768)"


def gemm_config(n_gpus: int) -> dict:
    return {"workload": "BASELINE config 2: MatMulQ8_0INT8 on the model's projection shapes (K x N = "
                        + ", ".join(f"{k}x{n}" for k, n, _ in GEMM_SHAPES) + f"), M in {GEMM_M}",
            "weights": "int8 uniform [-127,127], fp16 block scales |N(0,0.02)| max/127",
            "activations": "fp32 N(0,1), one quantisation scale per call", "parallelism": f"replicas x{n_gpus}",
            "l2": "L2 flushed (256 MB write) before every timed launch"}


def gemm_algorithmic(K: int, N: int, M: int, prequant: bool) -> tuple[float, float]:
    """FLOPs and algorithmic bytes of one call: A (fp32, or its int8 codes), the
    34-byte-per-32 Q8_0 weight, fp32 C."""
    a_bytes = M * K * (1 if prequant else 4)
    return 2.0 * M * K * N, a_bytes + 34.0 / 32.0 * K * N + 4.0 * M * N


def gemm_cpu_baseline(rows_per_thread: int = 1536) -> dict:
    """The oracle's MatMulQ8_0INT8 restatement on every host thread: each thread
    takes its own slice of rows of each config-2 shape (ctypes releases the GIL)."""
    import concurrent.futures as cf
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the CPU baseline leg is one of the places allowed to run the oracle
    threads = max(1, min(os.cpu_count() or 1, 64))
    rng = np.random.default_rng(77)
    work = []
    for K, N, _ in GEMM_SHAPES:
        raw = synth.q8_0_blocks(rng, N, K)
        codes, scale = oracle.quantize_sym_int8(rng.standard_normal((rows_per_thread * threads, K)).astype(np.float32))
        work.append((raw, codes, scale, N, K))
    flops = sum(2.0 * c.shape[0] * K * N for _, c, _, N, K in work)
    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as ex:
        futs = [ex.submit(oracle.matmul_q8_0_int8, raw, codes[i * rows_per_thread:(i + 1) * rows_per_thread], scale, N)
                for raw, codes, scale, N, _ in work for i in range(threads)]
        for f in futs:
            f.result()
    dt = time.perf_counter() - t0
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows_per_thread} rows per thread x {threads} threads on each of the 6 shapes ({dt:.1f} s); "
                      "C restatement of MatMulQ8_0INT8 (oracle/semantica_oracle.c)"}


def run_gemm_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    times = []
    cb = None
    for _ in range(max(args.steps, 1)):
        cb = gemm_cpu_baseline()
        times.append(cb["value"])
    value = statistics.median(times)
    cb["value"] = value
    print(json.dumps({"metric": GEMM_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
                      "config": gemm_config(args.gpus), "cpu_baseline": cb,
                      "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def run_gemm(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    import _lib
    import runtime

    ctx = _lib.Context(local)
    stream = torch.cuda.ExternalStream(ctx.stream)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2
    peaks = json.load(open(PEAKS_PATH)) if os.path.exists(PEAKS_PATH) else {}
    tc_peak = peaks.get("bf16_tflops") or 1590.0
    bw_peak = peaks.get("hbm_gbs") or 6650.0
    rng = np.random.default_rng(2 + rank)
    results = {}
    head_flops = head_ms = 0.0
    head_e2e_s = 0.0
    h2d = d2h = 0
    launches = 0
    clocks = ClockSampler(None)
    clocks.start()
    for K, N, name in GEMM_SHAPES:
        w = runtime.Q8Weight(ctx, synth.q8_0_blocks(rng, N, K), K, N)
        for M in GEMM_M:
            a = torch.randn((M, K), dtype=torch.float32, device="cuda")
            codes = torch.empty((M, K), dtype=torch.float16, device="cuda")
            absmax = torch.zeros(4, dtype=torch.int32, device="cuda")
            c = torch.empty((M, N), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            w.run(a.data_ptr(), M, c.data_ptr(), codes.data_ptr(), absmax.data_ptr(), ctx.stream)  # quantises A

            def timed(fn, n):
                ts = []
                for _ in range(n):
                    with torch.cuda.stream(stream):
                        flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    fn()
                    e1.record(stream)
                    e1.synchronize()
                    ts.append(e0.elapsed_time(e1))
                return statistics.median(ts)

            kern = lambda: w.matmul_int8(codes.data_ptr(), absmax.data_ptr(), M, c.data_ptr(), ctx.stream)
            full = lambda: w.run(a.data_ptr(), M, c.data_ptr(), codes.data_ptr(), absmax.data_ptr(), ctx.stream)
            timed(kern, max(args.warmup, 3))
            ms_k = timed(kern, args.steps)
            ms_f = timed(full, args.steps)
            launches += 2 * args.steps * (1 + 3)
            fl, by_k = gemm_algorithmic(K, N, M, True)
            _, by_f = gemm_algorithmic(K, N, M, False)
            tf_k = fl / (ms_k * 1e-3) / 1e12
            gb_k = by_k / (ms_k * 1e-3) / 1e9
            # roofline time of the launch: the slower of bytes over HBM and FLOPs over the tensor peak
            t_roof = max(by_k / (bw_peak * 1e9), fl / (tc_peak * 1e12))
            results[f"{K}x{N} M={M}"] = {
                "kernel_ms": round(ms_k, 4), "kernel_tflops": round(tf_k, 2), "kernel_gbs": round(gb_k, 1),
                "kernel_roofline_frac": round(t_roof / (ms_k * 1e-3), 3),
                "bound": "hbm" if by_k / (bw_peak * 1e9) > fl / (tc_peak * 1e12) else "tensor",
                "with_quantize_ms": round(ms_f, 4), "with_quantize_tflops": round(fl / (ms_f * 1e-3) / 1e12, 2)}
            if M == GEMM_HEAD_M:
                head_flops += fl
                head_ms += ms_k
                # e2e through the public call with host buffers: pinned A in, C out
                a_h = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
                a_h.copy_(a.cpu())
                c_h = torch.empty((M, N), dtype=torch.float32, pin_memory=True)
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                with torch.cuda.stream(stream):
                    a.copy_(a_h, non_blocking=True)
                full()
                with torch.cuda.stream(stream):
                    c_h.copy_(c, non_blocking=True)
                stream.synchronize()
                head_e2e_s += time.perf_counter() - t0
                h2d += M * K * 4
                d2h += M * N * 4
                # pinned buffers used on the library's stream are released while that stream exists
                del a_h, c_h
            del a, codes, c
        w.close()
    clk = clocks.stop()
    t = torch.tensor([head_ms, head_e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    head_ms, head_e2e_s = float(t[0]), float(t[1])
    if rank == 0:
        value = world * head_flops / (head_ms * 1e-3) / 1e12
        dom = max(((k, v) for k, v in results.items() if k.endswith(f"M={GEMM_HEAD_M}")),
                  key=lambda kv: kv[1]["kernel_ms"])
        K, N = (int(x) for x in dom[0].split()[0].split("x"))
        fl, _ = gemm_algorithmic(K, N, GEMM_HEAD_M, True)
        ach = fl / (dom[1]["kernel_ms"] * 1e-3) / 1e12
        line = {"metric": GEMM_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": head_ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8 codes in fp16 MMAs, fp32 accumulate", "data": "synthetic",
                "config": gemm_config(world), "clocks": clk,
                "e2e": {"value": world * head_flops / head_e2e_s / 1e12, "unit": "TFLOP/s",
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "gpu_launches": launches,
                "roofline": {"kernel": f"gemm_q8_tc {dom[0]}", "bound": "tensor", "achieved": ach, "peak": tc_peak,
                             "unit": "TFLOP/s", "frac": ach / tc_peak,
                             "peak_source": "measured bf16_tflops (burst; fp16 MMAs run at the bf16 rate)",
                             "algorithmic_flops_per_launch": fl, "traffic": None},
                "shapes": results}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = gemm_cpu_baseline()
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# --workload search: BASELINE config 5, search/brute exact int8 scan + top-10
# ---------------------------------------------------------------------------
SEARCH_N = 1 << 22
SEARCH_D = 768
SEARCH_Q = 16384
SEARCH_K = 10
SEARCH_SMALL = (1, 8, 32)
SEARCH_METRIC = "search QPS (4M x 768 int8 rows, 16384 int8 queries, top-10 by exact int32 score)"
SEARCH_CHUNK = 1 << 16


def search_config(n_gpus: int) -> dict:
    return {"workload": f"BASELINE config 5: {SEARCH_N} pre-normalised rows of N(0,1) draws, D={SEARCH_D}, int8 "
                        f"(x127), {SEARCH_Q} queries quantised the same way, exact int32 dot products, "
                        f"top-{SEARCH_K} by (score desc, row asc)",
            "parallelism": f"rows sharded across {n_gpus} GPU(s) ({SEARCH_N // n_gpus} rows each), candidate keys "
                           "all-gathered (NCCL) and merged" if n_gpus > 1 else "1 GPU",
            "l2": f"corpus ({SEARCH_N * SEARCH_D / 1e9:.2f} GB) is streamed by every query batch; above L2 (126 MB) "
                  "at the configured size"}


def search_codes(torch, rows: range, dim: int, seed0: int, device: str):
    """Seeded N(0,1) rows, L2-normalised and scaled to int8 (x127) on the device;
    chunk c of SEARCH_CHUNK rows always comes from seed seed0 + c, so every
    shard layout sees the same corpus."""
    out = torch.empty((len(rows), dim), dtype=torch.int8, device=device)
    r = rows.start
    while r < rows.stop:
        c = r // SEARCH_CHUNK
        c0, c1 = c * SEARCH_CHUNK, (c + 1) * SEARCH_CHUNK
        g = torch.Generator(device=device)
        g.manual_seed(seed0 + c)
        v = torch.randn((SEARCH_CHUNK, dim), generator=g, device=device, dtype=torch.float32)
        v = v / v.norm(dim=1, keepdim=True)
        codes = torch.round(v.clamp(-1, 1) * 127).to(torch.int8)
        a, b = max(r, c0), min(rows.stop, c1)
        out[a - rows.start:b - rows.start] = codes[a - c0:b - c0]
        r = b
    return out


def search_cpu_baseline(codes_host: np.ndarray, q_host: np.ndarray, target_s: float = 10.0) -> dict:
    """Exact scan + top-10 on the host cores: batches of one query per thread
    over a corpus sample, repeated until target_s has passed, scaled to the
    full corpus by rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the CPU baseline leg is one of the places allowed to run the oracle
    threads = max(1, min(os.cpu_count() or 1, 128))
    done, qi = 0, 0
    t0 = time.perf_counter()
    while True:
        idx = [(qi + t) % q_host.shape[0] for t in range(threads)]
        oracle.search_exact_batch(1, codes_host, q_host[idx], SEARCH_K, nthreads=threads)
        done += threads
        qi += threads
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    scale = SEARCH_N / codes_host.shape[0]
    return {"value": done / (dt * scale), "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{done} queries x {codes_host.shape[0]} rows in {dt:.1f} s ({threads} threads, one query "
                      f"per thread), scaled to the {SEARCH_N}-row corpus; C restatement of the exact int8 scan and "
                      "top-k (oracle/semantica_oracle.c)"}


def search_host_corpus(rows: int, nq: int):
    """Host copy of the sample used by the reference arm: the same
    normalise-and-quantise recipe, numpy generator."""
    rng = np.random.default_rng(10_000)
    codes = np.empty((rows, SEARCH_D), dtype=np.int8)
    for r in range(0, rows, SEARCH_CHUNK):
        v = rng.standard_normal((min(SEARCH_CHUNK, rows - r), SEARCH_D), dtype=np.float32)
        v /= np.linalg.norm(v, axis=1, keepdims=True)
        codes[r:r + v.shape[0]] = np.round(np.clip(v, -1, 1) * 127).astype(np.int8)
    q = rng.standard_normal((nq, SEARCH_D), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    return codes, np.round(np.clip(q, -1, 1) * 127).astype(np.int8)


def run_search(args) -> None:
    import ctypes as C
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)
    import _lib
    lib = _lib.load()
    ctx = _lib.Context(local)
    stream = torch.cuda.ExternalStream(ctx.stream)
    dev = f"cuda:{local}"
    import sharded
    row_base, row_stop = sharded.shard_rows(SEARCH_N, world, rank)
    per = row_stop - row_base
    codes = search_codes(torch, range(row_base, row_stop), SEARCH_D, 10_000, dev)
    qcodes = search_codes(torch, range(0, SEARCH_Q), SEARCH_D, 90_000, dev)
    torch.cuda.synchronize()
    h = C.c_void_p()
    _lib.check(lib.sem_index_create(ctx.handle, SEARCH_D, 1, C.c_void_p(codes.data_ptr()), None, per, C.byref(h)))
    keys = torch.zeros((SEARCH_Q, SEARCH_K), dtype=torch.int64, device=dev)
    rows = torch.empty((SEARCH_Q, SEARCH_K), dtype=torch.int32, device=dev)
    scores = torch.empty((SEARCH_Q, SEARCH_K), dtype=torch.int32, device=dev)
    st = C.c_void_p(ctx.stream)

    def scan(nq: int, qsrc):
        _lib.check(lib.sem_index_search_keys(h, C.c_void_p(qsrc.data_ptr()), nq, SEARCH_K, 1, row_base,
                                             C.c_void_p(keys.data_ptr()), st))

    def step(nq: int = SEARCH_Q, qsrc=None):
        # sharded.ShardedIndex.search_codes, with the buffers kept across steps
        scan(nq, qcodes if qsrc is None else qsrc)
        with torch.cuda.stream(stream):
            allk = sharded.gather_candidates(keys[:nq]).contiguous()
        _lib.check(lib.sem_topk_merge(ctx.handle, C.c_void_p(allk.data_ptr()), world, nq, SEARCH_K, SEARCH_K, 1, 1,
                                      C.c_void_p(rows.data_ptr()), C.c_void_p(scores.data_ptr()), None, st))

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 0)):
        step()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    # the scan kernel alone (the dominant launch) for the roofline
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        scan(SEARCH_Q, qcodes)
    f1.record(stream)
    torch.cuda.synchronize()
    scan_ms = f0.elapsed_time(f1) / args.steps
    # small-batch regime: one corpus pass per batch of 1 / 8 / 32 queries
    small = {}
    for nq in SEARCH_SMALL:
        step(nq)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        g0.record(stream)
        for _ in range(reps):
            scan(nq, qcodes)
        g1.record(stream)
        torch.cuda.synchronize()
        t = g0.elapsed_time(g1) / reps
        small[f"nq={nq}"] = {"scan_ms": round(t, 4), "qps": round(nq / (t * 1e-3), 1),
                             "corpus_gbs": round(per * SEARCH_D / (t * 1e-3) / 1e9, 1)}
    clk = clocks.stop()
    # e2e: float queries from pinned host memory, quantised on the device, ids back to the host
    qf_host = torch.empty((SEARCH_Q, SEARCH_D), dtype=torch.float32, pin_memory=True)
    qf_host.copy_((qcodes.float() / 127.0).cpu())
    ids_host = torch.empty((SEARCH_Q, SEARCH_K), dtype=torch.int32, pin_memory=True)
    qf_dev = torch.empty((SEARCH_Q, SEARCH_D), dtype=torch.float32, device=dev)
    q_dev = torch.empty_like(qcodes)

    out_ids = np.empty((SEARCH_Q, SEARCH_K), dtype=np.int32)
    out_dist = np.empty((SEARCH_Q, SEARCH_K), dtype=np.float32)
    qf_np = qf_host.numpy()

    def e2e_step():
        if world == 1:
            # Index.SearchVector for the whole batch through the public C ABI:
            # host floats in, ids and distances back in host memory
            _lib.check(lib.sem_index_search(h, C.c_void_p(qf_np.ctypes.data), SEARCH_Q, SEARCH_D, SEARCH_K, 1, 1,
                                            C.c_void_p(out_ids.ctypes.data), C.c_void_p(out_dist.ctypes.data), None))
            return
        with torch.cuda.stream(stream):
            qf_dev.copy_(qf_host, non_blocking=True)
            n = qf_dev / qf_dev.norm(dim=1, keepdim=True)
            q_dev.copy_(torch.round(n.clamp(-1, 1) * 127).to(torch.int8))
        step(SEARCH_Q, q_dev)
        with torch.cuda.stream(stream):
            ids_host.copy_(rows, non_blocking=True)
        stream.synchronize()

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    n_e2e = max(1, min(args.steps, 3))
    for _ in range(n_e2e):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / n_e2e
    barrier()
    tt = torch.tensor([ms, scan_ms, e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms, scan_ms, e2e_s = float(tt[0]), float(tt[1]), float(tt[2])
    if rank == 0:
        peaks = json.load(open(PEAKS_PATH)) if os.path.exists(PEAKS_PATH) else {}
        bf16 = peaks.get("bf16_tflops") or 1590.0
        ops = 2.0 * per * SEARCH_D * SEARCH_Q
        traffic = None
        if os.path.exists(TRAFFIC_PATH):
            bpr = json.load(open(TRAFFIC_PATH)).get("search_tc_bytes_per_corpus_row")
            traffic = bpr * per if bpr else None
        ach = ops / (scan_ms * 1e-3) / 1e12
        line = {"metric": SEARCH_METRIC, "value": SEARCH_Q / (ms * 1e-3), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> int32", "data": "synthetic",
                "config": search_config(world), "clocks": clk,
                "e2e": {"value": SEARCH_Q / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": SEARCH_Q * SEARCH_D * 4,
                        "d2h_bytes_per_step": SEARCH_Q * SEARCH_K * (8 if world == 1 else 4),
                        "api": "sem_index_search (host fp32 queries, normalised and quantised on the device)"
                        if world == 1 else "sem_index_search_keys per shard + NCCL all-gather + sem_topk_merge"},
                "gpu_launches": int(args.steps * 3),
                "roofline": {"kernel": "search_tc_kernel (rows of one GPU x 16384 queries)", "bound": "tensor",
                             "achieved": ach, "peak": 2 * bf16, "unit": "TOP/s", "frac": ach / (2 * bf16),
                             "peak_source": "2 x measured bf16_tflops (dense int8 runs at twice the bf16 rate; no "
                                            "int8 figure is measured on this pool)",
                             "algorithmic_ops_per_launch": ops, "launch_ms": scan_ms, "traffic": traffic,
                             "small_batch_hbm": {"peak_gbs": peaks.get("hbm_gbs") or 6650.0, **small}}}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = search_cpu_baseline(codes[:1 << 20].cpu().numpy(), qcodes[:1024].cpu().numpy())
        print(json.dumps(line), flush=True)
    # tensors used on the library's stream (the NCCL all-gather runs there) go
    # first, then the process group, and only then the stream itself
    torch.cuda.synchronize()
    del qf_np, qf_host, ids_host, qf_dev, q_dev, keys, rows, scores, qcodes  # qf_np views the pinned qf_host
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    lib.sem_index_free(h)
    del codes
    torch.cuda.synchronize()
    ctx.close()


def run_search_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    codes, qc = search_host_corpus(1 << 20, 1024)
    for _ in range(max(args.warmup, 0)):
        search_cpu_baseline(codes, qc, target_s=0.0)
    vals = [search_cpu_baseline(codes, qc, target_s=5.0) for _ in range(max(args.steps, 1))]
    cb = vals[-1]
    value = statistics.median(x["value"] for x in vals)
    cb["value"] = value
    print(json.dumps({"metric": SEARCH_METRIC, "value": value, "unit": "queries/s", "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * SEARCH_Q / value,
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                      "dtype": "int8 x int8 -> int32", "data": "synthetic", "impl": "reference",
                      "config": search_config(args.gpus), "cpu_baseline": cb,
                      "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def main():
    global BATCH, SEQ_LEN, SEARCH_N, SEARCH_Q
    import faulthandler
    faulthandler.enable()  # a crash prints the Python stack
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="embed", choices=["embed", "gemm", "search"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=1024, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--search-rows", type=int, default=SEARCH_N, help="search corpus rows (profiling runs use fewer)")
    ap.add_argument("--search-queries", type=int, default=SEARCH_Q)
    args = ap.parse_args()
    BATCH, SEQ_LEN = args.batch, args.seq_len
    SEARCH_N, SEARCH_Q = args.search_rows, args.search_queries
    if args.workload == "gemm":
        run_gemm_reference(args) if args.impl == "reference" else run_gemm(args)
    elif args.workload == "search":
        run_search_reference(args) if args.impl == "reference" else run_search(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
