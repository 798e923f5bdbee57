"""Benchmark of the B200 embedding forward and search with its CPU baselines.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload embed|gemm|search]

Default workload (the headline): EmbeddingGemma-300M-shaped
Q8_0 forward, 1024 sequences x 512 tokens per GPU (weak scaling: every rank
runs its own 1024 sequences, no collective on the data path), synthetic GGUF
weights and seeded token ids. One JSON line on rank 0. `value` is
device-timed (inputs resident in HBM, CUDA events on the library's stream,
max over ranks); `e2e` goes through the public host API (sem_embed) with
pinned host ids and the host copy of the embeddings inside the timed region.

The same line carries BASELINE's other measurements, each with its own
roofline fraction: `long_context` (config 4: 128 sequences of 256-2048
tokens, split across ranks by tokens), `search` (config 5: the 4M-row scan
at 16384 queries and at 1/8/32-query batches, int8/int16 x D 768/256, rows
split across ranks), `gemm` (config 2 at M = 4096 and 32768), `small_batch`
(config 1 latency through sem_embed) and `parity` (the first sequences of the
timed batch and 64 search queries over the whole corpus against the CPU
oracle).

--impl reference times the CPU restatement of the reference Go path (oracle/;
the reference itself cannot be built here: no Go toolchain) with all host
threads on a bounded sample of the same workload, its inner loops in the
reference's assembly order (AVX512-VNNI / AVX2 intrinsics).
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import shutil
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
H, F, NH, HD, L = 768, 1152, 3, 256, 24

LONG_N, LONG_LO, LONG_HI, LONG_SEED = 128, 256, 2048, 4004

GEMM_SHAPES = [(768, 768, "q/o"), (768, 256, "k/v"), (768, 1152, "gate/up"), (1152, 768, "down"),
               (768, 3072, "dense up"), (3072, 768, "dense down")]
GEMM_M = [1, 64, 512, 4096, 32768]
GEMM_HEAD_M = 32768
GEMM_METRIC = "Q8_0 projection TFLOP/s (kernel on pre-quantised activations, 6 model shapes, M=32768)"

SEARCH_N = 1 << 22
SEARCH_D = 768
SEARCH_Q = 16384
SEARCH_K = 10
SEARCH_SMALL = (1, 8, 32)
SEARCH_CHUNK = 1 << 16
PARITY_SEQS = 4
PARITY_QUERIES = 64


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
              "HBM, about 520 GB of element-wise traffic and 0.4 GB of weight planes per step",
    }


def load_peaks() -> dict:
    return json.load(open(PEAKS_PATH)) if os.path.exists(PEAKS_PATH) else {}


def host_info() -> dict:
    """The host the CPU baseline ran on, and whether the reference's own
    toolchain is there (Go and its module cache)."""
    model = platform.processor() or ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    go = shutil.which("go")
    info = {"cpu_model": model, "host_threads": os.cpu_count()}
    if go:
        try:
            info["go_version"] = subprocess.run([go, "version"], capture_output=True, text=True, timeout=20).stdout.strip()
            info["go_modcache"] = subprocess.run([go, "env", "GOMODCACHE"], capture_output=True, text=True,
                                                 timeout=20).stdout.strip()
        except Exception as e:  # noqa: BLE001
            info["go_version"] = f"go present, probe failed: {e}"
    else:
        info["go_version"] = "go not found on PATH (probed)"
    return info


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
# CPU baseline: the oracle (C restatement of the reference Go path) with its
# inner loops in the reference's assembly order
# ---------------------------------------------------------------------------
def _oracle_timed():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # the CPU baseline legs are among the places allowed to run the oracle
    simd = oracle.set_simd(True)
    return oracle, simd


def _port_note(simd: bool) -> str:
    return ("C restatement of the reference Go INT8 forward (oracle/semantica_oracle.c), Q8_0 inner loop and float32 "
            "dot products as AVX512-VNNI / AVX2 intrinsics in the reference's assembly order" if simd else
            "C restatement of the reference Go INT8 forward (oracle/semantica_oracle.c), plain C loops (no "
            "AVX512-VNNI on this host)")


def cpu_baseline(model_path: str) -> dict:
    oracle, simd = _oracle_timed()
    threads = max(1, min(os.cpu_count() or 1, 32))
    n_seq = threads
    m = oracle.OracleModel(model_path)
    ids, offs = synth.token_batch(4242, [SEQ_LEN] * n_seq, m.config.vocab_size)
    t0 = time.perf_counter()
    m.forward_batch(ids, offs, 768, nthreads=threads)
    dt = time.perf_counter() - t0
    m.close()
    oracle.set_simd(False)
    return {"value": n_seq / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_seq} sequences x {SEQ_LEN} tokens, one per thread ({dt:.1f} s, "
                      f"{dt * threads / n_seq:.2f} CPU-s per embedding); {_port_note(simd)}",
            **host_info()}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = synth.cached_gguf(MODEL_DIR, seed=1234)
    oracle, simd = _oracle_timed()
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
                             "sample": f"{threads} sequences x {SEQ_LEN} tokens per step, one per thread "
                                       f"({per:.2f} s per step, {per:.2f} CPU-s per embedding); {_port_note(simd)}",
                             **host_info()},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# roofline helpers
# ---------------------------------------------------------------------------
def attention_flops(seq_lens) -> float:
    """Scores + P.V of the reference (attention.go:267-310) over sequences."""
    return float(sum(4.0 * int(s) * int(s) * HD * NH for s in seq_lens))


def stage_roofline(stage: str, total_ms: float, launches: int, T: int, seq_lens, peaks: dict) -> dict:
    per_ms = total_ms / max(launches, 1)
    gemm = {"gemm_q8_qkv": (H, NH * HD + 2 * HD), "gemm_q8_o": (H, H), "gemm_q8_gate_up": (H, 2 * F),
            "gemm_q8_down": (F, H)}
    peak = peaks.get("bf16_tflops_sustained") or 1415.9
    if stage in gemm:
        K, N = gemm[stage]
        flops = 2.0 * T * N * K
        achieved = flops / (per_ms * 1e-3) / 1e12
        return {"kernel": stage, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained (the projections run "
                "kind::f16 MMAs, the bf16 rate; algorithmic FLOPs: the hi and lo planes execute twice that)",
                "algorithmic_flops_per_launch": flops, "launch_ms": per_ms}
    if stage in ("attention", "attention_short"):
        flops = attention_flops(seq_lens)
        achieved = flops / (per_ms * 1e-3) / 1e12
        return {"kernel": stage, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained",
                "algorithmic_flops_per_launch": flops, "launch_ms": per_ms}
    # per-launch averages over a forward: quantize runs once on the first
    # attention norm and per layer on the attention output (K = H) and on the
    # MLP product (K = F), fp32 in and fp16 codes out; the residual kernel
    # reads o and hidden, writes hidden, and in all but the last of its 2 L
    # launches also writes the next norm's fp16 codes; the Q/K norm kernel
    # reads the float32 q and k heads and writes their fp16 hi / lo planes
    # (the QKV projection writes V's planes itself on the bench's workload)
    bytes_per_row = {"quantize": 6.0 * ((L + 1) * H + L * F) / (2 * L + 1),
                     "residual_norm": 3 * 4 * H + 2.0 * H * (2 * L - 1) / (2 * L), "row_stats": 4 * H,
                     "qk_norm_rope": 4 * (NH * HD + HD) + 2 * 2 * (NH * HD + HD), "embed": 4 * H + H,
                     "pool_l2": 4 * H}.get(stage, 4 * H)
    b = bytes_per_row * T
    achieved = b / (per_ms * 1e-3) / 1e9
    bw = peaks.get("hbm_gbs") or 6650.0
    return {"kernel": stage, "bound": "hbm", "achieved": achieved, "peak": bw, "unit": "GB/s", "frac": achieved / bw,
            "algorithmic_bytes_per_launch": b, "launch_ms": per_ms}


def dominant_roofline(stages: dict, steps: int, T: int, seq_lens, peaks: dict, traffic_key_scale=None) -> dict:
    dom = max(stages.items(), key=lambda kv: kv[1][0])
    roof = stage_roofline(dom[0], dom[1][0], dom[1][1], T, seq_lens, peaks)
    traffic = None
    if os.path.exists(TRAFFIC_PATH):
        tr = json.load(open(TRAFFIC_PATH))
        traffic = tr.get(dom[0])
        if traffic is not None and traffic_key_scale is not None:
            traffic = traffic * traffic_key_scale
    roof["traffic"] = traffic
    roof["stages_ms_per_step"] = {k: round(v[0] / steps, 3) for k, v in stages.items() if v[1]}
    return roof


def events_time(torch, stream, fn, n: int) -> float:
    """Mean ms of fn() over n calls, CUDA events on `stream`."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / max(n, 1)


class Env:
    """One rank's GPU context and process group for the legs of a run."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.args = torch, dist, args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        torch.cuda.set_device(self.local)
        import _lib
        self._lib = _lib
        self.lib = _lib.load()
        self.ctx = _lib.Context(self.local)
        self.stream = torch.cuda.ExternalStream(self.ctx.stream)
        self.dev = f"cuda:{self.local}"
        self.peaks = load_peaks()

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, *vals) -> list:
        t = self.torch.tensor(list(vals), dtype=self.torch.float64, device=self.dev)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return [float(x) for x in t]

    def uuid(self):
        try:
            return "GPU-" + str(self.torch.cuda.get_device_properties(self.local).uuid)
        except Exception:  # noqa: BLE001
            return None

    def close(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()
        self.ctx.close()


# ---------------------------------------------------------------------------
# long context, 128 sequences of 256-2048 tokens
# ---------------------------------------------------------------------------
def leg_long_context(env: Env, model, steps: int, warmup: int) -> dict:
    """The 128 sequences are split across ranks by token count
    (sharded.split_sequences, deterministic on every rank); each rank embeds
    its share, so the job time is the slowest rank's (strong scaling)."""
    import sharded
    torch = env.torch
    lengths = [int(x) for x in synth.ragged_lengths(LONG_SEED, LONG_N, LONG_LO, LONG_HI)]
    ids_all, offs_all = synth.token_batch(LONG_SEED + 1, lengths, model.config().vocab_size)
    mine = sharded.split_sequences(lengths, env.world)[env.rank]
    my_lens = [lengths[i] for i in mine]
    ids = np.concatenate([ids_all[offs_all[i]:offs_all[i + 1]] for i in mine]) if mine else np.zeros(0, np.int32)
    offs = np.zeros(len(mine) + 1, dtype=np.int32)
    offs[1:] = np.cumsum(my_lens)
    T = int(offs[-1])
    d_ids = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).to(env.dev)
    d_out = torch.empty((max(len(mine), 1), 768), dtype=torch.float32, device=env.dev)
    torch.cuda.synchronize()

    def step():
        if mine:
            model.embed_device(d_ids.data_ptr(), offs, len(mine), 768, d_out.data_ptr(), env.ctx.stream)

    for _ in range(max(warmup, 1)):
        step()
    torch.cuda.synchronize()
    env.barrier()
    ms = events_time(torch, env.stream, step, steps)
    model.check()  # device-detected errors of the timed forwards (timed-out waits, bad ids)
    env.barrier()
    model.profile(True)
    for _ in range(steps):
        step()
    stages = model.profile_read()
    model.profile(False)
    ms, = env.max_over_ranks(ms)
    total_tokens = int(sum(lengths))
    out = {"config": f"BASELINE config 4: {LONG_N} sequences, lengths uniform in [{LONG_LO}, {LONG_HI}] (seed "
                     f"{LONG_SEED}: {total_tokens} tokens), 768-dim, split across {env.world} GPU(s) by tokens; "
                     "full bidirectional attention in every layer, as the reference runs it",
           "embeddings_per_s": LONG_N / (ms * 1e-3), "tokens_per_s": total_tokens / (ms * 1e-3),
           "ms_per_step": ms, "scaling": "strong", "tokens_this_rank": T,
           "attention_share_of_flops": attention_flops(lengths) / (attention_flops(lengths) + 2.0 * total_tokens * (
               H * (NH * HD + 2 * HD) + H * H + H * 2 * F + F * H))}  # per layer, both terms
    if mine and any(v[1] for v in stages.values()):
        out["roofline"] = dominant_roofline(stages, steps, T, my_lens, env.peaks)
    # the same batch in the model-faithful mode (EmbeddingGemma's sliding
    # layers: window 512, every 6th layer global; the reference runs full
    # attention everywhere, so this variant is reported apart from the parity
    # workload above)
    model.set_faithful(512, 6)
    step()
    torch.cuda.synchronize()
    env.barrier()
    ms_swa = events_time(torch, env.stream, step, steps)
    model.check()
    model.set_faithful()
    ms_swa, = env.max_over_ranks(ms_swa)
    out["sliding_window_variant"] = {
        "config": "model-faithful mode: sliding-window layers (window 512, every 6th layer global), same batch",
        "embeddings_per_s": LONG_N / (ms_swa * 1e-3), "tokens_per_s": total_tokens / (ms_swa * 1e-3),
        "ms_per_step": ms_swa}
    return out


# ---------------------------------------------------------------------------
# the isolated Q8_0 projection
# ---------------------------------------------------------------------------
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


def gemm_measure(env: Env, Ms, reps: int, warmup: int, e2e_m: int | None = None) -> tuple[dict, dict]:
    """Per (shape, M): kernel-only and with-quantiser times (median of reps,
    L2 flushed before each), TFLOP/s, GB/s and roofline fraction. Returns
    (results, totals at the largest M incl. an e2e time through host buffers)."""
    import runtime
    torch = env.torch
    flush = torch.empty(64 << 20, dtype=torch.float32, device=env.dev)  # 256 MB > L2
    tc_peak = env.peaks.get("bf16_tflops") or 1590.0
    bw_peak = env.peaks.get("hbm_gbs") or 6650.0
    rng = np.random.default_rng(2 + env.rank)
    results, tot = {}, {"flops": 0.0, "ms": 0.0, "e2e_s": 0.0, "h2d": 0, "d2h": 0, "launches": 0}
    top = max(Ms)
    for K, N, name in GEMM_SHAPES:
        w = runtime.Q8Weight(env.ctx, synth.q8_0_blocks(rng, N, K), K, N)
        for M in Ms:
            a = torch.randn((M, K), dtype=torch.float32, device=env.dev)
            codes = torch.empty((M, K), dtype=torch.float16, device=env.dev)
            absmax = torch.zeros(4, dtype=torch.int32, device=env.dev)
            c = torch.empty((M, N), dtype=torch.float32, device=env.dev)
            torch.cuda.synchronize()
            w.run(a.data_ptr(), M, c.data_ptr(), codes.data_ptr(), absmax.data_ptr(), env.ctx.stream)  # quantises A

            def timed(fn, n):
                ts = []
                for _ in range(n):
                    with torch.cuda.stream(env.stream):
                        flush.zero_()
                    ts.append(events_time(torch, env.stream, fn, 1))
                return statistics.median(ts)

            kern = lambda: w.matmul_int8(codes.data_ptr(), absmax.data_ptr(), M, c.data_ptr(), env.ctx.stream)  # noqa: E731
            full = lambda: w.run(a.data_ptr(), M, c.data_ptr(), codes.data_ptr(), absmax.data_ptr(), env.ctx.stream)  # noqa: E731
            timed(kern, max(warmup, 3))
            ms_k = timed(kern, reps)
            ms_f = timed(full, reps)
            tot["launches"] += reps * (1 + 4)
            fl, by_k = gemm_algorithmic(K, N, M, True)
            t_roof = max(by_k / (bw_peak * 1e9), fl / (tc_peak * 1e12))
            results[f"{K}x{N} M={M}"] = {
                "kernel_ms": round(ms_k, 4), "kernel_tflops": round(fl / (ms_k * 1e-3) / 1e12, 2),
                "kernel_gbs": round(by_k / (ms_k * 1e-3) / 1e9, 1),
                "kernel_roofline_frac": round(t_roof / (ms_k * 1e-3), 3),
                "bound": "hbm" if by_k / (bw_peak * 1e9) > fl / (tc_peak * 1e12) else "tensor",
                "with_quantize_ms": round(ms_f, 4), "with_quantize_tflops": round(fl / (ms_f * 1e-3) / 1e12, 2)}
            if M == top:
                tot["flops"] += fl
                tot["ms"] += ms_k
                if e2e_m:
                    # through the public call with host buffers: pinned A in, C out
                    a_h = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
                    a_h.copy_(a.cpu())
                    c_h = torch.empty((M, N), dtype=torch.float32, pin_memory=True)
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    with torch.cuda.stream(env.stream):
                        a.copy_(a_h, non_blocking=True)
                    full()
                    with torch.cuda.stream(env.stream):
                        c_h.copy_(c, non_blocking=True)
                    env.stream.synchronize()
                    tot["e2e_s"] += time.perf_counter() - t0
                    tot["h2d"] += M * K * 4
                    tot["d2h"] += M * N * 4
                    del a_h, c_h  # pinned buffers used on the library's stream go while that stream exists
            del a, codes, c
        w.close()
    return results, tot


def leg_gemm(env: Env, steps: int, warmup: int) -> dict:
    results, tot = gemm_measure(env, [4096, 32768], max(3, min(steps, 10)), warmup)
    ms, = env.max_over_ranks(tot["ms"])
    tc_peak = env.peaks.get("bf16_tflops") or 1590.0
    tf = tot["flops"] / (ms * 1e-3) / 1e12
    worst = min(((k, v) for k, v in results.items() if k.endswith("M=4096")), key=lambda kv: kv[1]["kernel_roofline_frac"])
    return {"config": "BASELINE config 2 at M = 4096 and 32768 (kernel on pre-quantised codes, L2 flushed before "
                      "each launch; with_quantize adds QuantizeSymmetricINT8Into)",
            "tflops_m32768": tf * env.world, "unit": "TFLOP/s", "parallelism": f"replicas x{env.world}",
            "roofline": {"kernel": "Q8_0 projection, 6 shapes at M=32768", "bound": "tensor", "achieved": tf,
                         "peak": tc_peak, "unit": "TFLOP/s", "frac": tf / tc_peak,
                         "peak_source": "measured bf16_tflops (burst; fp16 MMAs run at the bf16 rate; algorithmic "
                                        "FLOPs, the split planes execute twice that)"},
            "lowest_frac_at_m4096": {"shape": worst[0], **worst[1]},
            "shapes": results}


# ---------------------------------------------------------------------------
# search/brute quantised scan + top-10
# ---------------------------------------------------------------------------
def search_metric(quant: int = 1, dim: int | None = None) -> str:
    """The search line's metric for the configured corpus and batch (BASELINE
    config 5's at the defaults)."""
    dim = dim or SEARCH_D
    t = "int8" if quant == 1 else "int16"
    rows = f"{SEARCH_N >> 20}M" if SEARCH_N % (1 << 20) == 0 else str(SEARCH_N)
    return f"search QPS ({rows} x {dim} {t} rows, {SEARCH_Q} {t} queries, top-{SEARCH_K} by exact int32 score)"


def search_config(n_gpus: int, quant: int = 1, dim: int | None = None) -> dict:
    dim = dim or SEARCH_D
    el, scale = (1, "int8 (x127)") if quant == 1 else (2, "int16 (x32767)")
    return {"workload": f"BASELINE config 5: {SEARCH_N} pre-normalised rows of N(0,1) draws, D={dim}, {scale}, "
                        f"{SEARCH_Q} queries quantised the same way, exact int32 dot products, "
                        f"top-{SEARCH_K} by (score desc, row asc)",
            "parallelism": f"rows sharded across {n_gpus} GPU(s) ({SEARCH_N // n_gpus} rows each), candidate keys "
                           "all-gathered (NCCL) and merged" if n_gpus > 1 else "1 GPU",
            "l2": f"corpus ({SEARCH_N * dim * el / 1e9:.2f} GB) is streamed by every query batch; above L2 (126 MB) "
                  "at the configured size"}


def search_codes(torch, rows: range, dim: int, seed0: int, device: str, quant: int = 1):
    """Seeded N(0,1) rows, L2-normalised and scaled to int8 (x127, quant 1) or
    int16 (x32767, quant 2) on the device; chunk c of SEARCH_CHUNK rows always
    comes from seed seed0 + c, so every shard layout sees the same corpus, and
    the int8 and int16 corpora of one dimension quantise the same vectors."""
    dtype, scale = (torch.int8, 127.0) if quant == 1 else (torch.int16, 32767.0)
    out = torch.empty((len(rows), dim), dtype=dtype, device=device)
    r = rows.start
    while r < rows.stop:
        c = r // SEARCH_CHUNK
        c0, c1 = c * SEARCH_CHUNK, (c + 1) * SEARCH_CHUNK
        g = torch.Generator(device=device)
        g.manual_seed(seed0 + c)
        v = torch.randn((SEARCH_CHUNK, dim), generator=g, device=device, dtype=torch.float32)
        v = v / v.norm(dim=1, keepdim=True)
        codes = torch.round(v.clamp(-1, 1) * scale).to(dtype)
        a, b = max(r, c0), min(rows.stop, c1)
        out[a - rows.start:b - rows.start] = codes[a - c0:b - c0]
        r = b
    return out


class SearchVariant:
    """This rank's row shard of one corpus (quant, dim), its index and query codes."""

    def __init__(self, env: Env, quant: int, dim: int, nq_max: int):
        import ctypes as C
        import sharded
        self.env, self.quant, self.dim, self.C = env, quant, dim, C
        torch = env.torch
        self.row_base, row_stop = sharded.shard_rows(SEARCH_N, env.world, env.rank)
        self.per = row_stop - self.row_base
        self.codes = search_codes(torch, range(self.row_base, row_stop), dim, 10_000 + dim, env.dev, quant)
        self.qcodes = search_codes(torch, range(0, nq_max), dim, 90_000 + dim, env.dev, quant)
        torch.cuda.synchronize()
        h = C.c_void_p()
        env._lib.check(env.lib.sem_index_create(env.ctx.handle, dim, quant, C.c_void_p(self.codes.data_ptr()), None,
                                                self.per, C.byref(h)))
        self.h = h
        self.keys = torch.zeros((nq_max, SEARCH_K), dtype=torch.int64, device=env.dev)
        self.rows = torch.empty((nq_max, SEARCH_K), dtype=torch.int32, device=env.dev)
        self.scores = torch.empty((nq_max, SEARCH_K), dtype=torch.int32, device=env.dev)
        self.st = C.c_void_p(env.ctx.stream)

    def scan(self, nq: int, qsrc=None):
        q = self.qcodes if qsrc is None else qsrc
        self.env._lib.check(self.env.lib.sem_index_search_keys(self.h, self.C.c_void_p(q.data_ptr()), nq, SEARCH_K, 1,
                                                               self.row_base, self.C.c_void_p(self.keys.data_ptr()),
                                                               self.st))

    def step(self, nq: int, qsrc=None):
        """sharded.ShardedIndex.search_codes with the buffers kept across steps:
        shard scan, all-gather of the candidate keys, merge."""
        import sharded
        self.scan(nq, qsrc)
        with self.env.torch.cuda.stream(self.env.stream):
            allk = sharded.gather_candidates(self.keys[:nq]).contiguous()
        C = self.C
        self.env._lib.check(self.env.lib.sem_topk_merge(self.env.ctx.handle, C.c_void_p(allk.data_ptr()),
                                                        self.env.world, nq, SEARCH_K, SEARCH_K, 1, self.quant,
                                                        C.c_void_p(self.rows.data_ptr()),
                                                        C.c_void_p(self.scores.data_ptr()), None, self.st))

    def small_batches(self, reps: int = 20) -> dict:
        torch, env = self.env.torch, self.env
        bw = env.peaks.get("hbm_gbs") or 6650.0
        out = {}
        for nq in SEARCH_SMALL:
            self.step(nq)
            torch.cuda.synchronize()
            t = events_time(torch, env.stream, lambda: self.scan(nq), reps)
            gbs = self.per * self.dim * self.quant / (t * 1e-3) / 1e9
            out[f"nq={nq}"] = {"scan_ms": round(t, 4), "qps": round(nq / (t * 1e-3), 1), "corpus_gbs": round(gbs, 1),
                               "hbm_frac": round(gbs / bw, 3)}
        return out

    def close(self):
        self.env.torch.cuda.synchronize()
        self.env.lib.sem_index_free(self.h)
        self.h = None
        del self.codes, self.qcodes, self.keys, self.rows, self.scores


def search_parity(env: Env, var: SearchVariant) -> dict | None:
    """64 queries through the sharded search path (every rank) against the
    oracle's exact scan over the whole corpus (rank 0): ids and int32 scores
    bit-exact, ties to the lower row."""
    torch = env.torch
    # with several ranks the other processes hold host cores while rank 0
    # scans on the CPU: a quarter of the queries keeps the check short
    nq = PARITY_QUERIES if env.world == 1 else PARITY_QUERIES // 4
    var.step(nq)
    torch.cuda.synchronize()
    if env.rank != 0:
        return None
    got_rows = var.rows[:nq].cpu().numpy()
    got_scores = var.scores[:nq].cpu().numpy()
    q_host = var.qcodes[:nq].cpu().numpy()
    if env.world == 1:
        corpus = var.codes.cpu().numpy()
    else:  # the whole corpus, regenerated from the same seeds on this GPU
        full = search_codes(torch, range(0, SEARCH_N), var.dim, 10_000 + var.dim, env.dev, var.quant)
        corpus = full.cpu().numpy()
        del full
    oracle, _ = _oracle_timed()
    oracle.set_simd(False)
    t0 = time.perf_counter()
    rrows, rscores, _ = oracle.search_exact_batch(var.quant, corpus, q_host, SEARCH_K)
    dt = time.perf_counter() - t0
    del corpus
    return {"queries": nq, "rows": SEARCH_N, "dim": var.dim, "k": SEARCH_K,
            "ids_exact": bool(np.array_equal(got_rows, rrows)), "scores_exact": bool(np.array_equal(got_scores, rscores)),
            "mismatched_queries": int((got_rows != rrows).any(axis=1).sum()), "oracle_s": round(dt, 2)}


def leg_search(env: Env, steps: int, warmup: int, parity: bool) -> tuple[dict, dict | None]:
    torch = env.torch
    bf16 = env.peaks.get("bf16_tflops") or 1590.0
    out, par = {"config": search_config(env.world)}, None
    # (quant, dim, time the 16384-query batch): int8 rows on kind::i8 tensor
    # cores, int16 rows as byte planes on four kind::i8 products
    for quant, dim, full in ((1, 768, True), (1, 256, True), (2, 768, True), (2, 256, True)):
        name = f"{'int8' if quant == 1 else 'int16'}_d{dim}"
        var = SearchVariant(env, quant, dim, SEARCH_Q if full else max(max(SEARCH_SMALL), PARITY_QUERIES))
        res = {"rows_per_gpu": var.per}
        if full:
            for _ in range(max(warmup, 1)):
                var.step(SEARCH_Q)
            torch.cuda.synchronize()
            env.barrier()
            ms = events_time(torch, env.stream, lambda: var.step(SEARCH_Q), steps)
            env.barrier()
            scan_ms = events_time(torch, env.stream, lambda: var.scan(SEARCH_Q), steps)
            ms, scan_ms = env.max_over_ranks(ms, scan_ms)
            ops = 2.0 * var.per * dim * SEARCH_Q
            ach = ops / (scan_ms * 1e-3) / 1e12
            res.update({"queries": SEARCH_Q, "qps": SEARCH_Q / (ms * 1e-3), "ms_per_batch": ms, "scan_ms": scan_ms,
                        "scaling": "strong",
                        "roofline": {"kernel": ("search_tc_kernel" if quant == 1 else "search_tc16_kernel")
                                     + f" (rows of one GPU x {SEARCH_Q} queries)", "bound": "tensor",
                                     "achieved": ach, "peak": 2 * bf16, "unit": "TOP/s", "frac": ach / (2 * bf16),
                                     "peak_source": "2 x measured bf16_tflops (dense int8 runs at twice the bf16 rate; "
                                                    "no int8 figure is measured on this pool)"
                                     + ("" if quant == 1 else "; algorithmic int16 ops, the byte planes execute 4x "
                                                             "as many int8 MACs"),
                                     "algorithmic_ops_per_launch": ops, "launch_ms": scan_ms}})
        res["small_batch"] = var.small_batches()
        if parity and quant == 1 and dim == 768:
            par = search_parity(env, var)
        out[name] = res
        var.close()
        torch.cuda.empty_cache()
        env.barrier()
    return out, par


def embed_parity(model_path: str, ids_h, offs, got: np.ndarray) -> dict:
    """The first PARITY_SEQS sequences of the timed batch against the oracle
    (the reference's default build): north_star's per-embedding bound."""
    oracle, _ = _oracle_timed()
    m = oracle.OracleModel(model_path)
    n = PARITY_SEQS
    t0 = time.perf_counter()
    ref = m.forward_batch(ids_h[:offs[n]], offs[:n + 1], 768, nthreads=n)
    dt = time.perf_counter() - t0
    m.close()
    oracle.set_simd(False)
    cos = [float(np.dot(got[i].astype(np.float64), ref[i]) / np.linalg.norm(got[i].astype(np.float64)) /
                 np.linalg.norm(ref[i].astype(np.float64))) for i in range(n)]
    mabs = [float(np.abs(got[i] - ref[i]).max()) for i in range(n)]
    return {"sequences": n, "tokens_each": int(offs[1] - offs[0]), "cosine_min": min(cos), "max_abs": max(mabs),
            "bound": "cosine >= 0.9995 and max-abs <= 2e-3 per embedding",
            "pass": bool(min(cos) >= 0.9995 and max(mabs) <= 2e-3), "oracle_s": round(dt, 2)}


# ---------------------------------------------------------------------------
# our arm: the headline and every leg
# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import ctypes as C
    env = Env(args)
    torch, world, rank, local = env.torch, env.world, env.rank, env.local
    import runtime
    lib = env.lib

    if world > 1 and local != 0:
        env.barrier()
    path = synth.cached_gguf(MODEL_DIR, seed=1234)
    if world > 1 and local == 0:
        env.barrier()

    ctx = env.ctx
    model = runtime.load_model(path, ctx)
    stream = env.stream
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

    clocks = ClockSampler(env.uuid())
    clocks.start()
    time.sleep(0.3)

    # ---- device-timed value ----
    env.barrier()
    torch.cuda.synchronize()
    ms = events_time(torch, stream, step, args.steps)
    env.barrier()
    model.check()  # errors the device recorded during the timed forwards

    # ---- per-kernel timing inside the same kind of steps ----
    model.profile(True)
    for _ in range(args.steps):
        step()
    stages = model.profile_read()
    model.profile(False)
    clk = clocks.stop()
    got_parity = d_out[:PARITY_SEQS].cpu().numpy() if rank == 0 else None

    # ---- e2e through the host API (pinned ids in, embeddings out) ----
    pinned = torch.empty(T, dtype=torch.int32, pin_memory=True)
    pinned.numpy()[:] = ids_h
    host_ids = pinned.numpy()
    out_pinned = torch.empty(BATCH * 768, dtype=torch.float32, pin_memory=True).numpy()
    dims = np.full(BATCH, 768, dtype=np.int32)
    offs32 = np.ascontiguousarray(offs, dtype=np.int32)

    def e2e_step():
        env._lib.check(lib.sem_embed(model.handle, host_ids.ctypes.data, offs32.ctypes.data, BATCH, dims.ctypes.data,
                                     out_pinned.ctypes.data))

    e2e_step()
    env.barrier()
    t0 = time.perf_counter()
    n_e2e = max(1, min(args.steps, 3))
    for _ in range(n_e2e):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / n_e2e
    env.barrier()

    # ---- small batch latency (8 x 64 tokens, 768-dim) ----
    # through sem_embed, which replays a CUDA graph of the forward once the
    # shape repeats; sequences under 128 tokens run the exact kernels
    small = None
    if world == 1:
        s_ids, s_offs = synth.token_batch(77, [64] * 8, model.config().vocab_size)
        s_ids = np.ascontiguousarray(s_ids, dtype=np.int32)
        s_offs = np.ascontiguousarray(s_offs, dtype=np.int32)
        s_dims = np.full(8, 768, dtype=np.int32)
        s_out = np.empty(8 * 768, dtype=np.float32)

        def small_call():
            env._lib.check(lib.sem_embed(model.handle, s_ids.ctypes.data, s_offs.ctypes.data, 8, s_dims.ctypes.data,
                                         s_out.ctypes.data))

        for _ in range(5):
            small_call()
        n_small = 50
        t0 = time.perf_counter()
        for _ in range(n_small):
            small_call()
        small_ms = (time.perf_counter() - t0) / n_small * 1e3
        # the same requests back to back through the request pipeline
        # (sem_embed_submit / sem_embed_wait, two in flight): the host side of
        # request i + 1 overlaps the device work of request i
        t_id = C.c_uint64()
        for _ in range(3):  # warm-up: the slots' pinned buffers and events are made on first use
            env._lib.check(lib.sem_embed_submit(model.handle, s_ids.ctypes.data, s_offs.ctypes.data, 8,
                                                s_dims.ctypes.data, C.byref(t_id)))
            env._lib.check(lib.sem_embed_wait(model.handle, C.c_uint64(t_id.value), s_out.ctypes.data))
        tickets = []
        t0 = time.perf_counter()
        for _ in range(n_small):
            env._lib.check(lib.sem_embed_submit(model.handle, s_ids.ctypes.data, s_offs.ctypes.data, 8,
                                                s_dims.ctypes.data, C.byref(t_id)))
            tickets.append(t_id.value)
            if len(tickets) == 2:
                env._lib.check(lib.sem_embed_wait(model.handle, C.c_uint64(tickets.pop(0)), s_out.ctypes.data))
        for t in tickets:
            env._lib.check(lib.sem_embed_wait(model.handle, C.c_uint64(t), s_out.ctypes.data))
        pipe_ms = (time.perf_counter() - t0) / n_small * 1e3
        # the per-block tensor-core projections and attention (not bit-exact)
        prev_path = lib.sem_q8_path(1)
        for _ in range(5):
            small_call()
        t0 = time.perf_counter()
        for _ in range(n_small):
            small_call()
        tc_ms = (time.perf_counter() - t0) / n_small * 1e3
        lib.sem_q8_path(prev_path)
        small = {"config": "BASELINE config 1: 8 sequences x 64 tokens, 768-dim, host ids in and embeddings out "
                           "through sem_embed (wall clock per call, CUDA graph replay; sequences under 128 tokens "
                           "take the kernels that are bit-identical to the reference)",
                 "ms_per_call": small_ms, "embeddings_per_s": 8 / (small_ms * 1e-3),
                 "pipelined_ms_per_request": pipe_ms,
                 "tensor_core_path_ms_per_call": tc_ms,
                 "tensor_core_path": "SEM_Q8_PATH_BLOCK: per-block tcgen05 projections and the tensor-core "
                                     "attention, within north_star's bound but not bit-identical"}

    ms, e2e_s = env.max_over_ranks(ms, e2e_s)
    legs = set(args.legs.split(",")) if args.legs not in ("", "none") else set()
    extra = {}
    if "long" in legs:
        extra["long_context"] = leg_long_context(env, model, args.steps, args.warmup)
    if "gemm" in legs:
        extra["gemm"] = leg_gemm(env, args.steps, args.warmup)
    search_par = None
    if "search" in legs:
        extra["search"], search_par = leg_search(env, args.steps, args.warmup, "parity" in legs)

    if rank == 0:
        roof = dominant_roofline(stages, args.steps, T, lengths, env.peaks)
        launches_per_step = sum(v[1] for v in stages.values()) // max(args.steps, 1)
        line = {
            "metric": METRIC, "value": BATCH * world / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": workload_config(world), "clocks": clk,
            "e2e": {"value": BATCH * world / e2e_s, "unit": UNIT, "h2d_bytes_per_step": int(T * 4),
                    "d2h_bytes_per_step": int(BATCH * 768 * 4),
                    "api": "sem_embed (host token ids in, embeddings out; the batch shape repeats, so only the ids "
                           "are uploaded)"},
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": roof,
        }
        if small:
            line["small_batch"] = small
        line.update(extra)
        if "parity" in legs:
            line["parity"] = {"embeddings": embed_parity(path, ids_h, offs, got_parity)}
            if search_par:
                line["parity"]["search"] = search_par
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(path)
        print(json.dumps(line), flush=True)
    model.close()
    env.close()


# ---------------------------------------------------------------------------
# --workload gemm: BASELINE config 2 on its own
# ---------------------------------------------------------------------------
def gemm_cpu_baseline(rows_per_thread: int = 1536) -> dict:
    """The oracle's MatMulQ8_0INT8 restatement on every host thread: each thread
    takes its own slice of rows of each config-2 shape (ctypes releases the GIL)."""
    import concurrent.futures as cf
    oracle, simd = _oracle_timed()
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
    oracle.set_simd(False)
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows_per_thread} rows per thread x {threads} threads on each of the 6 shapes ({dt:.1f} s); "
                      "C restatement of MatMulQ8_0INT8 (oracle/semantica_oracle.c)"
                      + (", the VNNI inner loop as AVX512-VNNI intrinsics" if simd else ""), **host_info()}


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
    env = Env(args)
    clocks = ClockSampler(None)
    clocks.start()
    results, tot = gemm_measure(env, GEMM_M, args.steps, args.warmup, e2e_m=GEMM_HEAD_M)
    clk = clocks.stop()
    head_ms, head_e2e_s = env.max_over_ranks(tot["ms"], tot["e2e_s"])
    if env.rank == 0:
        tc_peak = env.peaks.get("bf16_tflops") or 1590.0
        value = env.world * tot["flops"] / (head_ms * 1e-3) / 1e12
        dom = max(((k, v) for k, v in results.items() if k.endswith(f"M={GEMM_HEAD_M}")),
                  key=lambda kv: kv[1]["kernel_ms"])
        K, N = (int(x) for x in dom[0].split()[0].split("x"))
        fl, _ = gemm_algorithmic(K, N, GEMM_HEAD_M, True)
        ach = fl / (dom[1]["kernel_ms"] * 1e-3) / 1e12
        line = {"metric": GEMM_METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": env.world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": head_ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8 codes in fp16 MMAs, fp32 accumulate", "data": "synthetic",
                "config": gemm_config(env.world), "clocks": clk,
                "e2e": {"value": env.world * tot["flops"] / head_e2e_s / 1e12, "unit": "TFLOP/s",
                        "h2d_bytes_per_step": tot["h2d"], "d2h_bytes_per_step": tot["d2h"]},
                "gpu_launches": tot["launches"],
                "roofline": {"kernel": f"gemm_q8 {dom[0]}", "bound": "tensor", "achieved": ach, "peak": tc_peak,
                             "unit": "TFLOP/s", "frac": ach / tc_peak,
                             "peak_source": "measured bf16_tflops (burst; fp16 MMAs run at the bf16 rate)",
                             "algorithmic_flops_per_launch": fl, "traffic": None},
                "shapes": results}
        if env.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = gemm_cpu_baseline()
        print(json.dumps(line), flush=True)
    env.close()


# ---------------------------------------------------------------------------
# --workload search: BASELINE config 5 on its own
# ---------------------------------------------------------------------------
def search_cpu_baseline(codes_host: np.ndarray, q_host: np.ndarray, target_s: float = 10.0) -> dict:
    """Exact scan + top-10 on the host cores: batches of one query per thread
    over a corpus sample, repeated until target_s has passed, scaled to the
    full corpus by rows."""
    oracle, _ = _oracle_timed()
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
                      "top-k (oracle/semantica_oracle.c)", **host_info()}


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
    env = Env(args)
    torch, world, rank = env.torch, env.world, env.rank
    quant, dim = args.search_quant, args.search_dim
    var = SearchVariant(env, quant, dim, SEARCH_Q)
    for _ in range(max(args.warmup, 0)):
        var.step(SEARCH_Q)
    torch.cuda.synchronize()
    clocks = ClockSampler(env.uuid())
    clocks.start()
    time.sleep(0.3)
    env.barrier()
    torch.cuda.synchronize()
    ms = events_time(torch, env.stream, lambda: var.step(SEARCH_Q), args.steps)
    env.barrier()
    scan_ms = events_time(torch, env.stream, lambda: var.scan(SEARCH_Q), args.steps)  # the dominant launch
    small = var.small_batches()
    clk = clocks.stop()
    # e2e: float queries from pinned host memory, quantised on the device, ids back to the host
    qscale = 127.0 if quant == 1 else 32767.0
    qf_host = torch.empty((SEARCH_Q, dim), dtype=torch.float32, pin_memory=True)
    qf_host.copy_((var.qcodes.float() / qscale).cpu())
    ids_host = torch.empty((SEARCH_Q, SEARCH_K), dtype=torch.int32, pin_memory=True)
    qf_dev = torch.empty((SEARCH_Q, dim), dtype=torch.float32, device=env.dev)
    q_dev = torch.empty_like(var.qcodes)
    out_ids = np.empty((SEARCH_Q, SEARCH_K), dtype=np.int32)
    out_dist = np.empty((SEARCH_Q, SEARCH_K), dtype=np.float32)
    qf_np = qf_host.numpy()

    def e2e_step():
        if world == 1:
            # Index.SearchVector for the whole batch through the public C ABI:
            # host floats in, ids and distances back in host memory
            env._lib.check(env.lib.sem_index_search(var.h, C.c_void_p(qf_np.ctypes.data), SEARCH_Q, dim, SEARCH_K,
                                                    1, 1, C.c_void_p(out_ids.ctypes.data),
                                                    C.c_void_p(out_dist.ctypes.data), None))
            return
        with torch.cuda.stream(env.stream):
            qf_dev.copy_(qf_host, non_blocking=True)
            n = qf_dev / qf_dev.norm(dim=1, keepdim=True)
            q_dev.copy_(torch.round(n.clamp(-1, 1) * qscale).to(q_dev.dtype))
        var.step(SEARCH_Q, q_dev)
        with torch.cuda.stream(env.stream):
            ids_host.copy_(var.rows, non_blocking=True)
        env.stream.synchronize()

    e2e_step()
    env.barrier()
    t0 = time.perf_counter()
    n_e2e = max(1, min(args.steps, 3))
    for _ in range(n_e2e):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / n_e2e
    env.barrier()
    ms, scan_ms, e2e_s = env.max_over_ranks(ms, scan_ms, e2e_s)
    if rank == 0:
        bf16 = env.peaks.get("bf16_tflops") or 1590.0
        ops = 2.0 * var.per * dim * SEARCH_Q
        traffic = None
        if os.path.exists(TRAFFIC_PATH) and quant == 1 and dim == SEARCH_D:
            bpr = json.load(open(TRAFFIC_PATH)).get("search_tc_bytes_per_corpus_row")
            traffic = bpr * var.per if bpr else None
        metric = search_metric(quant, dim)
        ach = ops / (scan_ms * 1e-3) / 1e12
        line = {"metric": metric, "value": SEARCH_Q / (ms * 1e-3), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "int8 x int8 -> int32" if quant == 1 else "int16 x int16 -> int32 (byte planes on kind::i8)",
                "data": "synthetic",
                "config": search_config(world, quant, dim), "clocks": clk,
                "e2e": {"value": SEARCH_Q / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": SEARCH_Q * dim * 4,
                        "d2h_bytes_per_step": SEARCH_Q * SEARCH_K * (8 if world == 1 else 4),
                        "api": "sem_index_search (host fp32 queries, normalised and quantised on the device)"
                        if world == 1 else "sem_index_search_keys per shard + NCCL all-gather + sem_topk_merge"},
                "gpu_launches": int(args.steps * 3),
                "roofline": {"kernel": ("search_tc_kernel" if quant == 1 else "search_tc16_kernel")
                             + f" (rows of one GPU x {SEARCH_Q} queries)", "bound": "tensor",
                             "achieved": ach, "peak": 2 * bf16, "unit": "TOP/s", "frac": ach / (2 * bf16),
                             "peak_source": "2 x measured bf16_tflops (dense int8 runs at twice the bf16 rate; no "
                                            "int8 figure is measured on this pool)",
                             "algorithmic_ops_per_launch": ops, "launch_ms": scan_ms, "traffic": traffic,
                             "small_batch_hbm": {"peak_gbs": env.peaks.get("hbm_gbs") or 6650.0, **small}}}
        if world == 1 and not args.no_cpu_baseline and quant == 1:
            line["cpu_baseline"] = search_cpu_baseline(var.codes[:1 << 20].cpu().numpy(),
                                                       var.qcodes[:1024].cpu().numpy())
        print(json.dumps(line), flush=True)
    # tensors used on the library's stream (the NCCL all-gather runs there) go
    # first, then the process group, and only then the stream itself
    torch.cuda.synchronize()
    del qf_np, qf_host, ids_host, qf_dev, q_dev  # qf_np views the pinned qf_host
    var.close()
    env.close()


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
    print(json.dumps({"metric": search_metric(), "value": value, "unit": "queries/s", "n_gpus": args.gpus,
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
    ap.add_argument("--legs", default="long,search,gemm,parity",
                    help="extra measurements in the embed line (comma list of long,search,gemm,parity, or none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=1024, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--seq-len", type=int, default=512)
    ap.add_argument("--search-rows", type=int, default=SEARCH_N, help="search corpus rows (profiling runs use fewer)")
    ap.add_argument("--search-queries", type=int, default=SEARCH_Q)
    ap.add_argument("--search-quant", type=int, default=1, choices=[1, 2], help="--workload search: int8 (1) or int16 (2) rows")
    ap.add_argument("--search-dim", type=int, default=SEARCH_D, help="--workload search: vector dimension")
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
