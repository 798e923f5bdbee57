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
        "l2": "inputs larger than L2: ~10 GB of activations and 0.32 GB of weights stream per step",
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
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained (no int8 figure is measured "
                "on this pool; int8 dense nominal is 2x bf16)", "algorithmic_flops_per_launch": flops,
                "launch_ms": per_ms}
    if stage == "attention":
        S = T // n_seqs
        flops = n_seqs * 4.0 * S * S * hd * nh  # scores + P.V of the reference (attention.go:267-310)
        achieved = flops / (per_ms * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained") or 1415.9
        return {"kernel": stage, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": "measured bf16_tflops_sustained",
                "algorithmic_flops_per_launch": flops, "launch_ms": per_ms}
    bytes_per_row = {"quantize": 4 * 1152 + 1152, "residual_norm": 3 * 4 * H, "row_stats": 4 * H,
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
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(path)
        print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    global BATCH, SEQ_LEN
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=1024, help="sequences per GPU (profiling runs use fewer)")
    ap.add_argument("--seq-len", type=int, default=512)
    args = ap.parse_args()
    BATCH, SEQ_LEN = args.batch, args.seq_len
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
