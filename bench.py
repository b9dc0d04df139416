"""Benchmark of the fused Waller attention on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gae|reference]
                    [--workload mha|mha-noncausal|long]

Workloads (synthetic inputs, numpy/torch seeded, iid N(0,1) -> bf16):
  mha            BASELINE config 2, causal: B=4, H=16, N=8192, head_dim=128
  mha-noncausal  the same, non-causal
  long           config 5, causal: one sequence, H=8, head_dim=128, N=131072
  mha64          the attention of config 4 alone: B=8, H=12, N=2048, head_dim=64, causal
  ring           config 5, causal: one sequence of N=1,048,576 (H=8, head_dim=128)
                 sharded over the N GPUs (contiguous N/P shards, ring attention with
                 zig-zag balance, K/V rotated by NCCL send/recv; strong scaling).
                 The default: `--gpus N` measures the north-star ring curve.
  ulysses        config 5 like `ring`, but sequence parallel by head/sequence
                 all-to-all (each rank attends the whole sequence for H/P heads)
  int8           config 3: B=1, H=32, N=16384, head_dim=128, non-causal; Q, K
                 quantised per row to int8 (fp32 scales), V bf16; QK^T on the int8
                 tensor cores (int32 accumulation), P*V in bf16.  Ops counted as
                 4*d per pair like the bf16 path.
  gpt2           config 4: 12 pre-norm GPT-2-small layers (d_model 768, 12 x 64
                 heads, MLP 3072, causal), B=8, seq=2048, weights N(0, 0.02); one
                 step = the whole stack (gae_layer_stack_fwd, replayed as a CUDA
                 graph); FLOPs = GEMMs 2*T*768*9216 + causal attention per layer.
One step = one fused attention forward over the whole batch.  FLOPs count only
visible (unmasked) score entries: 4*d per (query, key) pair, causal pairs
N(N+1)/2 per head.  Inputs (3 x 128 MiB for mha) exceed the 126 MB L2, so no
flush between steps is needed.

--gpus N > 1 (torchrun, one process per GPU): every rank runs its own batch of
the workload (weak scaling; attention over independent (batch, head) units
needs no exchange), except for `ring`, where the ranks share one sequence.  Timing: CUDA events on the launching stream, barrier +
synchronize on both sides, max over ranks.

--impl reference: the reference's CPU attention path (the oracle's restatement
of rust_src/src/waller_operator.rs, OpenMP over rows like
waller_operator_parallel) on the host cores, on a bounded sample of the same
workload (one (batch, head) slice per step), in the same metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "mha": dict(B=4, H=16, N=8192, D=128, causal=True, cfg="config2-causal"),
    "mha-noncausal": dict(B=4, H=16, N=8192, D=128, causal=False, cfg="config2-noncausal"),
    "long": dict(B=1, H=8, N=131072, D=128, causal=True, cfg="config5-131072"),
    "mha64": dict(B=8, H=12, N=2048, D=64, causal=True, cfg="config4-attention-d64"),
    "ring": dict(B=1, H=8, N=1048576, D=128, causal=True, cfg="config5-ring-1M", ring=True),
    # sequence-parallel backward of the same sequence (no reference counterpart)
    "ring-bwd": dict(B=1, H=8, N=1048576, D=128, causal=True, cfg="config5-ring-1M-backward", ring=True,
                     sp="ring-bwd", metric="ring attention backward TFLOPS (bf16 d=128)"),
    "ulysses": dict(B=1, H=8, N=1048576, D=128, causal=True, cfg="config5-ulysses-1M", ring=True,
                    sp="ulysses"),
    "int8": dict(B=1, H=32, N=16384, D=128, causal=False, cfg="config3-int8", int8=True),
    "gpt2": dict(B=8, H=12, N=2048, D=64, causal=True, cfg="config4-gpt2-small-12L", gpt2=True,
                 layers=12, d_model=768, d_ff=3072),
    # training-side backward of config 2 causal (no reference counterpart)
    "mha-bwd": dict(B=4, H=16, N=8192, D=128, causal=True, cfg="config2-causal-backward", bwd=True,
                    metric="attention backward TFLOPS (bf16 d=128)"),
    # the reference's fused symphony layer (waller_fused_layer.cu:64-247) at its
    # benchmark's largest single-launch length with HEAD_DIM 64 (:17, :407)
    "symphony": dict(B=1, H=1, N=131072, D=64, causal=True, cfg="symphony-layer-131072-d64",
                     sym=True, metric="fused symphony layer TFLOPS (d=64, int8 K/V)"),
    # the reference's head_dim-256 fused layer (waller_fused_realistic.cu:151-274)
    # at its benchmark's largest length (:490)
    "symphony256": dict(B=1, H=1, N=65536, D=256, causal=True, cfg="symphony-layer-65536-d256",
                        sym=True, metric="fused symphony layer TFLOPS (d=256, int8 K/V)"),
}
METRIC = "fused-attention TFLOPS (bf16 d=128)"


def attn_flops(B, H, Nq, Nkv, D, causal):
    pairs = Nq * (Nq + 1) // 2 if causal else Nq * Nkv
    return 4.0 * D * B * H * pairs


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}, "fallback"


def profile_traffic(kernel_tag):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/*.md."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".md"):
            continue
        txt = open(os.path.join(d, fn)).read()
        m = re.search(r"traffic_bytes_per_launch\[%s\]:\s*([0-9.eE+]+)" % re.escape(kernel_tag), txt)
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons.  A reader thread
    stamps every sample with the host clock; summary() keeps the samples taken
    inside [t0, t1], the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, period_ms=50):
        self.index, self.period_ms = index, period_ms
        self.proc, self.samples, self.t0, self.t1 = None, [], None, None

    def start(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self

        def reader():
            for ln in self.proc.stdout:
                self.samples.append((time.time(), ln.strip()))
        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        deadline = time.time() + 10
        while not self.samples and time.time() < deadline:  # nvidia-smi is up
            time.sleep(0.05)
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # A sample stamps the end of its period: keep every sample whose
        # period overlaps [t0, t1]; a region shorter than one period still
        # gets the sample that covers it.
        slack = self.period_ms / 1000.0
        for ts, ln in list(self.samples):
            if self.t0 is not None and not (self.t0 <= ts <= self.t1 + slack):
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def symphony_flops(N, D):
    """Causal attention (4*D per query-key pair, as for every workload here),
    the MLP (2 x 2*D*4D per token) and the two RMSNorms (4*D per token each)."""
    return attn_flops(1, 1, N, N, D, True) + 16.0 * N * D * D + 8.0 * N * D


def symphony_arrays(N, D, seed):
    """The reference benchmark's input distribution (waller_fused_layer.cu:
    265-283): inputs uniform in [-0.5, 0.5), K/V uniform int8, weights uniform
    in [-0.05, 0.05), unit norm weights; seeded numpy instead of rand()."""
    import numpy as np
    rng = np.random.default_rng(seed)
    return dict(x=(rng.integers(0, 1000, (N, D)) / 1000.0 - 0.5).astype(np.float32),
                k=rng.integers(-128, 128, (N, D)).astype(np.int8),
                v=rng.integers(-128, 128, (N, D)).astype(np.int8),
                w_up=(rng.integers(0, 1000, (D, 4 * D)) / 10000.0 - 0.05).astype(np.float32),
                w_down=(rng.integers(0, 1000, (4 * D, D)) / 10000.0 - 0.05).astype(np.float32),
                n1=np.ones(D, np.float32), n2=np.ones(D, np.float32))


def make_inputs(torch, w, device, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    shape = (w["B"], w["H"], w["N"], w["D"])
    return [torch.randn(*shape, generator=g).to(torch.bfloat16).to(device) for _ in range(3)]


def cpu_sample(w, slices=8, rows_cap=None):
    """Times the oracle's Waller recurrence (OpenMP over rows, all host
    threads) on `slices` (batch, head) slices of the workload: every query row
    with its full (causal) key range, or `rows_cap` evenly spaced rows per
    slice.  Returns (TFLOPS, seconds, description, threads)."""
    import numpy as np
    from oracle import oracle
    oracle.use_all_cores()
    N, D = w["N"], w["D"]
    rng = np.random.default_rng(1234)
    if w.get("gpt2"):
        # one layer of one sequence (batch 1 of the workload's B), full length
        Dm, F, H = w["d_model"], w["d_ff"], w["H"]
        x = rng.standard_normal((N, Dm)).astype(np.float32)
        mk = lambda *sh: (rng.standard_normal(sh) * 0.02).astype(np.float32)
        wts = dict(ln1_g=np.ones(Dm, np.float32), ln1_b=np.zeros(Dm, np.float32),
                   wqkv=mk(Dm, 3 * Dm), bqkv=np.zeros(3 * Dm, np.float32), wproj=mk(Dm, Dm),
                   bproj=np.zeros(Dm, np.float32), ln2_g=np.ones(Dm, np.float32),
                   ln2_b=np.zeros(Dm, np.float32), wfc=mk(Dm, F), bfc=np.zeros(F, np.float32),
                   wfc2=mk(F, Dm), bfc2=np.zeros(Dm, np.float32))
        oracle.lib()
        t0 = time.perf_counter()
        oracle.gpt2_layer(x, 1, N, Dm, H, F, 1e-5, wts, round_bf16=False)
        dt = time.perf_counter() - t0
        flops = 2.0 * N * Dm * (4 * Dm + 2 * F) + attn_flops(1, H, N, N, D, True)
        return flops / dt / 1e12, dt, f"one layer of one {N}-token sequence (fp32 oracle)", oracle.num_threads()
    if w.get("int8"):
        n_rows = N if rows_cap is None else min(N, rows_cap)
        rows = None if n_rows == N else np.linspace(0, N - 1, n_rows).round().astype(np.int64)
        q, sq = oracle.quantize_rows_int8(rng.standard_normal((slices, N, D)).astype(np.float32))
        k, sk = oracle.quantize_rows_int8(rng.standard_normal((slices, N, D)).astype(np.float32))
        v = rng.standard_normal((slices, N, D)).astype(np.float32)
        t0 = time.perf_counter()
        oracle.attention_int8(q, k, sq, sk, v, 1.0 / math.sqrt(D), causal=w["causal"], rows=rows)
        dt = time.perf_counter() - t0
        flops = 4.0 * D * n_rows * N * slices
        return (flops / dt / 1e12, dt, f"{slices} head(s) x {n_rows} query rows, full key range each",
                oracle.num_threads())
    if w.get("bwd") or w.get("sp") == "ring-bwd":
        # gradients of one (batch, head) slice over its first `rows_cap` tokens
        # (a causal prefix is a complete problem of its own)
        n = N if rows_cap is None else min(N, rows_cap)
        q, k, v, g = (rng.standard_normal((slices, n, D)).astype(np.float32) for _ in range(4))
        oracle.lib()
        t0 = time.perf_counter()
        oracle.attention_bwd(q, k, v, g, 1.0 / math.sqrt(D), w["causal"])
        dt = time.perf_counter() - t0
        return (2.5 * attn_flops(1, slices, n, n, D, w["causal"]) / dt / 1e12, dt,
                f"gradients of {slices} slice(s) over the first {n} tokens (float64 oracle)",
                oracle.num_threads())
    if w.get("sym"):
        # the first `rows_cap` tokens: a causal prefix is a complete layer of its own
        n = N if rows_cap is None else min(N, rows_cap)
        a = symphony_arrays(n, D, 1234)
        tf = (1.0 / (math.sqrt(D) * 127.0 * 127.0), 1.0, 1.0, 1.0, 1e-6, 1.0, 1.0)
        oracle.lib()
        t0 = time.perf_counter()
        oracle.symphony_layer(a["x"], a["k"], a["v"], a["w_up"], a["w_down"], a["n1"], a["n2"], tf, 0)
        dt = time.perf_counter() - t0
        return (symphony_flops(n, D) / dt / 1e12, dt,
                f"symphony layer over the first {n} tokens (causal prefix, fp32 oracle)",
                oracle.num_threads())
    q, k, v = (rng.standard_normal((1, slices, N, D)).astype(np.float32) for _ in range(3))
    n_rows = N if rows_cap is None else min(N, rows_cap)
    rows = None if n_rows == N else np.linspace(0, N - 1, n_rows).round().astype(np.int64)
    oracle.lib()
    t0 = time.perf_counter()
    oracle.attention_batched(q, k, v, 1.0 / math.sqrt(D), w["causal"], rows=rows)
    dt = time.perf_counter() - t0
    if rows is None:
        flops = attn_flops(1, slices, N, N, D, w["causal"])
        desc = (f"{slices} (batch, head) slice(s) of {N} query rows, each with its full "
                f"{'causal ' if w['causal'] else ''}key range")
    else:
        pairs = float(np.sum(rows + 1)) if w["causal"] else float(n_rows * N)
        flops = 4.0 * D * pairs * slices
        desc = (f"{slices} slice(s) x {n_rows} evenly spaced query rows, each with its full "
                f"{'causal ' if w['causal'] else ''}key range")
    return flops / dt / 1e12, dt, desc, oracle.num_threads()


def run_reference(args, w):
    """The reference arm: the CPU path on a bounded sample per step, sized so
    that warm-up plus timed steps take about two minutes in total."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if w.get("gpt2"):
        vals, secs = [], []
        for _ in range(args.warmup):
            cpu_sample(w)
        for _ in range(min(args.steps, 5)):
            v, s, desc, threads = cpu_sample(w)
            vals.append(v); secs.append(s)
        return _print_reference(args, w, statistics.mean(vals), statistics.mean(secs), desc, threads)
    if w.get("bwd") or w.get("sp") == "ring-bwd":
        budget = 120.0 / (args.steps + args.warmup)
        _, s_cal, _, _ = cpu_sample(w, slices=1, rows_cap=512)
        n = int(min(w["N"], 512 * math.sqrt(budget / max(s_cal, 1e-6))))
        n = max(256, n // 128 * 128)
        for _ in range(args.warmup):
            cpu_sample(w, slices=1, rows_cap=n)
        vals, secs = [], []
        for _ in range(args.steps):
            v_, s_, desc, threads = cpu_sample(w, slices=1, rows_cap=n)
            vals.append(v_); secs.append(s_)
        return _print_reference(args, w, statistics.mean(vals), statistics.mean(secs), desc, threads)
    if w.get("sym") and args.reference_kernel:
        return run_reference_kernel(args, w)
    if args.reference_kernel:
        return run_reference_chain(args, w)
    if w.get("sym"):
        # cost grows with the square of the prefix length: calibrate at 4096
        _, s_cal, _, _ = cpu_sample(w, rows_cap=4096)
        budget = 120.0 / (args.steps + args.warmup)
        n = int(min(w["N"], 4096 * math.sqrt(budget / max(s_cal, 1e-6))))
        n = max(1024, n // 256 * 256)
        for _ in range(args.warmup):
            cpu_sample(w, rows_cap=n)
        vals, secs = [], []
        for _ in range(args.steps):
            v, s, desc, threads = cpu_sample(w, rows_cap=n)
            vals.append(v); secs.append(s)
        return _print_reference(args, w, statistics.mean(vals), statistics.mean(secs), desc, threads)
    # Calibrate: seconds per row of one slice (full key range).
    _, s_cal, _, _ = cpu_sample(w, slices=1, rows_cap=256)
    per_row = s_cal / 256
    budget = 120.0 / (args.steps + args.warmup)
    rows_cap = int(max(64, min(w["N"], budget / per_row)))
    for _ in range(args.warmup):
        cpu_sample(w, slices=1, rows_cap=rows_cap)
    vals, secs = [], []
    desc, threads = "", 1
    for _ in range(args.steps):
        v, s, desc, threads = cpu_sample(w, slices=1, rows_cap=rows_cap)
        vals.append(v)
        secs.append(s)
    return _print_reference(args, w, statistics.mean(vals), statistics.mean(secs), desc, threads)


def run_reference_kernel(args, w):
    """The reference's own symphony CUDA kernel (built from its source into
    oracle/_ref by the oracle's Makefile) on this GPU, same workload and input
    distribution; CUDA-event timed.  A comparison point, not the CPU arm."""
    import torch
    from oracle import oracle
    N, D = w["N"], w["D"]
    if D == 64:
        L = oracle.ref_symphony()
        fwd = L.ref_symphony_fwd if L is not None else None
    else:
        L = oracle.ref_symphony128()
        fwd = getattr(L, f"ref_symphony{D}_fwd", None) if L is not None else None
    if fwd is None:
        emit({"impl": "reference", "unavailable":
                          "reference symphony kernel not built (oracle/_ref missing)"})
        return 0
    a = {n_: torch.from_numpy(v_).cuda() for n_, v_ in symphony_arrays(N, D, 1000).items()}
    out = torch.empty_like(a["x"])
    tf = np.asarray((1.0 / (math.sqrt(D) * 127.0 * 127.0), 1.0, 1.0, 1.0, 1e-6, 1.0, 1.0), np.float32)
    st = torch.cuda.current_stream()

    def launch():
        rc = fwd(a["k"].data_ptr(), a["v"].data_ptr(), a["w_up"].data_ptr(),
                                a["w_down"].data_ptr(), a["n1"].data_ptr(), a["n2"].data_ptr(),
                                a["x"].data_ptr(), out.data_ptr(), N, tf, 0, st.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"reference kernel launch failed: {rc}")

    launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(args.steps, 3))
    e0.record(st)
    for _ in range(steps):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    value = symphony_flops(N, D) / (ms * 1e-3) / 1e12
    emit({"impl": "reference", "kind": "reference-gpu-kernel",
                      "metric": w.get("metric", METRIC), "value": value, "unit": "TFLOPS",
                      "ms_per_step": ms, "steps": steps, "n_gpus": 1,
                      "config": {"workload": w["cfg"], "seq_len": N, "head_dim": D}})
    return 0


def run_reference_chain(args, w):
    """The reference's published GPU attention chain (cuda_src/
    waller_kernel_bench.cu: per tile cuBLAS fp16 QK^T, an online-softmax
    kernel, cuBLAS P*V and an update kernel; built from its source into
    oracle/_ref) on this GPU, one sequence (head) at a time as it runs, with
    its own tile auto-tuning over {512, 1024, 2048, 4096}.  Reported in this
    repository's FLOP convention (visible pairs only) and in the reference's
    (4 N^2 d per head, :272).  A comparison point, not the CPU arm."""
    from oracle import oracle
    L = oracle.ref_kernel_bench()
    if L is None:
        emit({"impl": "reference", "unavailable":
                          "reference kernel chain not built (oracle/_ref missing)"})
        return 0
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    N, D, H, B = w["N"], w["D"], w["H"], w["B"]
    if N > 131072:  # one launch list per row tile: keep the run bounded
        N = 131072
    tiles = [t for t in (512, 1024, 2048, 4096) if t <= N]
    sweep = {t: float(L.ref_kernel_bench_tflops(N, D, t, 1)) for t in tiles}
    best = max(sweep, key=sweep.get)
    iters = max(1, min(args.steps, 3))
    ref_tflops = float(L.ref_kernel_bench_tflops(N, D, best, iters))
    ms_head = 4.0 * N * N * D / (ref_tflops * 1e12) * 1e3
    ours = attn_flops(1, 1, N, N, D, w["causal"]) / (ms_head * 1e-3) / 1e12
    emit({"impl": "reference", "kind": "reference-gpu-kernel-chain",
                      "metric": w.get("metric", METRIC), "value": ours, "unit": "TFLOPS",
                      "value_reference_convention": ref_tflops,
                      "flop_conventions": {"value": "4*d per visible (causal) pair",
                                           "value_reference_convention": "4*N^2*d per head (waller_kernel_bench.cu:272)"},
                      "ms_per_head": ms_head, "tile": best,
                      "tile_sweep_reference_convention": sweep, "steps": iters, "n_gpus": 1,
                      "dtype": "f16", "config": {"workload": w["cfg"], "seq_len": N, "head_dim": D,
                                                 "heads_timed_as": "one sequence, scaled by B*H"}})
    return 0


def _print_reference(args, w, value, sec, desc, threads):
    line = {
        "impl": "reference", "metric": w.get("metric", METRIC), "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * sec, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w["cfg"], "B": w["B"], "H": w["H"], "seq_len": w["N"],
                   "head_dim": w["D"], "causal": w["causal"]},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": threads, "kind": "port",
                         "sample": desc + " per step"},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


_JSON_FD = None


def emit(line: dict):
    """Prints the one JSON result line on the process's real stdout."""
    text = json.dumps(line) + "\n"
    if _JSON_FD is None:
        print(text, end="", flush=True)
    else:
        os.write(_JSON_FD, text.encode())


def main():
    # Everything else that reaches file descriptor 1 (libraries' banners,
    # e.g. NCCL's version line) goes to stderr; the JSON line keeps stdout.
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="gae", choices=["gae", "reference"])
    ap.add_argument("--workload", default="ring", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--reference-kernel", action="store_true",
                    help="with --impl reference: time the reference's own CUDA code on this GPU "
                         "(oracle/_ref: its symphony kernel for --workload symphony, else its "
                         "published cuBLAS+SIMT attention chain) instead of the CPU path")
    ap.add_argument("--seq-len", type=int, default=None,
                    help="override the workload's sequence length (small profiling cases)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    w = WORKLOADS[args.workload]
    if args.seq_len:
        w = dict(w, N=args.seq_len)
    if args.impl == "reference":
        return run_reference(args, w)

    import torch
    import torch.distributed as dist
    import __graft_entry__ as ge
    gae = ge.load_package()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    B, H, N, D, causal = w["B"], w["H"], w["N"], w["D"], w["causal"]
    is_ring = bool(w.get("ring"))
    stream = torch.cuda.current_stream()
    is_int8 = bool(w.get("int8"))
    is_gpt2 = bool(w.get("gpt2"))
    is_sym = bool(w.get("sym"))
    is_bwd = bool(w.get("bwd"))
    if is_bwd:
        q0, k, v = make_inputs(torch, w, dev, 1000 + rank)
        o0, lse0 = gae.attention(q0, k, v, causal=causal, return_lse=True)
        g = torch.Generator(device="cpu").manual_seed(2000 + rank)
        do0 = torch.randn(q0.shape, generator=g).to(torch.bfloat16).to(dev)
        q = (q0, o0, do0, lse0)
        grads = torch.empty((3,) + tuple(q0.shape), dtype=q0.dtype, device=dev)
        out = grads
        bws = torch.empty(gae.lib().gae_attn_bwd_workspace_bytes(B, H, N, D), dtype=torch.uint8, device=dev)
        flops = 2.5 * attn_flops(B, H, N, N, D, causal)  # S recomputed, dP, dV, dK, dQ

        def run_step(q, k, v):
            gae.attention_backward(q[0], k, v, q[1], q[2], q[3], causal=causal, dq=grads[0], dk=grads[1],
                                   dv=grads[2], workspace=bws)
    elif is_sym:
        arrs = symphony_arrays(N, D, 1000 + rank)
        sd = {n_: torch.from_numpy(a_).to(dev) for n_, a_ in arrs.items()}
        tf = gae.TuningFork.reference_defaults(D)
        q, k, v = sd["x"], sd["k"], sd["v"]
        out = torch.empty_like(q)
        ws = torch.empty(gae.lib().gae_symphony_workspace_bytes(N, D), dtype=torch.uint8, device=dev)
        flops = symphony_flops(N, D)

        def run_step(q, k, v):
            gae.symphony_forward(q, k, v, sd["w_up"], sd["w_down"], sd["n1"], sd["n2"], tf,
                                 out=out, workspace=ws)
    elif is_gpt2:
        T = B * N
        L = w["layers"]
        gemm = 2.0 * T * w["d_model"] * (3 * w["d_model"] + w["d_model"] + 2 * w["d_ff"])
        flops = L * (gemm + attn_flops(B, H, N, N, D, True))
        layers = [gae.Gpt2Layer.random(w["d_model"], H, w["d_ff"], device=dev, seed=100 + i)
                  for i in range(L)]
        g = torch.Generator(device="cpu").manual_seed(1000 + rank)
        q = torch.randn(B, N, w["d_model"], generator=g).to(torch.bfloat16).to(dev)
        k = v = q  # e2e copies only the input activations
        out = torch.empty_like(q)
        ws = layers[0].workspace(B, N, dev)
        graph_in = torch.empty_like(q)
        graph = torch.cuda.CUDAGraph()
        gae.layer_stack_forward(layers, q, out=out, workspace=ws)  # warm the launch path
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            gae.layer_stack_forward(layers, graph_in, out=out, workspace=ws)

        def run_step(q, k, v):
            if q.data_ptr() != graph_in.data_ptr():
                graph_in.copy_(q, non_blocking=True)
            graph.replay()
    elif is_int8:
        gen = torch.Generator(device="cpu").manual_seed(1000 + rank)
        xq = torch.randn(B * H, N, D, generator=gen).to(dev)
        xk = torch.randn(B * H, N, D, generator=gen).to(dev)
        v = torch.randn(B * H, N, D, generator=gen).to(torch.bfloat16).to(dev)
        qi, qs = gae.quantize_rows_int8(xq)
        ki, ks = gae.quantize_rows_int8(xk)
        del xq, xk
        out = torch.empty_like(v)
        flops = attn_flops(B, H, N, N, D, causal)
        q, k = (qi, qs), (ki, ks)

        def run_step(q, k, v):
            gae.attention_int8(q[0], k[0], q[1], k[1], v, causal=causal, out=out)
    elif is_ring:
        from gae_b200 import ring
        S = N // world
        ws = dict(w, N=S)
        q, k, v = make_inputs(torch, ws, dev, 1000 + rank)
        out = torch.empty_like(q)
        flops = attn_flops(B, H, N, N, D, causal) / world  # per rank share of the job

        if w.get("sp") == "ring-bwd":
            q0 = q
            o0, lse0 = ring.ring_attention(q0, k, v, causal=causal, return_lse=True)
            g = torch.Generator(device="cpu").manual_seed(2000 + rank)
            do0 = torch.randn(q0.shape, generator=g).to(torch.bfloat16).to(dev)
            q = (q0, o0, do0, lse0)
            out = torch.empty((3,) + tuple(q0.shape), dtype=q0.dtype, device=dev)
            flops = 2.5 * attn_flops(B, H, N, N, D, causal) / world

            def run_step(q, k, v):
                for dst, src in zip(out, ring.ring_attention_backward(q[0], k, v, q[1], q[2], q[3],
                                                                      causal=causal)):
                    dst.copy_(src)
        elif w.get("sp") == "ulysses":
            from gae_b200 import ulysses

            def run_step(q, k, v):
                out.copy_(ulysses.ulysses_attention(q, k, v, causal=causal))
        else:
            def run_step(q, k, v):
                out.copy_(ring.ring_attention(q, k, v, causal=causal))
    else:
        q, k, v = make_inputs(torch, w, dev, 1000 + rank)
        out = torch.empty_like(q)
        flops = attn_flops(B, H, N, N, D, causal)

        def run_step(q, k, v):
            gae.attention(q, k, v, causal=causal, out=out)

    # ---- device-resident timing (value, roofline) -------------------------
    # Bytes a step reads and writes; under twice the 126 MB L2, the L2 is
    # flushed (a 256 MiB write, outside the timed spans) before every step.
    def _flat(t):
        return list(t) if isinstance(t, tuple) else [t]
    seen, step_bytes = set(), 0
    for t in _flat(q) + _flat(k) + _flat(v) + [out]:
        if t.data_ptr() not in seen:
            seen.add(t.data_ptr())
            step_bytes += t.numel() * t.element_size()
    flush_l2 = step_bytes < 2 * 126e6
    l2_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush_l2 else None
    for _ in range(args.warmup):
        run_step(q, k, v)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    span_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)] if flush_l2 else []
    clk = ClockSampler(local).start()
    barrier()
    clk.t0 = time.time()
    ev0.record(stream)
    for i in range(args.steps):
        if flush_l2:
            l2_buf.fill_(i & 0xFF)
            span_ev[i][0].record(stream)
        run_step(q, k, v)
        if flush_l2:
            span_ev[i][1].record(stream)
    ev1.record(stream)
    barrier()
    clk.t1 = time.time()
    clk.stop()
    gae.device_status()
    if flush_l2:
        ev_ms = sum(a.elapsed_time(b) for a, b in span_ev)
    else:
        ev_ms = ev0.elapsed_time(ev1)
    t_ms = max_over_ranks(ev_ms)
    ms_step = t_ms / args.steps
    value = world * flops / (ms_step * 1e-3) / 1e12

    # kernels of this library per step: the ring runs 3 block pairs + 1 merge at
    # P=1 and 2 pairs + 2 merges per further step (zig-zag balance).
    if is_ring and w.get("sp") == "ulysses":
        launches_per_step = 1
    else:
        # the C-ABI ring on rank 0: 1 launch at P=1; otherwise 9 re-deal
        # copies, 1 fill, 2 block launches + 2 merges at step 0 and 1 + 1 per
        # further step, 4 copies of the output re-deal
        launches_per_step = ((1 if world == 1 else 18 + 2 * (world - 1)) if is_ring
                             else (7 * w["layers"] if is_gpt2 else 1))
    if is_sym:
        launches_per_step = 3  # prep, attention, post
    if is_bwd:
        launches_per_step = 3  # dO.O row sums, backward, dQ conversion (plus one memset)
    if is_ring and w.get("sp") == "ring-bwd":
        launches_per_step = 3 * (3 + 2 * (world - 1))  # block pairs (zig-zag) x 3 launches

    # ---- end to end through the public API with host buffers ---------------
    def flat(t):
        return list(t) if isinstance(t, tuple) else [t]

    inputs = flat(q) + ([] if is_gpt2 else flat(k) + flat(v))
    host_in = [t.cpu().pin_memory() for t in inputs]
    dev_bufs = [[torch.empty_like(t) for t in inputs] for _ in range(2)]  # double-buffered inputs
    hout = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def regroup(ts):
        if is_gpt2:
            return ts[0], ts[0], ts[0]
        if is_int8:
            return (ts[0], ts[1]), (ts[2], ts[3]), ts[4]
        if is_bwd or (is_ring and w.get("sp") == "ring-bwd"):
            return (ts[0], ts[1], ts[2], ts[3]), ts[4], ts[5]
        return ts[0], ts[1], ts[2]

    # Pipelined end to end: the host->device copy of step i+1 (copy stream)
    # overlaps the compute of step i, and the device->host read of step i
    # (second copy stream) overlaps the next copy in.  Every step still copies
    # its own inputs in and its own result out inside the timed region.
    s_h2d, s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_h2d = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_d2h = torch.cuda.Event()

    def run_e2e(n, start_ev=None, end_ev=None):
        if start_ev is not None:
            start_ev.record(stream)
            s_h2d.wait_stream(stream)

        def h2d(i):
            with torch.cuda.stream(s_h2d):
                if i >= 2:
                    s_h2d.wait_event(ev_comp[i % 2])  # buffer free again
                for d_, h_ in zip(dev_bufs[i % 2], host_in):
                    d_.copy_(h_, non_blocking=True)
                ev_h2d[i % 2].record(s_h2d)

        h2d(0)
        for i in range(n):
            if i + 1 < n:
                h2d(i + 1)
            stream.wait_event(ev_h2d[i % 2])
            if i > 0:
                stream.wait_event(ev_d2h)  # the previous result has left `out`
            run_step(*regroup(dev_bufs[i % 2]))
            ev_comp[i % 2].record(stream)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_comp[i % 2])
                hout.copy_(out, non_blocking=True)
                ev_d2h.record(s_d2h)
        stream.wait_event(ev_d2h)
        stream.wait_stream(s_h2d)
        if end_ev is not None:
            end_ev.record(stream)

    run_e2e(2)
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    run_e2e(e2e_steps, ev0, ev1)
    barrier()
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1)) / e2e_steps
    e2e_value = world * flops / (e2e_ms * 1e-3) / 1e12
    bytes_in = sum(t.numel() * t.element_size() for t in inputs)
    bytes_out = out.numel() * out.element_size()

    if world > 1:
        dist.barrier()
    if rank != 0:
        dist.destroy_process_group()
        return 0

    peaks, peak_kind = measured_peaks()
    achieved = flops / (ms_step * 1e-3) / 1e12

    # The north-star single-GPU target (config 5 at N=131072, H=8, d=128,
    # causal) measured in the same run beside the 1M-token ring's P=1 line.
    north_star = None
    if is_ring and world == 1 and not w.get("sp"):
        wl = WORKLOADS["long"]
        ql, kl, vl = make_inputs(torch, wl, dev, 77)
        ol = torch.empty_like(ql)
        for _ in range(3):
            gae.attention(ql, kl, vl, causal=True, out=ol)
        n_l = 20
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(n_l):
            gae.attention(ql, kl, vl, causal=True, out=ol)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms_l = ev0.elapsed_time(ev1) / n_l
        v_l = attn_flops(wl["B"], wl["H"], wl["N"], wl["N"], wl["D"], True) / (ms_l * 1e-3) / 1e12
        north_star = {"workload": wl["cfg"], "value": v_l, "unit": "TFLOPS", "ms_per_step": ms_l,
                      "steps": n_l, "frac_of_peak": v_l / peaks["bf16_tflops"],
                      "target_frac": 0.60}
        del ql, kl, vl, ol
    peak = peaks["bf16_tflops"]
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_kind": f"{peak_kind} bf16 burst",
                "traffic": profile_traffic(args.workload)}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        if is_sym:
            v_cpu, s_cpu, desc, threads = cpu_sample(w, rows_cap=16384)
        elif is_bwd or w.get("sp") == "ring-bwd":
            v_cpu, s_cpu, desc, threads = cpu_sample(w, slices=1, rows_cap=1024)
        elif w.get("int8"):
            v_cpu, s_cpu, desc, threads = cpu_sample(w, slices=2, rows_cap=2048)
        else:
            if w["N"] <= 16384:
                v_cpu, s_cpu, desc, threads = cpu_sample(w, slices=8)
            elif w["N"] <= 131072:
                v_cpu, s_cpu, desc, threads = cpu_sample(w, slices=8, rows_cap=2048)
            else:  # 1M tokens: one head, 512 rows over the sequence (~10 s on 32 cores)
                v_cpu, s_cpu, desc, threads = cpu_sample(w, slices=1, rows_cap=512)
        cpu = {"value": v_cpu, "unit": "TFLOPS", "cores": threads, "kind": "port",
               "sample": desc + f" ({s_cpu:.1f} s)"}

    line = {
        "metric": w.get("metric", METRIC), "value": value, "unit": "TFLOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "strong" if is_ring else "weak",
        "vs_baseline": None,
        "dtype": "int8+f16+f32" if is_sym else ("int8+bf16" if is_int8 else "bf16"),
        "data": "synthetic",
        "config": {"workload": w["cfg"], "B": B, "H": H, "seq_len": N, "head_dim": D,
                   "causal": causal, "global_batch": B if is_ring else B * world,
                   "parallelism": ((f"{w.get('sp', 'ring')}-sp{world}") if is_ring else f"dp{world}") if world > 1 else "single",
                   "l2": ("L2 flushed before each step (256 MiB write outside the timed spans)"
                          if flush_l2 else "inputs larger than L2 (no flush)")},
        "e2e": {"value": e2e_value, "unit": "TFLOPS", "h2d_bytes_per_step": bytes_in,
                "d2h_bytes_per_step": bytes_out, "ms_per_step": e2e_ms,
                "pipelined": "H2D of step i+1 and D2H of step i overlap compute"},
        "gpu_launches": args.steps * launches_per_step,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
        "pct_of_tensor_peak": 100.0 * achieved / peak,
    }
    if north_star is not None:
        line["north_star_131072"] = north_star
    if is_int8:
        # Survey 8(d)'s split: QK^T (half the ops) against the int8 tensor peak,
        # taken as twice the measured bf16 peak (the dense int8 rate is twice
        # bf16's), and P*V against the bf16 peak.
        t_s = ms_step * 1e-3
        line["pct_of_peak_split"] = 100.0 * (flops / 2 / (2 * peak * 1e12) + flops / 2 / (peak * 1e12)) / t_s
        line["pct_of_peak_split_note"] = "QK^T ops / (2 x measured bf16 peak) + PV FLOP / bf16 peak, over the step time"
    emit(line)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
