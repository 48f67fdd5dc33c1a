"""Benchmark: batch-1 greedy decode tokens/s of the Qwen3-4B-shaped Q6_K model
on B200. The roofline object is the step kernel's (one launch per token: the dominant and only
kernel of the decode loop) against measured HBM bandwidth; the drop-in config-0 Q6_K GEMV is
reported beside it (gemv_config0), with the CPU baseline.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]
                  [--prompt P] [--layers L] [--tp]

--prompt sets the prefill length (default: the config's own, 128 / 4000 / 512 for configs 1 / 2 / 3);
--layers cuts the model to L layers for small ncu captures only (the line then names the layer
count and is not a measurement of the config). --tp (with N > 1 ranks) splits ONE model over the
ranks (tensor parallel, config 3: `--config qwen3-14b --tp`): value = that one sequence's tokens/s,
scaling "strong"; without it the N ranks are independent replicas (configs 1 and 2).

One JSON line is printed by rank 0. A step is one decode token (batch 1). Inputs are synthetic
(seeded random-init GGUF of the config's exact shapes; no checkpoints exist offline). With N > 1,
every rank decodes its own replica (weak scaling, no data-path collective); the value is the sum
over ranks of tokens / max-over-ranks time.

--impl reference times the reference's algorithm on the host cores (the oracle port of the token
loop, oracle/fence_oracle.c, all threads), on the same config; only rank 0 runs it.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
from __graft_entry__ import _load_pkg  # noqa: E402

PROMPT_LEN = {"qwen3-4b": 128, "llama3-8b-q8": 4000, "qwen3-14b": 512}
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
CONFIG0_BYTES = 4096 * 16 * 210 + 4096 * 2 + 4096 * 4  # W + fp16 x + fp32 y = 13,787,136


def hbm_peak():
    try:
        v = json.load(open(PEAKS_PATH))["hbm_gbs"]
        return float(v), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_from_profiles(name, key="traffic_bytes_per_launch"):
    """A per-launch DRAM byte count recorded in a committed ncu summary under profiles/, if any."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(p):
            if line.startswith(key + ":"):
                return int(line.split(":")[1].strip())
    except (OSError, ValueError):
        pass
    return None


def traffic_ratio_from_profiles(name):
    """DRAM bytes / algorithmic bytes of one step-kernel launch, from a committed ncu summary of a
    smaller cut of the same config (the traffic scales with the bytes streamed)."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name)):
            if line.startswith("traffic_ratio:"):
                return float(line.split(":")[1].strip())
    except (OSError, ValueError):
        pass
    return None


def step_algorithmic_bytes(cfg, positions):
    """Bytes one decode token must move (the roofline numerator): every weight streamed once
    (layer linears + the tied LM head, weight_bytes), the token's embedding row, and the K and V
    rows of the context read by attention (fp16), averaged over the timed positions."""
    kv_dim = cfg.n_kv_heads * cfg.head_dim
    embed_row = cfg.embed_dim // 32 * 34
    kv = sum(2 * cfg.n_layers * (p + 1) * kv_dim * 2 for p in positions) / max(1, len(positions))
    return int(cfg.weight_bytes + embed_row + kv)


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]
        else:
            self.lines = []

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def synth_model(fb, config, tmp, layers=0):
    path = os.path.join(tmp, f"{config}.gguf")
    if layers > 0:
        fb.synth_write(path, config, seed=2024, n_layers=layers)
    else:
        fb.synth_write(path, config, seed=2024)
    return path


def measure_gemv_roofline(fb, torch, copies=32, launches=256, pdl=True):
    """Config-0 Q6_K GEMV (4096x4096) through the drop-in C-ABI, rotating over `copies` weight
    copies (> L2) so every launch streams from HBM: one launch per copy captured in a CUDA graph,
    the graph replayed back to back; CUDA events on the replay stream. With pdl=True the launches
    use FENCE_LAUNCH_PDL (weights are never written), so each GEMV starts streaming while the
    previous one drains, as inside the decode step."""
    fb.lib().fence_set_launch_flags(fb.FENCE_LAUNCH_PDL if pdl else 0)
    M = K = 4096
    nblk = M * K // 256
    W = np.frombuffer(fb.synth_blocks(fb.GGML_Q6_K, nblk, seed=0), np.uint8)
    dW = torch.empty((copies, W.size), dtype=torch.uint8, device="cuda")
    dW[:] = torch.from_numpy(W.copy()).cuda()
    x = np.random.default_rng(0).standard_normal(K).astype(np.float32).astype(np.float16).view(np.int16)
    dx = torch.from_numpy(x.copy()).cuda()
    dy = torch.empty(M, dtype=torch.float32, device="cuda")
    L = fb.lib()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(copies):  # warm-up (and the kernel's shared-memory attribute) outside capture
            fb.check(L.fence_gemv_q6k(dW[i].data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, st.cuda_stream))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(copies):
            fb.check(L.fence_gemv_q6k(dW[i].data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K,
                                      torch.cuda.current_stream().cuda_stream))
    reps = max(1, launches // copies)
    with torch.cuda.stream(st):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    fb.lib().fence_set_launch_flags(0)
    del g, dW
    return ms


def cpu_decode_sample(path, budget_s, max_tokens, threads):
    """Oracle port of the token loop on the host cores: decode tokens at positions 0.. until the time
    budget is spent (at least one). Returns (tokens, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc  # CPU-baseline leg only
    m = orc.OracleModel(path, max_ctx=4096, kv_bf16=True, threads=threads)
    rng = np.random.default_rng(0)
    n, t0 = 0, time.perf_counter()
    while n < max_tokens:
        m.forward(int(rng.integers(0, m.vocab_size)), n)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    m.close()
    return n, dt


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    fb = _load_pkg()
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        path = synth_model(fb, args.config, tmp)
        # warm-up: touch the weights once (page cache) with one token
        cpu_decode_sample(path, 0.0, 1, threads)
        budget = min(150.0, 2.0 * max(args.steps, 1))
        n, dt = cpu_decode_sample(path, budget, args.steps, threads)
    value = n / dt
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": round(value, 4), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "warmup": 1, "ms_per_step": round(1e3 * dt / n, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic", "config": {"workload": f"{args.config} batch-1 greedy decode (CPU, reference algorithm)",
                                        "model": args.config},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{n} decode tokens at positions 0..{n - 1} of {args.config}, "
                                   f"oracle/fence_oracle.c on {threads} threads (steps bounded to {n} of {args.steps} "
                                   f"requested by a {150:.0f} s budget)"},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=248)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3-4b")
    ap.add_argument("--prompt", type=int, default=None, help="prefill tokens (default: the config's own)")
    ap.add_argument("--layers", type=int, default=0, help="cut the model to this many layers (ncu captures)")
    ap.add_argument("--tp", action="store_true",
                    help="with N > 1: one model split over the N ranks (tensor parallel, strong scaling) instead "
                         "of N independent replicas (the default for configs 1 and 2)")
    ap.add_argument("--kv", default="f16", choices=["f16", "bf16"])
    ap.add_argument("--tmp", default=None, help="directory for the synthetic GGUF (default: /dev/shm if roomy)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", default="decode", choices=["decode", "gemv"],
                    help="gemv: only the config-0 Q6_K GEMV roofline measurement (small; used for ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.prompt is None:
        args.prompt = PROMPT_LEN.get(args.config, 128)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.tmp is None:
        try:
            st = os.statvfs("/dev/shm")
            need = 12e9 * world + 12e9  # one model file per rank (+ the CPU-baseline copy)
            args.tmp = "/dev/shm" if st.f_bavail * st.f_frsize > need else None
        except OSError:
            args.tmp = None

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    torch.cuda.set_device(local)
    if args.mode == "gemv":
        fb = _load_pkg()
        peak, peak_kind = hbm_peak()
        ms = measure_gemv_roofline(fb, torch, copies=16, launches=max(args.steps, 1), pdl=True)
        print(json.dumps({"metric": "gemv_q6k_config0_GBps", "value": round(CONFIG0_BYTES / (ms * 1e-3) / 1e9, 1),
                          "unit": "GB/s", "us_per_launch": round(ms * 1e3, 3), "peak": peak, "peak_kind": peak_kind}))
        return
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    fb = _load_pkg()
    tp = args.tp and world > 1
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        if tp:
            # one model file for all ranks: rank 0 writes it, the others read it (same host)
            gloo = dist.new_group(backend="gloo")
            box = [tmp]
            dist.broadcast_object_list(box, src=0, group=gloo)
            path = os.path.join(box[0], f"{args.config}.gguf")
            if rank == 0:
                synth_model(fb, args.config, box[0], args.layers)
            dist.barrier(group=gloo)
        else:
            # every rank writes its own copy (same seed -> identical bytes); ranks stay independent
            path = synth_model(fb, args.config, tmp, args.layers)
        kv = fb.FENCE_KV_F16 if args.kv == "f16" else fb.FENCE_KV_BF16
        e2e_steps = min(args.steps, max(16, args.steps // 2))
        total_pos = args.prompt + args.warmup + args.steps + e2e_steps + 8
        max_ctx = max(4096, total_pos)
        if tp:
            model = fb.Model(path, max_ctx=max_ctx, kv_dtype=kv, device=local, tp_rank=rank, tp_size=world)
            import fence_b200.tp as fbtp
            fbtp.connect(model, gloo)
            dist.barrier(group=gloo)  # every rank has read the file before rank 0 removes it
        else:
            model = fb.Model(path, max_ctx=max_ctx, kv_dtype=kv, device=local)
        cfg = model.config
        rng = np.random.default_rng(7 if tp else 7 + rank)  # tensor parallel: every rank feeds the same tokens
        prompt = [int(t) for t in rng.integers(0, cfg.vocab_size, args.prompt)]
        # prefill (token by token, as the reference) — untimed
        d = None
        for pos, t in enumerate(prompt):
            d = model.forward(t, pos)
        first = model.sample_greedy(d)
        pos = args.prompt
        # warm-up decode steps (device-resident chain)
        warm_ids = model.decode_greedy(first, pos, args.warmup)
        pos += args.warmup
        tok = warm_ids[-1]
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        with ClockSampler(local) as clk:
            torch.cuda.synchronize()
            ms = model.time_decode(tok, pos, args.steps)
            torch.cuda.synchronize()
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        pos += args.steps
        tok_s = args.steps / (ms / 1e3)
        value = tok_s if tp else tok_s * world  # one sequence over all ranks / one per replica

        # e2e through the reference-facing API: forward(token, pos) from the host (16-byte state
        # H2D from pinned memory) + sample_greedy (4-byte id D2H + sync) every step
        e2e_pos = pos
        nxt = tok
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            dl = model.forward(nxt, e2e_pos + i)
            nxt = model.sample_greedy(dl)
        e2e_s = time.perf_counter() - t0
        e2e_val = e2e_steps / e2e_s * (1 if tp else world)
        step_bytes = step_algorithmic_bytes(cfg, range(pos - args.steps, pos))
        model.close()

    peak, peak_kind = hbm_peak()
    gemv_ms = measure_gemv_roofline(fb, torch, pdl=True)
    gemv_ms_serial = measure_gemv_roofline(fb, torch, pdl=False)
    achieved = CONFIG0_BYTES / (gemv_ms * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
            p = synth_model(fb, args.config, tmp)
            cpu_decode_sample(p, 0.0, 1, threads)
            n, dt = cpu_decode_sample(p, 20.0, 64, threads)
        cpu = {"value": round(n / dt, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens of {args.config} at positions 0..{n - 1} through the oracle port "
                         f"(oracle/fence_oracle.c, fp64) on {threads} host threads, ~20 s"}
    launches_per_step = 1  # the persistent step kernel: one launch per token
    step_us = ms / args.steps * 1e3
    step_gbs = step_bytes / (step_us * 1e-6) / 1e9
    ratio = traffic_ratio_from_profiles(f"step_kernel_{args.config.replace('-', '_')}.md")
    step_traffic = int(ratio * step_bytes) if ratio else None
    line = {
        "metric": "decode_tokens_per_s", "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "int8xint16",
        "data": "synthetic (seeded random-init GGUF, config shapes)",
        "config": {"workload": f"{args.config} batch-1 greedy decode, {args.prompt} prompt tokens, positions "
                               f"{args.prompt + args.warmup}..{args.prompt + args.warmup + args.steps - 1}"
                               + (f" ({args.layers}-layer cut for profiling, not the config)" if args.layers else ""),
                   "model": args.config, "kv_cache": args.kv, "global_batch": world, "seq_len": total_pos,
                   "parallelism": f"tp{world}" if tp else (f"replicas{world}" if world > 1 else "single"),
                   "l2": "weights larger than L2 (no flush needed)"},
        "roofline": {"bound": "hbm", "kernel": "step_kernel (one launch = one whole token step)",
                     "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind,
                     "traffic": step_traffic, "us_per_launch": round(step_us, 2),
                     "algorithmic_bytes_per_launch": step_bytes},
        "gemv_config0": {"kernel": "drop-in gemv_q6k 4096x4096 (config 0), back-to-back launches in a CUDA graph",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": traffic_from_profiles("gemv_q6k_config0.md"),
                         "us_per_launch": round(gemv_ms * 1e3, 3),
                         "us_per_launch_serialized": round(gemv_ms_serial * 1e3, 3),
                         "algorithmic_bytes_per_launch": CONFIG0_BYTES},
        "e2e": {"value": round(e2e_val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 4},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
